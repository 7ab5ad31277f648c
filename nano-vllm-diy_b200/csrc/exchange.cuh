// Vocabulary-parallel token selection and the small cross-rank exchanges of
// the decode step (rows f2 / f3 of the hot path).
//
// Token selection (src/layers/sampler.py:4-17 and the greedy argmax):
//   the reference gathers every rank's [B, V/tp] logits to rank 0
//   (src/layers/llm_head.py:65-68), then samples
//     token = argmax_j softmax(l / T)_j / max(E_j, 1e-10),  E ~ Exp(1).
//   softmax's normaliser is the same for every j of a row, so this is
//     token = argmax_j (l_j / T - ln max(E_j, 1e-10))       (Gumbel-max)
//   and each rank can take the maximum of its own vocabulary shard: only a
//   (score, index) pair per row crosses NVLink instead of the logits.  Greedy
//   decoding is the same with score = l_j.  Ties go to the lowest index, as
//   torch.argmax does over the gathered row.
//   A row's best (score, index) is packed into one int64 "key" whose signed
//   order is the selection order: the high word is the score's bits mapped to
//   a monotone signed integer, the low word 0xFFFFFFFF - index.  The maximum
//   key over ranks is the selected token.
//   The Exp(1) draws come from the caller (a [B, V/tp] fp32 tensor, the
//   reference's `exponential_` draw) or from Philox-4x32-10 (Salmon, Moraes,
//   Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3", SC 2011) keyed
//   by (seed, row, global vocabulary index, offset), so a row's noise does not
//   depend on how the vocabulary is sharded.
//
// Exchanges over the fused all-reduce's symmetric buffers (NVLink peer
// stores, one signal round, bounded waits):
//   keys       every rank pushes its [B] keys into slot [rank] of every
//              rank's key area (parity = call epoch & 1), signals, waits for
//              the others and takes the maximum per row -> tokens on every
//              rank (src/layers/llm_head.py:65-68 + sampler.py:4-17 without
//              the logits gather);
//   embedding  each token's row lives in exactly one rank's vocabulary shard
//              (src/layers/llm_head.py:38-49: masked lookup + all_reduce sum,
//              every other rank contributing zeros), so the all-reduce is a
//              scatter: the owner writes the row into every rank's output;
//              rank 0 writes the zero rows of ids outside the vocabulary.
// Flags carry the call epoch (a device-side counter per exchange kind,
// advanced by every call on every rank), so they never need a reset.
#pragma once
#include "common.cuh"

namespace b200 {

constexpr int kXchgMaxRanks = 8;

// ---------------------------------------------------------------------------
// Philox-4x32-10 (counter-based; the round function and constants of the
// paper cited above)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
  constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;
  constexpr uint32_t kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(kM0, c.x), lo0 = kM0 * c.x;
    const uint32_t hi1 = __umulhi(kM1, c.z), lo1 = kM1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += kW0;
    k.y += kW1;
  }
  return c;
}

// uniform in (0, 1): the top 24 bits of x, centred in their interval
__device__ __forceinline__ float u01_open(uint32_t x) {
  return ((float)(x >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

// Monotone int64 key of (score, index): larger score first, then lower index.
__device__ __forceinline__ long long select_key(float v, uint32_t idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // unsigned order of the floats
  const uint32_t hi = u ^ 0x80000000u;              // ... as a signed word
  return (long long)(((unsigned long long)hi << 32) | (unsigned long long)(0xFFFFFFFFu - idx));
}
__device__ __forceinline__ long long key_to_token(long long key) {
  return (long long)(0xFFFFFFFFu - (uint32_t)((unsigned long long)key & 0xFFFFFFFFull));
}

struct SelectArgs {
  const __nv_bfloat16* logits;  // [rows][stride], this rank's V columns
  long long stride;
  int rows, V;
  long long vocab_start;        // global index of column 0
  const float* temperatures;    // [rows] or null (greedy)
  const float* noise;           // [rows][noise_stride] Exp(1) draws or null (Philox)
  long long noise_stride;
  unsigned long long seed, offset;
  long long* keys;              // [rows] out
};

// One CTA per row: the row's best (score, global index) as a key.
__global__ void __launch_bounds__(1024) token_select_kernel(const SelectArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ long long s_k[32];
  const int row = blockIdx.x;
  const __nv_bfloat16* lp = a.logits + (size_t)row * a.stride;
  const bool greedy = a.temperatures == nullptr;
  const float inv_t = greedy ? 1.f : 1.f / a.temperatures[row];
  const float* np = a.noise ? a.noise + (size_t)row * a.noise_stride : nullptr;
  const uint2 key = make_uint2((uint32_t)a.seed, (uint32_t)(a.seed >> 32));
  long long best = LLONG_MIN;
  // 4 consecutive columns per step (one Philox draw), global columns aligned
  // to 4 so the draw of a column is the same whatever the shard boundaries
  const long long g0 = a.vocab_start & ~3ll;
  const long long g_end = a.vocab_start + a.V;
  for (long long g = g0 + 4ll * threadIdx.x; g < g_end; g += 4ll * blockDim.x) {
    float e[4] = {1.f, 1.f, 1.f, 1.f};
    if (!greedy && np == nullptr) {
      const uint4 r = philox4x32_10(
          make_uint4((uint32_t)(g >> 2), (uint32_t)row, (uint32_t)a.offset, (uint32_t)(a.offset >> 32)),
          key);
      e[0] = -__logf(u01_open(r.x));
      e[1] = -__logf(u01_open(r.y));
      e[2] = -__logf(u01_open(r.z));
      e[3] = -__logf(u01_open(r.w));
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const long long gj = g + k;
      if (gj < a.vocab_start || gj >= g_end) continue;
      const int j = (int)(gj - a.vocab_start);
      float s = __bfloat162float(lp[j]);
      if (!greedy) {
        const float ek = np ? np[j] : e[k];
        s = s * inv_t - __logf(fmaxf(ek, 1e-10f));
      }
      const long long kk = select_key(s, (uint32_t)gj);
      best = kk > best ? kk : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long ok = __shfl_xor_sync(0xffffffffu, best, o);
    best = ok > best ? ok : best;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) s_k[warp] = best;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? s_k[lane] : LLONG_MIN;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const long long ok = __shfl_xor_sync(0xffffffffu, best, o);
      best = ok > best ? ok : best;
    }
    if (lane == 0) a.keys[row] = best;
  }
}

// System-scope flag helpers for the exchanges.
__device__ __forceinline__ unsigned xchg_ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void xchg_st_relaxed_sys(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Per-rank exchange state: every address is this rank's view of rank r's
// buffer (index r), this rank's own at index `rank`.
struct ExchangeArgs {
  int rank, world;
  long long* key_slots[kXchgMaxRanks];  // [2 parity][world][max_rows] int64
  unsigned* flags[kXchgMaxRanks];       // [kind][kXchgMaxRanks] epoch flags, one per source rank
  unsigned* state;                       // this rank's [kind] epochs, then [kind] CTA counters
  long long max_rows;
  unsigned* err;
};

// Signal every peer that this rank finished call `tag` of exchange `kind`,
// then wait (bounded) until every peer has signalled it.  One thread.
__device__ __forceinline__ bool xchg_signal_wait(const ExchangeArgs& x, int kind, unsigned tag) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int r = 0; r < x.world; ++r)
    if (r != x.rank) xchg_st_relaxed_sys(x.flags[r] + kind * kXchgMaxRanks + x.rank, tag);
  const unsigned long long t0 = globaltimer_ns();
  for (int r = 0; r < x.world; ++r) {
    if (r == x.rank) continue;
    const unsigned* f = x.flags[x.rank] + kind * kXchgMaxRanks + r;
    while ((int)(xchg_ld_acquire_sys(f) - tag) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_error(x.err, ERR_PEER_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}

// One CTA: push this rank's keys to every rank, one signal round, maximum
// over ranks per row -> tokens.  world == 1: tokens straight from the keys.
__global__ void __launch_bounds__(1024) keys_exchange_kernel(const long long* __restrict__ keys, int rows,
                                                             long long* __restrict__ tokens,
                                                             const ExchangeArgs x) {
  griddep_wait();
  griddep_launch_dependents();
  if (x.world == 1) {
    for (int i = threadIdx.x; i < rows; i += blockDim.x) tokens[i] = key_to_token(keys[i]);
    return;
  }
  __shared__ unsigned s_epoch;
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_epoch = x.state[0];
  __syncthreads();
  const unsigned tag = s_epoch + 1u;
  const size_t par = (size_t)(tag & 1u) * x.world * x.max_rows;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    const long long k = keys[i];
    for (int r = 0; r < x.world; ++r) x.key_slots[r][par + (size_t)x.rank * x.max_rows + i] = k;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    s_ok = xchg_signal_wait(x, 0, tag);
    x.state[0] = tag;
  }
  __syncthreads();
  const long long* mine = x.key_slots[x.rank] + par;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    long long best = keys[i];
    if (s_ok)
      for (int r = 0; r < x.world; ++r) {
        const long long k = __ldcv(mine + (size_t)r * x.max_rows + i);
        best = k > best ? k : best;
      }
    tokens[i] = key_to_token(best);
  }
}

// Output addresses of the embedding exchange (rank r's view of each rank's
// output rows), passed by value.
struct EmbeddingOuts {
  __nv_bfloat16* p[kXchgMaxRanks];
};

// Vocabulary-parallel embedding with its all-reduce as a scatter: rank r
// writes the rows of the ids in its shard [start, end) into out[dst] of every
// rank dst (rank 0 also the zero rows of ids outside [0, vocab)); the last
// CTA to finish signals the peers and waits until every rank's rows are in.
__global__ void __launch_bounds__(256) embedding_exchange_kernel(
    const long long* __restrict__ ids, const __nv_bfloat16* __restrict__ w, int T, int H,
    long long start, long long end, long long vocab, const EmbeddingOuts out, long long ld_out,
    const ExchangeArgs x) {
  griddep_wait();
  griddep_launch_dependents();
  const int vpr = H / 8;
  const long long total = (long long)T * vpr;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / vpr);
    const int c = (int)(i - (long long)t * vpr) * 8;
    const long long id = ids[t];
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    bool mine = false;
    if (id >= start && id < end) {
      v = *reinterpret_cast<const uint4*>(w + (size_t)(id - start) * H + c);
      mine = true;
    } else if (x.rank == 0 && (id < 0 || id >= vocab)) {
      mine = true;  // nobody owns it: its row is zero on every rank
    }
    if (mine)
      for (int r = 0; r < x.world; ++r)
        *reinterpret_cast<uint4*>(out.p[r] + (size_t)t * ld_out + c) = v;
  }
  __syncthreads();
  if (x.world == 1 || threadIdx.x != 0) return;
  // this CTA's stores, then the CTA counter; the last CTA signals
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  unsigned* counter = x.state + 2 + 1;
  if (atomicAdd(counter, 1u) != gridDim.x - 1) return;
  atomicExch(counter, 0u);
  const unsigned tag = x.state[1] + 1u;
  xchg_signal_wait(x, 1, tag);
  x.state[1] = tag;
}

}  // namespace b200
