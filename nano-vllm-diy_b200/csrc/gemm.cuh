// Y[T, N] = X[T, K] * W[N, K]^T  (+ bias) on 5th-generation tensor cores.
//
// This is the device side of the reference's F.linear calls
// (src/layers/linear.py:75 ColumnParallelLinear.forward, :170
// RowParallelLinear.forward, src/layers/llm_head.py:64 ParallelLMHead).
//
// Tiling ("swap-AB"): the weight is the M operand (128 output features per
// CTA) and the tokens are the N operand (BN = 32..128 tokens per CTA).  The
// grid runs token tiles fastest, so the CTAs that share a 128-row slab of W
// are resident together and W is read from HBM once (the siblings hit L2).  Both operands are
// K-major in global memory (W is [out, in] row-major, X is [T, in]), which is
// what the tcgen05 K-major shared-memory descriptors want.
//
// Two CTAs fit per SM (ring < 110 KB), so one CTA's epilogue overlaps the
// other's main loop.  Split-K runs inside a thread-block cluster of S CTAs
// (grid z = S): each CTA reduces a K range into TMEM, stages its fp32 tile in its
// own shared memory, and after a cluster barrier every CTA sums one slice of
// the tile's token rows over the S CTAs through distributed shared memory
// and writes it -- no fp32 workspace in HBM and no separate reduce kernel.
//
// Roles (192 threads):
//   warp 0      TMA producer (one lane): W box 64x128, X box 64xBN, 128-byte
//               swizzle, into an S-stage ring guarded by full/empty mbarriers
//   warp 1      TMEM allocator + MMA issuer (one lane): 4 x tcgen05.mma
//               (M=128, N=BN, K=16) per 64-wide K block, accumulators in TMEM
//   warps 2..5  TMEM -> shared memory (tcgen05.ld 32x32b), [token][feature]
//   all warps   cluster reduction + epilogue with 16-byte coalesced stores
//
// Epilogues:
//   EPI_BF16     y = bf16(acc + bias)
//   EPI_ALLREDUCE  RowParallelLinear at tp > 1, the all-reduce fused over
//                NVLink peer stores.  one-shot: every rank pushes its bf16
//                partial to every rank and sums its own copy.  two-shot: the
//                rows of each CTA position are split among the ranks' CTAs
//                of that position; each sums its rows from the world's
//                partials (fp32, fixed rank order) and stores them into
//                every rank's output.  Flag handshakes are bounded waits.
//   EPI_SILU     tiles hold 64 gate rows + the 64 matching up rows of the
//                [gate ; up] weight; y = bf16(silu(bf16 g) * bf16 u)
//                (src/layers/activation.py:6-10 fused into the gate_up GEMM)
#pragma once
#include "common.cuh"

namespace b200 {

enum GemmEpilogue : int { EPI_BF16 = 0, EPI_SILU = 2, EPI_ALLREDUCE = 3 };

constexpr int kMaxTpRanks = 8;

// Symmetric buffers of the fused GEMM + all-reduce (EPI_ALLREDUCE); index r
// holds rank r's address of each buffer (this rank's own entry included).
struct AllReducePeers {
  __nv_bfloat16* stage[kMaxTpRanks];  // two-shot: [world][rows][ldo]; one-shot: [2][world][rows][ldo]
  __nv_bfloat16* out[kMaxTpRanks];    // [stage_rows][ldo] reduced output
  unsigned* flags[kMaxTpRanks];       // two-shot: [positions]; one-shot: [2][positions]
  unsigned* done[kMaxTpRanks];        // two-shot: [positions]; one-shot: call counter + exit counter
  int rank, world, oneshot;
  long long stage_rows, ldo, positions;
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;
constexpr int kGemmMaxStages = 8;

struct GemmArgs {
  int T, N, K;         // tokens, output features (rows of W), reduction dim
  int BN;              // token tile (multiple of 32, <= 256)
  int stages;          // smem ring depth
  int num_kb;          // ceil(K / 64)
  int kb_per_split;    // K blocks per cluster rank
  int splits;          // cluster size along z
  int tmem_cols;       // power of two >= BN
  int epi;             // GemmEpilogue
  int vec_ok;          // y rows are 16-byte aligned: vector stores
  __nv_bfloat16* y;    // output
  long long ldy;       // row stride of y (elements)
  const __nv_bfloat16* bias;  // [N] or nullptr (EPI_BF16 only)
  int silu_inter;      // EPI_SILU: I (rows of W are [gate(I) ; up(I)])
  // split-K state of the persistent SM-pair kernel (both schedules)
  int tiles_m;         // 256-row weight tiles (pairs of 128-row CTA tiles)
  int tiles_t;         // token tiles of BN
  unsigned* sk_flags;  // [pairs * 2] partial-ready flags, then the grouped schedule's done
                       // counters at word kGrpDoneOffset (all zero between launches)
  float* sk_part;      // [pairs * 2][BN][128] fp32 partial tiles
  int use_tma_store;   // outputs written by TMA tensor stores (needs y 16-byte aligned, ldy % 8 == 0)
  // schedule of the SM-pair kernel: 0 stream-K over the flat (tile, K block)
  // units; 1 grouped: split tiles [0, grp_split) are shared by grp_size pairs
  // each (pair p < grp_split * grp_size takes K share p % grp_size of tile
  // p / grp_size first), then every pair takes grp_whole whole tiles
  // grp_split + p + j * pairs
  int sched;
  int grp_whole, grp_split, grp_size;
  int kstep;           // SM-pair kernel: 64-wide K blocks per ring stage (1 or 2)
  // RMSNorm (+ residual add) of the activations fused ahead of the GEMM
  // (SM-pair kernel with every CTA co-resident; gbar == nullptr: off): rows
  // [0, T) of nx (+ nres) are normalised by nw into nxo, the X operand's
  // rows; nres_out receives bf16(nx + nres).  Then a grid barrier, then the
  // activation loads.
  const __nv_bfloat16* nx;
  long long ldnx;
  const __nv_bfloat16* nres;   // nullptr: plain RMSNorm
  __nv_bfloat16* nres_out;
  const __nv_bfloat16* nw;
  float neps;
  __nv_bfloat16* nxo;
  long long ldnxo;
  unsigned* gbar;              // [2] arrivals, generation (zero-initialised workspace)
  int csplit;          // 2: cluster split-K (clusters of 2 pairs, one tile each, K halves
                       // reduced through distributed shared memory); 0: off
  unsigned* err;
  AllReducePeers ar;   // EPI_ALLREDUCE only
};

// System-scope flag helpers for the cross-GPU handshake.
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_relaxed_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// One system-scope fence (cumulative over the CTA's writes ordered by the
// preceding barrier), then a relaxed increment of every peer's flag: one
// fence per signal instead of one per peer.
__device__ __forceinline__ void signal_peers(unsigned* const* flags, size_t index, int rank, int world) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int r = 0; r < world; ++r)
    if (r != rank) red_relaxed_sys_add(flags[r] + index, 1u);
}
// Bounded wait until *p == want; resets *p to 0 afterwards (the flag is
// consumed).  Returns false and records ERR_PEER_TIMEOUT after 1 s.
__device__ __forceinline__ bool wait_flag_and_reset(unsigned* p, unsigned want, unsigned* err) {
  const unsigned long long t0 = globaltimer_ns();
  while (ld_acquire_sys(p) < want) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_error(err, ERR_PEER_TIMEOUT);
      return false;
    }
  }
  atomicExch(p, 0u);
  return true;
}

// bf16 rounding (to nearest even) of two floats by one packed conversion,
// unpacked with integer shifts: half the conversions of two bf16_round calls
// (conversions issue at a fraction of the FP32 rate and bound the SiLU
// epilogue otherwise).
__device__ __forceinline__ void bf16_round2(float& a, float& b) {
  const uint32_t w = pack_bf16x2(a, b);
  a = __uint_as_float(w << 16);
  b = __uint_as_float(w & 0xFFFF0000u);
}

// Eager semantics of src/layers/activation.py:9-10 on bf16 tensors, for two
// lanes: g and u are the GEMM outputs rounded to bf16, silu(g) is rounded to
// bf16, then multiplied by u.  The product is returned in g0 / g1 UNROUNDED:
// every caller stores it through a round-to-nearest bf16 conversion, which is
// the eager op's final rounding.  The sigmoid uses the hardware exp2 /
// reciprocal paths (__expf, __fdividef): their last-bit fp32 differences from
// expf and IEEE division disappear in the bf16 rounding except for rare
// one-ulp cases, and they are several times cheaper.
__device__ __forceinline__ void silu_mul2(float& g0, float& g1, float u0, float u1) {
  bf16_round2(g0, g1);
  bf16_round2(u0, u1);
  float s0 = __fdividef(g0, 1.0f + __expf(-g0));
  float s1 = __fdividef(g1, 1.0f + __expf(-g1));
  bf16_round2(s0, s1);
  g0 = __fmul_rn(s0, u0);
  g1 = __fmul_rn(s1, u1);
}

// Rows one all-reduce epilogue thread advances by (16 threads span a row).
constexpr int kArRowStep = kGemmThreads / 16;

__device__ __forceinline__ uint4 pack_bf16x8(const float (&v)[8]) {
  uint4 pk;
  pk.x = pack_bf16x2(v[0], v[1]); pk.y = pack_bf16x2(v[2], v[3]);
  pk.z = pack_bf16x2(v[4], v[5]); pk.w = pack_bf16x2(v[6], v[7]);
  return pk;
}

// The all-reduce's sum: for this thread's rows tr = r0, r0 + kArRowStep, ...
// < rows2, the W staged partials at src + tr ldo + r rstride (r = rank,
// ascending: the same fp32 sum on every rank) are added and `emit(tr, bf16
// x 8)` stores the result.  The W loads of G rows are in flight together.
template <int W, typename Emit>
__device__ __forceinline__ void ar_reduce_rows(const __nv_bfloat16* src, size_t rstride, long long ldo,
                                               int rows2, int r0, Emit& emit) {
  constexpr int G = W >= 8 ? 1 : 8 / W;
  for (int tr0 = r0; tr0 < rows2; tr0 += G * kArRowStep) {
    uint4 q[G][W];
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int tr = tr0 + j * kArRowStep;
      if (tr < rows2) {
        const __nv_bfloat16* s = src + (size_t)tr * ldo;
#pragma unroll
        for (int r = 0; r < W; ++r) q[j][r] = __ldcg(reinterpret_cast<const uint4*>(s + r * rstride));
      }
    }
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int tr = tr0 + j * kArRowStep;
      if (tr >= rows2) break;
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
      for (int r = 0; r < W; ++r) {
        const uint32_t* qw = reinterpret_cast<const uint32_t*>(&q[j][r]);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_bf16x2(qw[k]);
          acc[2 * k] += f.x;
          acc[2 * k + 1] += f.y;
        }
      }
      emit(tr, pack_bf16x8(acc));
    }
  }
}

// Epilogue shared by the GEMM kernels: this CTA's token rows [tb, te) of
// the tile at (token t0, feature n0 / SiLU tile ntile).  `sum8(off, v)`
// returns the 8 fp32 accumulators at float offset `off` of the [token][128]
// tile summed over the CTA's split-K group; `pos` / `nctas` identify the CTA
// position in the grid (same on every rank) for the all-reduce handshakes.
template <typename SumFn>
__device__ __forceinline__ void gemm_epilogue(const GemmArgs& p, SumFn& sum8, int t0, int n0,
                                              int ntile, int tb, int te, unsigned pos,
                                              unsigned nctas) {
  if (p.epi == EPI_SILU) {
    // 8 output features (8 gate + the 8 matching up rows) per unit
    const int units = (te - tb) * 8;
    for (int u = threadIdx.x; u < units; u += kGemmThreads) {
      const int t = tb + (u >> 3), ch = u & 7;
      const int feat = ntile * 64 + ch * 8;
      if (feat >= p.silu_inter) continue;
      float g[8], up[8], o[8];
      sum8(t * kGemmBM + ch * 8, g);
      sum8(t * kGemmBM + 64 + ch * 8, up);
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        o[i] = g[i];
        o[i + 1] = g[i + 1];
        silu_mul2(o[i], o[i + 1], up[i], up[i + 1]);
      }
      __nv_bfloat16* dst = p.y + (size_t)(t0 + t) * p.ldy + feat;
      if (p.vec_ok && feat + 8 <= p.silu_inter) {
        uint4 pk;
        pk.x = pack_bf16x2(o[0], o[1]); pk.y = pack_bf16x2(o[2], o[3]);
        pk.z = pack_bf16x2(o[4], o[5]); pk.w = pack_bf16x2(o[6], o[7]);
        *reinterpret_cast<uint4*>(dst) = pk;
      } else {
        for (int i = 0; i < 8 && feat + i < p.silu_inter; ++i) dst[i] = __float2bfloat16_rn(o[i]);
      }
    }
  } else if (p.epi == EPI_ALLREDUCE) {
    // ---- all-reduce over NVLink peer memory.  One-shot: every rank pushes
    // its bf16 partial of this CTA position into every rank's staging, then
    // sums the world's partials for its own copy; staging and flags alternate
    // between two halves by call parity (a device-side call counter), so a
    // rank one call ahead never overwrites data still being read.  Two-shot:
    // the position's token rows are cut into `world` sub-slices and rank r's
    // CTA reduces sub-slice r: push sub-slice s of this rank's partial to
    // rank s; when the world's partials of sub-slice `rank` are in, sum them
    // and store the result into every rank's output; then wait until the
    // other sub-slices have arrived here, so the kernel's completion means
    // the output is complete.
    // Every thread keeps one 8-feature chunk (16 threads span the tile's 128
    // features) and walks the rows kArRowStep apart, with its addresses and
    // bias computed once: the epilogue runs on the CTA's 6 warps, and its
    // instruction count more than its bytes sets its time.
    const AllReducePeers& ar = p.ar;
    const bool one = ar.oneshot != 0;
    unsigned* calls = ar.done[ar.rank];
    const unsigned parity = one ? (__ldcg(calls) & 1u) : 0u;
    const size_t half = one ? (size_t)ar.world * ar.stage_rows * ar.ldo : 0;
    const int rows = te - tb;
    const int sub = (rows + ar.world - 1) / ar.world;
    const int ch = threadIdx.x & 15;
    const int n = n0 + ch * 8;
    const bool n_ok = n < p.N;
    const int r0 = threadIdx.x >> 4;
    float bias8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      bias8[i] = (p.bias != nullptr && n + i < p.N) ? __bfloat162float(p.bias[n + i]) : 0.f;
    // phase 1: this rank's partial rows [tb, te) -> the staging of every rank
    // (one-shot) or of the rank reducing the row (two-shot); the split-K sums
    // of four rows are formed before their stores
    const size_t off1 = parity * half + ((size_t)ar.rank * ar.stage_rows + t0 + tb) * ar.ldo + n;
    constexpr int kPushBatch = 4;
    for (int tr0 = r0; tr0 < rows; tr0 += kPushBatch * kArRowStep) {
      uint4 pk[kPushBatch];
#pragma unroll
      for (int j = 0; j < kPushBatch; ++j) {
        const int tr = tr0 + j * kArRowStep;
        if (tr < rows && n_ok) {
          float v[8];
          sum8((tb + tr) * kGemmBM + ch * 8, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] += bias8[i];
          pk[j] = pack_bf16x8(v);
        }
      }
#pragma unroll
      for (int j = 0; j < kPushBatch; ++j) {
        const int tr = tr0 + j * kArRowStep;
        if (tr >= rows || !n_ok) continue;
        const size_t off = off1 + (size_t)tr * ar.ldo;
        if (one) {
          for (int r = 0; r < ar.world; ++r) *reinterpret_cast<uint4*>(ar.stage[r] + off) = pk[j];
        } else {
          *reinterpret_cast<uint4*>(ar.stage[tr / sub] + off) = pk[j];
        }
      }
    }
    __syncthreads();
    __shared__ int s_ok;
    const size_t fbase = parity * (size_t)ar.positions;
    if (threadIdx.x == 0) {
      signal_peers(ar.flags, fbase + pos, ar.rank, ar.world);
      s_ok = ar.world == 1 ||
             wait_flag_and_reset(ar.flags[ar.rank] + fbase + pos, (unsigned)(ar.world - 1), p.err);
    }
    __syncthreads();
    // phase 2: the rows this CTA reduces -- all of them (one-shot) or
    // sub-slice `rank` (two-shot) -- summed over the world in rank order
    const int mb = one ? tb : tb + ar.rank * sub;
    const int me = one ? te : min(te, mb + sub);
    const int rows2 = max(0, me - mb);
    const __nv_bfloat16* src2 = ar.stage[ar.rank] + parity * half + (size_t)(t0 + mb) * ar.ldo + n;
    const size_t rstride = (size_t)ar.stage_rows * ar.ldo;
    const size_t off2 = (size_t)(t0 + mb) * ar.ldo + n;
    auto emit = [&](int tr, const uint4& pk) {
      const size_t off = off2 + (size_t)tr * ar.ldo;
      if (one) {
        *reinterpret_cast<uint4*>(ar.out[ar.rank] + off) = pk;
      } else {
        for (int r = 0; r < ar.world; ++r) *reinterpret_cast<uint4*>(ar.out[r] + off) = pk;
      }
    };
    if (s_ok && n_ok) {
      switch (ar.world) {
        case 1: ar_reduce_rows<1>(src2, rstride, ar.ldo, rows2, r0, emit); break;
        case 2: ar_reduce_rows<2>(src2, rstride, ar.ldo, rows2, r0, emit); break;
        case 3: ar_reduce_rows<3>(src2, rstride, ar.ldo, rows2, r0, emit); break;
        case 4: ar_reduce_rows<4>(src2, rstride, ar.ldo, rows2, r0, emit); break;
        case 5: ar_reduce_rows<5>(src2, rstride, ar.ldo, rows2, r0, emit); break;
        case 6: ar_reduce_rows<6>(src2, rstride, ar.ldo, rows2, r0, emit); break;
        case 7: ar_reduce_rows<7>(src2, rstride, ar.ldo, rows2, r0, emit); break;
        default: ar_reduce_rows<8>(src2, rstride, ar.ldo, rows2, r0, emit); break;
      }
    }
    __syncthreads();
    if (one) {
      // the last CTA to finish advances the call counter (every rank runs the
      // same calls, so the counters stay equal)
      if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(calls + 1, 1u) == nctas - 1) {
          atomicExch(calls + 1, 0u);
          atomicAdd(calls, 1u);
        }
      }
    } else if (threadIdx.x == 0) {
      signal_peers(ar.done, pos, ar.rank, ar.world);
      wait_flag_and_reset(ar.done[ar.rank] + pos, (unsigned)(ar.world - 1), p.err);
    }
    __syncthreads();
  } else {
    const int units = (te - tb) * 16;
    for (int u = threadIdx.x; u < units; u += kGemmThreads) {
      const int t = tb + (u >> 4), ch = u & 15;
      const int n = n0 + ch * 8;
      if (n >= p.N) continue;
      float v[8];
      sum8(t * kGemmBM + ch * 8, v);
      if (p.bias != nullptr) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (n + i < p.N) v[i] += __bfloat162float(p.bias[n + i]);
      }
      __nv_bfloat16* dst = p.y + (size_t)(t0 + t) * p.ldy + n;
      if (p.vec_ok && n + 8 <= p.N) {
        uint4 pk;
        pk.x = pack_bf16x2(v[0], v[1]); pk.y = pack_bf16x2(v[2], v[3]);
        pk.z = pack_bf16x2(v[4], v[5]); pk.w = pack_bf16x2(v[6], v[7]);
        *reinterpret_cast<uint4*>(dst) = pk;
      } else {
        for (int i = 0; i < 8 && n + i < p.N; ++i) dst[i] = __float2bfloat16_rn(v[i]);
      }
    }
  }
}

__global__ void __launch_bounds__(kGemmThreads, 2)
    gemm_tn_tcgen05_kernel(const __grid_constant__ CUtensorMap tmW,
                           const __grid_constant__ CUtensorMap tmX, const GemmArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int S = p.stages;
  constexpr uint32_t kABytes = kGemmBM * kGemmBK * 2;  // 16 KiB
  const uint32_t b_bytes = (uint32_t)p.BN * kGemmBK * 2;
  uint8_t* a_smem = smem;
  uint8_t* b_smem = smem + (size_t)S * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(b_smem + (size_t)S * b_bytes);
  uint64_t* empty = full + kGemmMaxStages;
  uint64_t* tmem_full = empty + kGemmMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full + 1);
  // after the main loop the ring is reused as the fp32 tile [BN][128]
  float* s_tile = reinterpret_cast<float*>(smem);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ntile = blockIdx.y;          // feature tile (EPI_SILU: gate rows 64*ntile)
  const int n0 = ntile * kGemmBM;
  const int t0 = blockIdx.x * p.BN;
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
  const int nk = max(0, kb1 - kb0);
  const int rot = nk > 0 ? (int)((blockIdx.y * 7u + blockIdx.x * 3u) % (unsigned)nk) : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(tmem_full, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // everything above overlaps the previous kernel's tail (programmatic
  // dependent launch), and so do the producer's weight loads for the first
  // ring stages (weights are parameters; no kernel of the step writes them);
  // activations, outputs and peer buffers are touched only after the wait
  const bool producer = warp == 0 && lane == 0;
  if (!producer) {
    griddep_wait();
    griddep_launch_dependents();
  }

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      auto load_w = [&](int i) {
        const int s = i % S;
        // rotated K order: concurrently running CTAs read different X blocks
        const int kc = (kb0 + (i + rot) % nk) * kGemmBK;
        if (p.epi == EPI_SILU) {
          const int g0 = ntile * 64;
          tma_load_2d(a_smem + (size_t)s * kABytes, &tmW, &full[s], kc, g0);
          tma_load_2d(a_smem + (size_t)s * kABytes + kABytes / 2, &tmW, &full[s], kc,
                      p.silu_inter + g0);
        } else {
          tma_load_2d(a_smem + (size_t)s * kABytes, &tmW, &full[s], kc, n0);
        }
      };
      auto load_x = [&](int i) {
        const int s = i % S;
        tma_load_2d(b_smem + (size_t)s * b_bytes, &tmX, &full[s], (kb0 + (i + rot) % nk) * kGemmBK, t0);
      };
      // the first pass over the ring needs no empty wait: weights first, then
      // (after the previous kernel) the activations of those stages
      const int pre = min(S, nk);
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], kABytes + b_bytes);
        load_w(i);
      }
      griddep_wait();
      griddep_launch_dependents();
      for (int i = 0; i < pre; ++i) load_x(i);
      issued = pre;
      for (int i = pre; i < nk; ++i) {
        const int s = i % S;
        const uint32_t ph = (uint32_t)(i / S) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, p.err)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], kABytes + b_bytes);
        load_w(i);
        load_x(i);
        ++issued;
      }
      if (!ok) {
        // drain the copies still in flight before the CTA can exit
        for (int j = max(0, issued - S); j < issued; ++j)
          mbar_wait(&full[j % S], (uint32_t)(j / S) & 1u, p.err);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(kGemmBM, p.BN);
      for (int i = 0; i < nk; ++i) {
        const int s = i % S;
        const uint32_t ph = (uint32_t)(i / S) & 1u;
        if (!mbar_wait(&full[s], ph, p.err)) break;
        tc_fence_after();
        const uint32_t a_base = smem_u32(a_smem + (size_t)s * kABytes);
        const uint32_t b_base = smem_u32(b_smem + (size_t)s * b_bytes);
#pragma unroll
        for (int kk = 0; kk < kGemmBK / 16; ++kk) {
          tc_mma_f16(tmem_base, umma_desc_sw128(a_base + kk * 32),
                     umma_desc_sw128(b_base + kk * 32), idesc, (i | kk) != 0 ? 1u : 0u);
        }
        tc_commit(&empty[s]);
      }
      tc_commit(tmem_full);
      // every MMA this thread issued has finished before TMEM can be freed
      mbar_wait(tmem_full, 0, p.err);
    }
  } else {
    // ---- TMEM -> shared memory: warps 2..5 own TMEM lane quarters 2,3,0,1
    const int q = warp & 3;
    const int row = q * 32 + lane;  // accumulator row = feature inside the tile
    const bool have = mbar_wait(tmem_full, 0, p.err);
    tc_fence_after();
    for (int c = 0; c < p.BN; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)c, r);
      tmem_ld_wait();
      if (have && nk > 0) {
#pragma unroll
        for (int j = 0; j < 32; ++j) s_tile[(c + j) * kGemmBM + row] = __uint_as_float(r[j]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) s_tile[(c + j) * kGemmBM + row] = 0.f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, (uint32_t)p.tmem_cols);
  }
  const int splits = p.splits;
  if (splits > 1) cluster_sync();

  // ---- reduction over the cluster + epilogue: this CTA's slice of token rows
  const uint32_t rank = splits > 1 ? cluster_ctarank() : 0u;
  const int rows_valid = min(p.BN, p.T - t0);
  const int per = (rows_valid + splits - 1) / splits;
  const int tb = min(rows_valid, (int)rank * per);
  const int te = min(rows_valid, tb + per);
  const uint32_t tile_local = smem_u32(s_tile);
  // the cluster ranks' tiles (splits <= 8), mapped once
  uint32_t rank_tile[8];
#pragma unroll
  for (int r = 0; r < 8; ++r)
    rank_tile[r] = (r < splits && splits > 1) ? map_to_rank(tile_local, (uint32_t)r) : tile_local;
  // 8 fp32 partials summed over the cluster ranks in rank order, the loads of
  // four ranks in flight together
  auto sum8 = [&](int off_floats, float* v) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
#pragma unroll
    for (int g = 0; g < 8; g += 4) {
      if (g < splits) {
        float4 x[8];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          if (g + r < splits) {
            const uint32_t a = rank_tile[g + r] + (uint32_t)off_floats * 4u;
            x[2 * r] = ld_dsmem_f4(a);
            x[2 * r + 1] = ld_dsmem_f4(a + 16);
          }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          if (g + r < splits) {
            v[0] += x[2 * r].x; v[1] += x[2 * r].y; v[2] += x[2 * r].z; v[3] += x[2 * r].w;
            v[4] += x[2 * r + 1].x; v[5] += x[2 * r + 1].y; v[6] += x[2 * r + 1].z; v[7] += x[2 * r + 1].w;
          }
        }
      }
    }
  };
  const unsigned pos = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  gemm_epilogue(p, sum8, t0, n0, ntile, tb, te, pos, gridDim.x * gridDim.y * gridDim.z);
  // peers may still be reading this CTA's tile
  if (splits > 1) cluster_sync();
}

}  // namespace b200
