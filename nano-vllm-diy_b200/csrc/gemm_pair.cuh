// Y[T, N] = X[T, K] * W[N, K]^T on SM pairs: tcgen05.mma.cta_group::2.
//
// Two CTAs on the two SMs of a cluster issue one M = 256 MMA together: each
// stages its own 128 token rows (A) and half of the pair's NP weight rows
// (B); the MMA reads A from both CTAs and B from both halves, and each CTA's
// TMEM receives its own 128 tokens x NP columns of the accumulator.  Per
// 64-wide K block an SM ingests 32 KB for 128 x 256 x 64 MACs, half the
// token bytes per weight byte of the single-SM kernel.
//
// Pair protocol (per 64-wide K block, stage s):
//   both producers  wait own empty[s]; the leader arms its full[s] with the
//                   bytes of both CTAs; both issue their TMA loads with
//                   .cta_group::2, completing on the LEADER's full[s]
//   leader MMA      waits full[s], issues 4 x (M=256, N=NP, K=16), then
//                   commits to empty[s] of both CTAs (two commits addressed
//                   through mapa), and after a tile to acc_full of both CTAs
//   both epilogues  wait own acc_full, read their TMEM lanes, release the
//                   accumulator to the leader's acc_empty
// Every wait is bounded (kWaitLimitNs) and records an error bit.
#pragma once
#include "gemm.cuh"

namespace b200 {

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D[tmem] (+)= A * B^T over the CTA pair (issued by the leader only).
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at a shared::cluster address (this CTA's or the
// peer's) once the pair MMAs issued so far by this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          bar_cluster_addr)
      : "memory");
}
// 2-D tiled load into this CTA's shared memory whose completion is counted on
// an mbarrier of the pair (given by its shared::cluster address).  Same
// 16-byte rule on c0 as tma_load_2d (callers pass multiples of 64 elements).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t smem_dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster_addr, int32_t c0,
                                                 int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
      : "memory");
}

// mbarrier arrive on a barrier given by its shared::cluster address (this
// CTA's or the pair peer's), release at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                   bar_cluster_addr)
               : "memory");
}
__device__ __forceinline__ void epi_bar_sync() {  // the 4 epilogue warps
  asm volatile("bar.sync 1, 128;" ::: "memory");
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Contiguous global -> shared copy by the bulk-copy engine, completing
// `bytes` on the mbarrier (addresses 16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t smem_dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_dst),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled store shared -> global by the TMA engine (clipped at the tensor
// bounds), tracked by bulk async-groups.  c0 * element size must be a
// multiple of 16 bytes and neither coordinate negative.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t smem_src, int32_t c0,
                                             int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_src), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N bulk groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_group_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// tcgen05.wait::ld that the compiler sees as producing `r`: uses of the
// registers of an asynchronous TMEM load cannot move above the wait.
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
        "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
        "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
        "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

// Stream-K range of pair `pr` of `pairs` over `total` K-block units.
__device__ __forceinline__ long long sk_begin(long long total, int pr, int pairs) {
  return total * pr / pairs;
}

// ---------------------------------------------------------------------------
// Persistent SM-pair GEMM with a grouped split-K or a stream-K schedule.
//
// Operand roles: the TOKENS are the M = 256 operand (128 per CTA of the pair,
// TMEM lane = token) and the weight rows the N operand (the pair's NP
// features, NP/2 staged by each CTA), so each epilogue thread owns one token
// row and writes contiguous output features straight from its registers;
// for the gate_up projection a tile's columns are [128 gate | the 128
// matching up rows], so SiLU-and-mul needs no exchange between threads.
//
// grid = 2 x pairs CTAs (all co-resident), cluster (2, 1, 1); tile =
// (feature tile m, token tile t) with t fastest (tiles sharing weights run
// back to back).
//
// Stream-K schedule (p.sched = 0): the work is the flat sequence of (tile, K
// block) units; pair p takes units [total p / P, total (p+1) / P).  A range
// cuts tiles into segments:
//   whole        all K blocks of a tile       -> epilogue writes the output
//   contributor  first segment of a range that starts inside a tile (its
//                tail K blocks)               -> fp32 partial to sk_part[p],
//                                                flag sk_flags[p] = 1
//   finisher     last segment of a range that ends inside a tile (its head
//                K blocks)                    -> waits for the flags of the
//                pairs p+1.. whose ranges start inside the tile, adds their
//                partials, writes the output, resets those flags to 0
// Contributions are the first thing a pair computes and finishes are the
// last, so a finisher never waits on work queued behind a wait.
// TMEM holds two accumulators (2 x NP columns): the MMA issuer fills one
// while the epilogue warps drain the other.
//
// Grouped schedule (p.sched = 1; the default whenever it balances): with P
// pairs and n tiles, w = n / P whole tiles per pair and r = n % P split
// tiles, each shared by a group of g = min(8, P / r, K blocks) pairs.  Pair
// p < r g first computes K share p % g of split tile p / g, then whole tiles
// r + p + j P (j < w).  Every member of a group owns the 32-wide output
// chunks m, m + g, ... (SiLU: gate / up chunk pairs): it writes the chunks
// the other members own to its partial slot, raises its flag, waits for the
// flags of the members whose chunks it owns (all pairs are co-resident and
// the members start together), then sums its own chunks from TMEM and the
// members' partials and writes them.  The reduction is spread over all
// members, and for w >= 1 it overlaps the MMAs of the next whole tile.  The
// last member to finish resets the group's flags for the next launch.
//
// Cluster split-K (p.csplit = C in 2..4; plain epilogue only): clusters of
// 2C CTAs = C pairs and one tile per cluster; member m = cluster rank / 2
// computes K blocks [m nkb / C, (m + 1) nkb / C).  Member m owns the 32-wide
// output chunks c with c % C == m.  After a cluster barrier (every ring of the
// cluster is idle) each CTA pushes the chunks other members own from TMEM
// straight into the owner's stage ring (st.async, counted on the owner's
// mbarrier; slot (c / C) (C - 1) + the sender's index among the owner's
// peers), then sums its own chunks from TMEM and the pushed partials (members
// in rank order) and writes them: no L2 round trip and no flags.
// ---------------------------------------------------------------------------

// One segment of a pair's work: K blocks [kbb, kbe) of `tile`; `member` is
// the pair's index in the tile's group under the grouped schedule (-1 for
// whole tiles and stream-K segments).
struct PairSeg {
  long long tile;
  int kbb, kbe, member;
};

// The segments of pair `pr` of `pairs` in order, walked identically by the
// producer, the MMA issuer and the epilogue (and by the host-side coverage
// check).  State: `u` (stream-K: next unit, starts at the pair's first unit)
// and `k` (grouped: segments taken, starts at 0).
__host__ __device__ inline bool pair_next_seg(int sched, long long tiles, int num_kb, int grp_whole,
                                              int grp_split, int grp_size, int pr, int pairs,
                                              long long& u, long long u_end, int& k, PairSeg& s) {
  if (sched == 0) {
    if (u >= u_end) return false;
    s.tile = u / num_kb;
    s.kbb = (int)(u - s.tile * num_kb);
    const long long left = u_end - u;
    s.kbe = left < (long long)(num_kb - s.kbb) ? s.kbb + (int)left : num_kb;
    s.member = -1;
    u += s.kbe - s.kbb;
    return true;
  }
  int j = k;
  if (grp_size > 0 && pr < grp_split * grp_size) {
    if (j == 0) {
      const int m = pr % grp_size;
      s.tile = pr / grp_size;
      s.kbb = (int)((long long)m * num_kb / grp_size);
      s.kbe = (int)((long long)(m + 1) * num_kb / grp_size);
      s.member = m;
      ++k;
      return true;
    }
    --j;
  }
  if (j >= grp_whole) return false;
  s.tile = grp_split + pr + (long long)j * pairs;
  if (s.tile >= tiles) return false;
  s.kbb = 0;
  s.kbe = num_kb;
  s.member = -1;
  ++k;
  return true;
}

// Word offset of the grouped schedule's per-(split tile, CTA half) done
// counters in the flag area (the partial-ready flags use words [0, 2 pairs)).
constexpr int kGrpDoneOffset = 512;

// One row of the fused RMSNorm prologue (GemmArgs::gbar) on the 128
// epilogue threads `et`: s = x (+ res) in fp32, res_out = bf16(s), out =
// bf16(w * (s * 1/sqrt(mean(s^2) + eps))) -- the rounding points of
// rms_norm_kernel (src/layers/layernorm.py:10-28).  Two passes over the row
// (sum of squares, then the outputs) keep the registers of the GEMM's
// epilogue free; `s_red` holds the 4 warps' partial sums.
__device__ __forceinline__ void norm_row_128(const GemmArgs& p, int row, int et, float* s_red) {
  const int nvec = p.K >> 3;
  const __nv_bfloat16* xr = p.nx + (size_t)row * p.ldnx;
  const __nv_bfloat16* rr = p.nres != nullptr ? p.nres + (size_t)row * p.K : nullptr;
  auto load_sum = [&](int vi, float (&sv)[8]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(xr + vi * 8);
    const uint32_t* rw = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = unpack_bf16x2(rw[k]);
      sv[2 * k] = f.x;
      sv[2 * k + 1] = f.y;
    }
    if (rr != nullptr) {
      const uint4 rv = *reinterpret_cast<const uint4*>(rr + vi * 8);
      const uint32_t* rp = reinterpret_cast<const uint32_t*>(&rv);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(rp[k]);
        sv[2 * k] = __fadd_rn(sv[2 * k], f.x);
        sv[2 * k + 1] = __fadd_rn(sv[2 * k + 1], f.y);
      }
    }
  };
  float ss = 0.f;
  for (int vi = et; vi < nvec; vi += 128) {
    float sv[8];
    load_sum(vi, sv);
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += sv[k] * sv[k];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((et & 31) == 0) s_red[et >> 5] = ss;
  epi_bar_sync();
  const float tot = ((s_red[0] + s_red[1]) + s_red[2]) + s_red[3];
  const float inv = 1.0f / sqrtf(__fadd_rn(tot / (float)p.K, p.neps));
  for (int vi = et; vi < nvec; vi += 128) {
    float sv[8];
    load_sum(vi, sv);
    const uint4 wv = *reinterpret_cast<const uint4*>(p.nw + vi * 8);
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(&wv);
    uint4 o, so;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
    uint32_t* sp = reinterpret_cast<uint32_t*>(&so);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 wf = unpack_bf16x2(wp[k]);
      op[k] = pack_bf16x2(__fmul_rn(wf.x, __fmul_rn(sv[2 * k], inv)), __fmul_rn(wf.y, __fmul_rn(sv[2 * k + 1], inv)));
      sp[k] = pack_bf16x2(sv[2 * k], sv[2 * k + 1]);
    }
    if (rr != nullptr) *reinterpret_cast<uint4*>(p.nres_out + (size_t)row * p.K + vi * 8) = so;
    *reinterpret_cast<uint4*>(p.nxo + (size_t)row * p.ldnxo + vi * 8) = o;
  }
  epi_bar_sync();  // s_red is reused by the next row
}

// Grid-wide barrier of a launch whose CTAs are all co-resident: gbar[0]
// counts arrivals, gbar[1] is a generation number; the last CTA to arrive
// resets the count and advances the generation.  Bounded (kWaitLimitNs).
__device__ __forceinline__ bool grid_barrier(unsigned* gbar, unsigned nctas, unsigned* err) {
  const unsigned gen = ld_acquire_gpu(gbar + 1);
  __threadfence();
  if (atomicAdd(gbar, 1u) == nctas - 1u) {
    atomicExch(gbar, 0u);
    __threadfence();
    st_release_gpu(gbar + 1, gen + 1u);
    return true;
  }
  const unsigned long long t0 = globaltimer_ns();
  while (ld_acquire_gpu(gbar + 1) == gen) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_error(err, ERR_PEER_TIMEOUT);
      return false;
    }
  }
  return true;
}

// Partial tiles are [NP/32 chunks] of 16 KiB, each [8][128 tokens][4
// features] fp32: a thread's 32 columns of a chunk are 8 float4 at stride
// 2 KiB, so a warp's accesses are 512 contiguous bytes.  A finisher streams
// them through up to kFixSlots 16 KiB slots of the (by then idle) stage ring.
constexpr int kFixSlots = 12;
constexpr int kChunkFloats = 32 * kGemmBM;

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_pair_tcgen05_kernel(const __grid_constant__ CUtensorMap tmW,
                             const __grid_constant__ CUtensorMap tmX,
                             const __grid_constant__ CUtensorMap tmY, const GemmArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int S = p.stages;
  const bool silu = p.epi == EPI_SILU;
  constexpr uint32_t kABytes = kGemmBM * kGemmBK * 2;  // 16 KiB: 128 tokens
  const int NP = p.BN;                                  // the pair's tile columns
  const uint32_t b_bytes = (uint32_t)(NP / 2) * kGemmBK * 2;
  // a ring stage holds KS consecutive 64-wide K blocks (one TMA box per
  // block and operand); the MMA issuer waits once per stage
  const int KS = p.kstep >= 2 ? 2 : 1;
  const uint32_t a_stage = (uint32_t)KS * kABytes, b_stage = (uint32_t)KS * b_bytes;
  uint8_t* a_smem = smem;
  uint8_t* b_smem = smem + (size_t)S * a_stage;
  // output staging for the TMA stores: 4 x [128 tokens][32 features] bf16,
  // 64-byte rows with the 64-byte swizzle (16-byte chunk c of row r at
  // chunk c ^ ((r >> 1) & 3)), 1 KiB aligned
  uint8_t* stage_out = b_smem + (size_t)S * b_stage;
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_out + 4 * kGemmBM * 64);
  uint64_t* empty = full + kGemmMaxStages;
  uint64_t* acc_full = empty + kGemmMaxStages;   // [2] per CTA
  uint64_t* acc_empty = acc_full + 2;            // [2] used in the leader
  uint64_t* fix_bar = acc_empty + 2;             // [kFixSlots] stream-K partial loads
  uint64_t* norm_bar = fix_bar + kFixSlots;      // fused RMSNorm rows of this CTA written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(norm_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const uint32_t v = crank & 1u;  // 0: leader (issues the MMAs), 1: peer
  const uint32_t leader = crank & ~1u;
  const int pr = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;
  const long long tiles = (long long)p.tiles_m * p.tiles_t;
  const long long total = tiles * p.num_kb;
  const int C = p.csplit;              // cluster split-K: pairs per tile (0: off)
  const bool csk = C >= 2;
  const int cmem = (int)(crank >> 1);  // cluster split-K: member index (0 .. C - 1)
  // stream-K: this pair's units (unused by the grouped schedule); cluster
  // split-K: this member's share of the cluster's tile (one segment)
  long long u_begin, u_end;
  if (csk) {
    const long long t0 = (long long)(blockIdx.x / (2 * C)) * p.num_kb;
    u_begin = t0 + (long long)cmem * p.num_kb / C;
    u_end = t0 + (long long)(cmem + 1) * p.num_kb / C;
  } else {
    u_begin = sk_begin(total, pr, pairs);
    u_end = sk_begin(total, pr + 1, pairs);
  }
  auto next_seg = [&](long long& u, int& k, PairSeg& sg) {
    return pair_next_seg(p.sched, tiles, p.num_kb, p.grp_whole, p.grp_split, p.grp_size, pr, pairs, u,
                         u_end, k, sg);
  };
  const uint32_t acc_stride = (uint32_t)p.tmem_cols / 2;  // columns per accumulator
  // output features of a tile: NP (plain) or the 128 gate rows (SiLU)
  const int tile_feats = silu ? 128 : NP;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
    mbar_init(&acc_empty[0], 2);  // one release from each CTA's epilogue
    mbar_init(&acc_empty[1], 2);
    for (int i = 0; i < kFixSlots; ++i) mbar_init(&fix_bar[i], 1);
    mbar_init(norm_bar, 128);  // the epilogue threads
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
    if (p.use_tma_store) tma_prefetch_desc(&tmY);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, (uint32_t)p.tmem_cols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised before either signals the other
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // everything above overlaps the previous kernel's tail (programmatic
  // dependent launch), and so do the producer's weight loads for the first
  // ring stages (weights are parameters; no kernel of the step writes them);
  // activations, outputs and the split-K workspace are touched only after
  // the wait
  const bool producer = warp == 0 && lane == 0;
  if (!producer) {
    griddep_wait();
    griddep_launch_dependents();
  }

  if (warp == 0) {
    // ---- producer (both CTAs): this CTA's 128 tokens and NP/2 weight rows
    if (lane == 0) {
      const uint32_t full_leader = map_to_rank(smem_u32(full), leader);
      auto weight_row = [&](long long tile) {
        // plain: features mt*NP + v*NP/2; SiLU: gate rows (leader) or the
        // matching up rows (peer) of features mt*128
        const int mt = (int)(tile / p.tiles_t);
        return silu ? (int)v * p.silu_inter + mt * 128 : mt * NP + (int)v * (NP / 2);
      };
      int it = 0;
      bool ok = true;
      long long su = u_begin;
      int sk = 0;
      PairSeg sg;
      // the first pass over the ring needs no empty wait: the first
      // segment's weights first, the activations of those stages after the
      // previous kernel
      int pre = 0;
      {
        long long su0 = u_begin;
        int sk0 = 0;
        PairSeg s0;
        if (next_seg(su0, sk0, s0)) {
          const int wrow = weight_row(s0.tile);
          pre = min(S, (s0.kbe - s0.kbb + KS - 1) / KS);
          for (int j = 0; j < pre; ++j) {
            const int kb = s0.kbb + j * KS, nb = min(KS, s0.kbe - kb);
            if (v == 0) mbar_arrive_expect_tx(&full[j], 2u * (uint32_t)nb * (kABytes + b_bytes));
            for (int h = 0; h < nb; ++h)
              tma_load_2d_pair(smem_u32(b_smem + (size_t)j * b_stage + (size_t)h * b_bytes), &tmW,
                               full_leader + (uint32_t)j * 8u, (kb + h) * kGemmBK, wrow);
          }
        }
      }
      griddep_wait();
      griddep_launch_dependents();
      if (p.gbar != nullptr) {
        // fused RMSNorm: this CTA's rows are written (the epilogue threads
        // arrive after their stores); publish them and wait for every CTA's
        // before the first activation load.  A timeout is recorded and the
        // loads go ahead (the results are then flagged, never a hang).
        mbar_wait(norm_bar, 0u, p.err);
        grid_barrier(p.gbar, gridDim.x, p.err);
        fence_proxy_async_global();
      }
      while (ok && next_seg(su, sk, sg)) {
        const int kbb = sg.kbb, kbe = sg.kbe;
        const int mt = (int)(sg.tile / p.tiles_t);
        const int tt = (int)(sg.tile - (long long)mt * p.tiles_t);
        const int tok = tt * 2 * kGemmBM + (int)v * kGemmBM;
        const int wrow = weight_row(sg.tile);
        for (int kb = kbb; kb < kbe; kb += KS, ++it) {
          const int s = it % S;
          const uint32_t ph = (uint32_t)(it / S) & 1u;
          const int nb = min(KS, kbe - kb);
          const uint32_t bar = full_leader + (uint32_t)s * 8u;
          if (it < pre) {  // weights already in flight: the activations now
            for (int h = 0; h < nb; ++h)
              tma_load_2d_pair(smem_u32(a_smem + (size_t)s * a_stage + (size_t)h * kABytes), &tmX, bar,
                               (kb + h) * kGemmBK, tok);
            continue;
          }
          if (!mbar_wait(&empty[s], ph ^ 1u, p.err)) {
            ok = false;
            break;
          }
          if (v == 0) mbar_arrive_expect_tx(&full[s], 2u * (uint32_t)nb * (kABytes + b_bytes));
          for (int h = 0; h < nb; ++h) {
            const int kc = (kb + h) * kGemmBK;
            tma_load_2d_pair(smem_u32(a_smem + (size_t)s * a_stage + (size_t)h * kABytes), &tmX, bar, kc, tok);
            tma_load_2d_pair(smem_u32(b_smem + (size_t)s * b_stage + (size_t)h * b_bytes), &tmW, bar, kc, wrow);
          }
        }
      }
      if (!ok && v == 0) {
        // drain the copies still in flight before the CTA can exit
        for (int j = max(0, it - S); j < it; ++j)
          mbar_wait(&full[j % S], (uint32_t)(j / S) & 1u, p.err);
      }
    }
    if (csk) cluster_arrive();  // this warp is done with the ring (cluster split-K)
  } else if (warp == 1) {
    // ---- MMA issuer (leader only): M = 256 tokens, N = NP columns
    if (lane == 0 && v == 0) {
      const uint32_t idesc = umma_idesc_bf16(2 * kGemmBM, NP);
      const uint32_t empty_own = map_to_rank(smem_u32(empty), leader);
      const uint32_t empty_peer = map_to_rank(smem_u32(empty), leader + 1u);
      const uint32_t accf_own = map_to_rank(smem_u32(acc_full), leader);
      const uint32_t accf_peer = map_to_rank(smem_u32(acc_full), leader + 1u);
      int it = 0, seg = 0;
      bool ok = true;
      long long su = u_begin;
      int sk = 0;
      PairSeg sg;
      for (; ok && next_seg(su, sk, sg); ++seg) {
        const int kbb = sg.kbb, kbe = sg.kbe;
        const int b = seg & 1;
        // the epilogues of both CTAs have drained this accumulator
        if (!mbar_wait(&acc_empty[b], (((uint32_t)seg >> 1) & 1u) ^ 1u, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)b * acc_stride;
        for (int kb = kbb; kb < kbe; kb += KS, ++it) {
          const int s = it % S;
          const uint32_t ph = (uint32_t)(it / S) & 1u;
          const int nb = min(KS, kbe - kb);
          if (!mbar_wait(&full[s], ph, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int h = 0; h < nb; ++h) {
            const uint32_t a_base = smem_u32(a_smem + (size_t)s * a_stage + (size_t)h * kABytes);
            const uint32_t b_base = smem_u32(b_smem + (size_t)s * b_stage + (size_t)h * b_bytes);
#pragma unroll
            for (int kk = 0; kk < kGemmBK / 16; ++kk) {
              tc_mma_f16_pair(d, umma_desc_sw128(a_base + kk * 32), umma_desc_sw128(b_base + kk * 32),
                              idesc, (kb != kbb || h != 0 || kk != 0) ? 1u : 0u);
            }
          }
          tc_commit_pair(empty_own + (uint32_t)s * 8u);
          tc_commit_pair(empty_peer + (uint32_t)s * 8u);
        }
        tc_commit_pair(accf_own + (uint32_t)b * 8u);
        tc_commit_pair(accf_peer + (uint32_t)b * 8u);
      }
    }
    if (csk) cluster_arrive();  // this warp is done with the ring (cluster split-K)
  } else {
    // ---- epilogue warps 2..5: TMEM lane quarters 2,3,0,1; thread = token
    if (p.gbar != nullptr) {
      // fused RMSNorm first: rows blockIdx.x, + gridDim.x, ... of the
      // activations, while the producer's first weight loads are in flight
      __shared__ float s_nred[4];
      for (int r = blockIdx.x; r < p.T; r += gridDim.x) norm_row_128(p, r, (int)threadIdx.x - 64, s_nred);
      __threadfence();
      mbar_arrive(norm_bar);
    }
    const int q = warp & 3;
    const int row = q * 32 + lane;  // token inside this CTA's 128
    const bool lead_thread = (warp == 2 && lane == 0);
    const uint32_t acc_empty_leader = map_to_rank(smem_u32(acc_empty), leader);
    const int nchunks = NP / 32;
    // TMEM chunks in consumption order (SiLU: gate chunk m, then up chunk m)
    auto chunk_at = [&](int i) { return silu ? ((i & 1) ? nchunks / 2 + (i >> 1) : (i >> 1)) : i; };
    bool ok = true;
    int seg = 0;
    // output chunks staged so far (staging buffer = outs & 3); it keeps
    // counting across segments, so the buffer written next was last used four
    // stores ago, which the wait after every store has retired
    int outs = 0;
    // one output chunk: bias / SiLU already applied, bf16 rounding here;
    // staged for a TMA store (64-byte swizzle) or stored from registers
    auto emit_chunk = [&](float (&a)[32], int f0, int fmax, int row0, int tok) {
      if (p.use_tma_store) {
        const bool staged = f0 < fmax && row0 < p.T;  // uniform over the CTA
        uint8_t* stg = stage_out + (outs & 3) * (kGemmBM * 64);
        if (staged) {
          const uint32_t sw = (uint32_t)((row >> 1) & 3);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(stg + row * 64 + ((j ^ sw) * 16)) =
                make_uint4(pack_bf16x2(a[8 * j], a[8 * j + 1]), pack_bf16x2(a[8 * j + 2], a[8 * j + 3]),
                           pack_bf16x2(a[8 * j + 4], a[8 * j + 5]), pack_bf16x2(a[8 * j + 6], a[8 * j + 7]));
          fence_proxy_async_smem();
        }
        epi_bar_sync();
        if (staged) {
          if (lead_thread) {
            tma_store_2d(&tmY, smem_u32(stg), f0, row0);
            bulk_commit_group();
            bulk_wait_group_read<2>();  // the buffer written two stores from now is free
          }
          ++outs;
        }
      } else if (tok < p.T && f0 < fmax) {
        __nv_bfloat16* dst = p.y + (size_t)tok * p.ldy + f0;
        if (p.vec_ok && f0 + 32 <= fmax) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            reinterpret_cast<uint4*>(dst)[j] =
                make_uint4(pack_bf16x2(a[8 * j], a[8 * j + 1]), pack_bf16x2(a[8 * j + 2], a[8 * j + 3]),
                           pack_bf16x2(a[8 * j + 4], a[8 * j + 5]), pack_bf16x2(a[8 * j + 6], a[8 * j + 7]));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (f0 + j < fmax) dst[j] = __float2bfloat16_rn(a[j]);
        }
      }
    };
    if (csk) {
      // ---- cluster split-K (see the schedule notes above).  The other
      // members push their partials of this CTA's output chunks (c % C ==
      // cmem) into its ring: arm the byte count before the barrier.
      const int n_own = cmem < nchunks ? (nchunks - cmem + C - 1) / C : 0;
      if (lead_thread) mbar_arrive_expect_tx(&fix_bar[0], (uint32_t)(n_own * (C - 1)) * kChunkFloats * 4);
      const bool have = mbar_wait(&acc_full[0], 0u, p.err);
      tc_fence_before();
      cluster_arrive();
      cluster_wait();  // every pair of the cluster has finished its MMAs: every ring is idle
      tc_fence_after();
      const uint32_t d = tmem_base + ((uint32_t)(q * 32) << 16);
      const uint32_t my_ring = smem_u32(smem) + (uint32_t)row * 16u;
      const uint32_t my_bar = smem_u32(&fix_bar[0]);
      // push the chunks owned by the other members, the next TMEM load
      // overlapping this chunk's remote stores
      auto next_push = [&](int c) {
        do {
          ++c;
        } while (c < nchunks && c % C == cmem);
        return c;
      };
      {
        uint32_t rc[32], rn[32];
        int c = next_push(-1);
        if (c < nchunks) {
          tmem_ld_32x32b_x32(d + (uint32_t)(c * 32), rc);
          tmem_ld_wait_regs(rc);
        }
        while (c < nchunks) {
          const int nx = next_push(c);
          if (nx < nchunks) tmem_ld_32x32b_x32(d + (uint32_t)(nx * 32), rn);
          const int owner = c % C;
          const uint32_t peer = (uint32_t)(owner * 2) + v;  // the owner, same token half
          const int slot = (c / C) * (C - 1) + (cmem < owner ? cmem : cmem - 1);
          const uint32_t dst = map_to_rank(my_ring, peer) + (uint32_t)slot * (uint32_t)(kChunkFloats * 4);
          const uint32_t bar = map_to_rank(my_bar, peer);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            st_async_v4(dst + (uint32_t)(j * kGemmBM * 16), rc[4 * j], rc[4 * j + 1], rc[4 * j + 2],
                        rc[4 * j + 3], bar);
          if (nx < nchunks) tmem_ld_wait_regs(rn);
#pragma unroll
          for (int j = 0; j < 32; ++j) rc[j] = rn[j];
          c = nx;
        }
      }
      const bool got = mbar_wait_cluster(&fix_bar[0], 0u, p.err);
      const long long tile = blockIdx.x / (2 * C);
      const int mt = (int)(tile / p.tiles_t);
      const int tt = (int)(tile - (long long)mt * p.tiles_t);
      const int row0 = tt * 2 * kGemmBM + (int)v * kGemmBM;
      const int tok = row0 + row;
      for (int c = cmem; c < nchunks; c += C) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(d + (uint32_t)(c * 32), r);
        tmem_ld_wait_regs(r);
        float acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = have ? __uint_as_float(r[j]) : 0.f;
        if (got) {
          // own partial, then the other members' in rank order (one owner
          // per chunk: a fixed summation order)
          for (int si = 0; si < C - 1; ++si) {
            const float4* src =
                reinterpret_cast<const float4*>(smem + (size_t)((c / C) * (C - 1) + si) * kChunkFloats * 4) + row;
            float4 f[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) f[j] = src[j * kGemmBM];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              acc[4 * j] += f[j].x; acc[4 * j + 1] += f[j].y; acc[4 * j + 2] += f[j].z; acc[4 * j + 3] += f[j].w;
            }
          }
        }
        const int f0 = mt * NP + c * 32;
        if (p.bias != nullptr) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (f0 + j < p.N) acc[j] += __bfloat162float(p.bias[f0 + j]);
        }
        emit_chunk(acc, f0, p.N, row0, tok);
      }
    }
    long long su = csk ? u_end : u_begin;  // cluster split-K: no segment loop
    int sk = 0;
    PairSeg sg;
    for (; next_seg(su, sk, sg); ++seg) {
      const long long tile = sg.tile;
      const int kbb = sg.kbb, kbe = sg.kbe;
      const int mt = (int)(tile / p.tiles_t);
      const int tt = (int)(tile - (long long)mt * p.tiles_t);
      const int tok = tt * 2 * kGemmBM + (int)v * kGemmBM + row;  // this thread's token
      const int f_base = mt * tile_feats;
      const bool contributor = sg.member < 0 && kbb > 0;
      const bool finisher = sg.member < 0 && kbb == 0 && kbe < p.num_kb;
      const int b = seg & 1;
      if (ok) ok = mbar_wait(&acc_full[b], ((uint32_t)seg >> 1) & 1u, p.err);
      tc_fence_after();
      if (sg.member >= 0) {
        // ---- grouped split-K member (see the schedule notes above)
        const int g = p.grp_size, me = sg.member;
        const int first = (int)tile * g;  // the group's pairs: first .. first + g - 1
        const int nout = silu ? nchunks / 2 : nchunks;
        const int hn = silu ? nchunks / 2 : 0;  // SiLU: up chunk of output o is o + hn
        const uint32_t d = tmem_base + (uint32_t)b * acc_stride + ((uint32_t)(q * 32) << 16);
        float* my_part = p.sk_part + ((size_t)pr * 2 + v) * (size_t)NP * kGemmBM;
        // pass 1: the chunks of outputs other members own -> this CTA's
        // partial slot; the TMEM load of the next such chunk overlaps the
        // stores of this one
        auto owned = [&](int ch) { return ((silu ? ch % hn : ch) % g) == me; };
        auto next_pub = [&](int ch) {
          do {
            ++ch;
          } while (ch < nchunks && owned(ch));
          return ch;
        };
        {
          uint32_t rc[32], rn[32];
          int ch = next_pub(-1);
          if (ch < nchunks) {
            tmem_ld_32x32b_x32(d + (uint32_t)(ch * 32), rc);
            tmem_ld_wait_regs(rc);
          }
          while (ch < nchunks) {
            const int nx = next_pub(ch);
            if (nx < nchunks) tmem_ld_32x32b_x32(d + (uint32_t)(nx * 32), rn);
            float4* dst = reinterpret_cast<float4*>(my_part + (size_t)ch * kChunkFloats) + row;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              __stcg(dst + j * kGemmBM, make_float4(__uint_as_float(rc[4 * j]), __uint_as_float(rc[4 * j + 1]),
                                                    __uint_as_float(rc[4 * j + 2]), __uint_as_float(rc[4 * j + 3])));
            if (nx < nchunks) tmem_ld_wait_regs(rn);
#pragma unroll
            for (int j = 0; j < 32; ++j) rc[j] = rn[j];
            ch = nx;
          }
        }
        __threadfence();
        epi_bar_sync();
        if (lead_thread) st_release_gpu(p.sk_flags + (size_t)pr * 2 + v, 1u);
        if (me < nout) {
          // pass 2: wait for the other members' partials (bounded), then sum
          // this member's outputs: own TMEM first, the members in order after
          __shared__ int s_grp_ok;
          if (lead_thread) {
            bool all = true;
            for (int m = 0; m < g && all; ++m) {
              if (m == me) continue;
              unsigned* f = p.sk_flags + (size_t)(first + m) * 2 + v;
              const unsigned long long t_start = globaltimer_ns();
              while (ld_acquire_gpu(f) == 0u) {
                if (globaltimer_ns() - t_start > kWaitLimitNs) {
                  raise_error(p.err, ERR_PEER_TIMEOUT);
                  all = false;
                  break;
                }
              }
            }
            s_grp_ok = all;
          }
          // With no whole tile after this segment the stage ring is idle
          // (every MMA of the pair has completed): the members' chunks this
          // CTA needs are pulled into it by one burst of bulk copies (slot
          // (owned output, member, gate/up)); otherwise they are read with
          // plain loads, two members per round trip.
          const int H = silu ? 2 : 1;
          const int n_own = (nout - me + g - 1) / g;
          const int copies = n_own * (g - 1) * H;
          const int ring_slots = (int)(((size_t)S * (a_stage + b_stage)) / (kChunkFloats * 4));
          const bool burst = p.grp_whole == 0 && copies <= ring_slots && copies <= 32;
          if (burst && lead_thread && s_grp_ok) {
            fence_proxy_async_global();  // the acquired partials, then bulk reads of them
            mbar_arrive_expect_tx(&fix_bar[0], (uint32_t)copies * kChunkFloats * 4);
            int k = 0;
            for (int o = me; o < nout; o += g)
              for (int m = 0; m < g; ++m) {
                if (m == me) continue;
                for (int h = 0; h < H; ++h, ++k)
                  bulk_load(smem_u32(smem) + (uint32_t)k * kChunkFloats * 4,
                            p.sk_part + ((size_t)(first + m) * 2 + v) * (size_t)NP * kGemmBM +
                                (size_t)(o + h * hn) * kChunkFloats,
                            kChunkFloats * 4, &fix_bar[0]);
              }
          }
          epi_bar_sync();
          const bool peers_ok = s_grp_ok != 0;
          const bool burst_ok = burst && peers_ok && mbar_wait(&fix_bar[0], 0u, p.err);
          int oi = 0;  // owned-output index (burst slots)
          auto group_chunk = [&](int ch, float (&a)[32]) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(d + (uint32_t)(ch * 32), r);
            tmem_ld_wait_regs(r);
#pragma unroll
            for (int j = 0; j < 32; ++j) a[j] = ok ? __uint_as_float(r[j]) : 0.f;
            if (!peers_ok) return;
            if (burst) {
              if (!burst_ok) return;
              const int h = (silu && ch >= hn) ? 1 : 0;
              int mi = 0;
              for (int m = 0; m < g; ++m) {
                if (m == me) continue;
                const float4* src = reinterpret_cast<const float4*>(
                                        smem + (size_t)((oi * (g - 1) + mi) * H + h) * kChunkFloats * 4) + row;
                float4 f[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) f[j] = src[j * kGemmBM];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  a[4 * j] += f[j].x; a[4 * j + 1] += f[j].y; a[4 * j + 2] += f[j].z; a[4 * j + 3] += f[j].w;
                }
                ++mi;
              }
              return;
            }
            auto part = [&](int m) {
              return reinterpret_cast<const float4*>(p.sk_part +
                                                     ((size_t)(first + m) * 2 + v) * (size_t)NP * kGemmBM +
                                                     (size_t)ch * kChunkFloats) + row;
            };
            // the other members in order
            for (int m = 0; m < g; ++m) {
              if (m == me) continue;
              const float4* src = part(m);
              float4 f[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) f[j] = __ldcg(src + j * kGemmBM);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                a[4 * j] += f[j].x; a[4 * j + 1] += f[j].y; a[4 * j + 2] += f[j].z; a[4 * j + 3] += f[j].w;
              }
            }
          };
          const int row0 = tt * 2 * kGemmBM + (int)v * kGemmBM;
          for (int o = me; o < nout; o += g) {
            float acc[32];
            group_chunk(o, acc);
            int f0, fmax;
            if (silu) {
              float up[32];
              group_chunk(o + hn, up);
#pragma unroll
              for (int j = 0; j < 32; j += 2) silu_mul2(acc[j], acc[j + 1], up[j], up[j + 1]);
              f0 = f_base + o * 32;
              fmax = p.silu_inter;
            } else {
              f0 = f_base + o * 32;
              fmax = p.N;
              if (p.bias != nullptr) {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (f0 + j < fmax) acc[j] += __bfloat162float(p.bias[f0 + j]);
              }
            }
            emit_chunk(acc, f0, fmax, row0, tok);
            ++oi;
          }
        }
        // every TMEM load of this accumulator is done: release it; the last
        // member of the group (this CTA half) resets the group's flags
        tc_fence_before();
        epi_bar_sync();
        if (lead_thread) {
          if (v == 0) mbar_arrive(&acc_empty[b]);
          else mbar_arrive_cluster(acc_empty_leader + (uint32_t)b * 8u);
          unsigned* done = p.sk_flags + kGrpDoneOffset + (size_t)tile * 2 + v;
          if (atomicAdd(done, 1u) == (unsigned)(g - 1)) {
            for (int m = 0; m < g; ++m) p.sk_flags[(size_t)(first + m) * 2 + v] = 0u;
            *done = 0u;
          }
        }
        continue;
      }
      // contributors of this tile: pairs pr+1, ... whose ranges start inside it
      const long long tile_end = (tile + 1) * p.num_kb;
      int last_contrib = pr;
      if (finisher) {
        while (last_contrib + 1 < pairs && sk_begin(total, last_contrib + 1, pairs) < tile_end)
          ++last_contrib;
        __shared__ int s_flags_ok;
        if (lead_thread) {
          bool all = true;
          for (int c = pr + 1; c <= last_contrib && all; ++c) {
            unsigned* f = p.sk_flags + (size_t)c * 2 + v;
            const unsigned long long t_start = globaltimer_ns();
            while (ld_acquire_gpu(f) == 0u) {
              if (globaltimer_ns() - t_start > kWaitLimitNs) {
                raise_error(p.err, ERR_PEER_TIMEOUT);
                all = false;
                break;
              }
            }
          }
          s_flags_ok = all;
        }
        epi_bar_sync();
        if (!s_flags_ok) last_contrib = pr;  // give up on the partials, keep going
      }
      const uint32_t d = tmem_base + (uint32_t)b * acc_stride + ((uint32_t)(q * 32) << 16);
      float* my_part = p.sk_part + ((size_t)pr * 2 + v) * (size_t)NP * kGemmBM;
      const int ncontrib = last_contrib - pr;
      // finisher: contributor partials stream into the idle stage ring
      const int ring_slots = min(kFixSlots, (int)(((size_t)S * (a_stage + b_stage)) / (kChunkFloats * 4)));
      const int copies = ncontrib * nchunks;
      auto issue_copy = [&](int k) {  // copy k: TMEM chunk chunk_at(k / ncontrib) of contributor pr+1 + k % ncontrib
        const int slot = k % ring_slots;
        const int cq = pr + 1 + k % ncontrib;
        const float* src = p.sk_part + ((size_t)cq * 2 + v) * (size_t)NP * kGemmBM +
                           (size_t)chunk_at(k / ncontrib) * kChunkFloats;
        mbar_arrive_expect_tx(&fix_bar[slot], kChunkFloats * 4);
        bulk_load(smem_u32(smem) + (uint32_t)slot * kChunkFloats * 4, src, kChunkFloats * 4,
                  &fix_bar[slot]);
      };
      if (copies > 0 && lead_thread) {
        fence_proxy_async_global();  // the acquired partials, then bulk reads of them
        fence_proxy_async_smem();
        for (int k = 0; k < min(copies, ring_slots); ++k) issue_copy(k);
      }
      float keep[32];  // SiLU: the gate chunk, held until its up chunk arrives
      // the barrier after which every TMEM load of this accumulator is done
      const int rel_i = nchunks >= 2 ? nchunks - 2 : 0;
      uint32_t rc[32], rn[32];
      tmem_ld_32x32b_x32(d + (uint32_t)(chunk_at(0) * 32), rc);
      tmem_ld_wait_regs(rc);
      for (int i = 0; i < nchunks; ++i) {
        const int ch = chunk_at(i);
        // the next chunk's TMEM load overlaps this chunk's work
        if (i + 1 < nchunks) tmem_ld_32x32b_x32(d + (uint32_t)(chunk_at(i + 1) * 32), rn);
        float acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = ok ? __uint_as_float(rc[j]) : 0.f;
        bool staged = false;
        int f0 = 0, row0 = 0;
        uint8_t* stg = nullptr;
        if (contributor) {
          float4* dst = reinterpret_cast<float4*>(my_part + (size_t)ch * kChunkFloats) + row;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            __stcg(dst + j * kGemmBM,
                   make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]));
        } else {
          for (int c = 0; c < ncontrib; ++c) {
            const int k = i * ncontrib + c;
            const int slot = k % ring_slots;
            if (!mbar_wait(&fix_bar[slot], (uint32_t)(k / ring_slots) & 1u, p.err)) continue;
            const float4* src = reinterpret_cast<const float4*>(smem + (size_t)slot * kChunkFloats * 4) + row;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 f = src[j * kGemmBM];
              acc[4 * j] += f.x; acc[4 * j + 1] += f.y; acc[4 * j + 2] += f.z; acc[4 * j + 3] += f.w;
            }
          }
          bool out = true;
          int fmax;
          if (silu) {
            if ((i & 1) == 0) {  // gate chunk: keep it for the up chunk
#pragma unroll
              for (int j = 0; j < 32; ++j) keep[j] = acc[j];
              out = false;
            } else {
#pragma unroll
              for (int j = 0; j < 32; j += 2) {
                float g0 = keep[j], g1 = keep[j + 1];
                silu_mul2(g0, g1, acc[j], acc[j + 1]);
                acc[j] = g0;
                acc[j + 1] = g1;
              }
            }
            f0 = f_base + (ch - nchunks / 2) * 32;
            fmax = p.silu_inter;
          } else {
            f0 = f_base + ch * 32;
            fmax = p.N;
            if (p.bias != nullptr) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (f0 + j < fmax) acc[j] += __bfloat162float(p.bias[f0 + j]);
            }
          }
          if (out && p.use_tma_store) {
            // stage the chunk ([128 tokens][32 features] bf16, 64-byte
            // swizzle) for the TMA engine; rows past T / columns past the
            // output width are clipped by the tensor map, boxes wholly
            // outside are not issued
            row0 = tt * 2 * kGemmBM + (int)v * kGemmBM;
            if (f0 < fmax && row0 < p.T) {
              stg = stage_out + (outs & 3) * (kGemmBM * 64);
              const uint32_t sw = (uint32_t)((row >> 1) & 3);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                *reinterpret_cast<uint4*>(stg + row * 64 + ((j ^ sw) * 16)) =
                    make_uint4(pack_bf16x2(acc[8 * j], acc[8 * j + 1]), pack_bf16x2(acc[8 * j + 2], acc[8 * j + 3]),
                               pack_bf16x2(acc[8 * j + 4], acc[8 * j + 5]), pack_bf16x2(acc[8 * j + 6], acc[8 * j + 7]));
              fence_proxy_async_smem();
              staged = true;
            }
          } else if (out && tok < p.T && f0 < fmax) {
            // this thread's token row: 32 consecutive features
            __nv_bfloat16* dst = p.y + (size_t)tok * p.ldy + f0;
            if (p.vec_ok && f0 + 32 <= fmax) {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                reinterpret_cast<uint4*>(dst)[j] =
                    make_uint4(pack_bf16x2(acc[8 * j], acc[8 * j + 1]), pack_bf16x2(acc[8 * j + 2], acc[8 * j + 3]),
                               pack_bf16x2(acc[8 * j + 4], acc[8 * j + 5]), pack_bf16x2(acc[8 * j + 6], acc[8 * j + 7]));
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (f0 + j < fmax) dst[j] = __float2bfloat16_rn(acc[j]);
            }
          }
        }
        if (i + 1 < nchunks) tmem_ld_wait_regs(rn);
        // one barrier per chunk (contributors: only the TMEM release): the
        // staging writes and partial-slot reads of every thread are done
        if (!contributor || i == rel_i) {
          if (i == rel_i) tc_fence_before();
          epi_bar_sync();
          if (lead_thread) {
            if (i == rel_i) {  // every TMEM load of this accumulator is done
              if (v == 0) mbar_arrive(&acc_empty[b]);
              else mbar_arrive_cluster(acc_empty_leader + (uint32_t)b * 8u);
            }
            if (staged) {
              tma_store_2d(&tmY, smem_u32(stg), f0, row0);
              bulk_commit_group();
              bulk_wait_group_read<2>();  // the buffer written two chunks from now is free
            }
            if (ncontrib > 0) {  // refill this chunk's partial slots
              fence_proxy_async_smem();
              for (int c = 0; c < ncontrib; ++c) {
                const int k = i * ncontrib + c + ring_slots;
                if (k < copies) issue_copy(k);
              }
            }
          }
        }
        if (staged) ++outs;
#pragma unroll
        for (int j = 0; j < 32; ++j) rc[j] = rn[j];
      }
      if (contributor) {
        // publish the partial: every epilogue thread's stores, then the flag
        __threadfence();
        epi_bar_sync();
        if (lead_thread) st_release_gpu(p.sk_flags + (size_t)pr * 2 + v, 1u);
      } else if (ncontrib > 0) {
        // the partials are consumed: reset their flags for the next launch
        if (lead_thread)
          for (int cq = pr + 1; cq <= last_contrib; ++cq) p.sk_flags[(size_t)cq * 2 + v] = 0u;
      }
    }
    if (lead_thread && p.use_tma_store) bulk_wait_group_all();  // outputs written before exit
  }
  // the producer and MMA warps complete the cluster barrier they arrived on
  if (csk && warp < 2) cluster_wait();
  // every TMEM read and remote arrive of both CTAs is done before the pair
  // frees its TMEM and either CTA exits
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, (uint32_t)p.tmem_cols);
  }
}

}  // namespace b200
