// Prefill attention on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Device side of src/layers/attention.py:79-104 (flash_attn_varlen_func,
// causal, bottom-right aligned, GQA, K/V from the paged cache through the
// block table or per token) for prefill, chunked prefill, prefix hits and
// mixed batches, head_dim 128.
//
// One CTA = 128 queries of one query head of one sequence (the TMEM lanes),
// streaming the visible keys in tiles of 128:
//   warp 0      TMA producer: the Q tile once, then K and V tiles of 128 keys
//               (3-D tensor maps {dims, kv heads, rows}, boxes of 64 dims x
//               128 rows, 128-byte swizzle) into a 2-stage ring; with a
//               block table a tile is one half of a 256-key page
//   warp 1      TMEM owner and MMA issuer (one thread):
//                 S_j = Q K_j^T   M = 128 queries, N = 128 keys, K = 128 dims,
//                                 both operands K-major, into one of two TMEM
//                                 S buffers (S_{j+1} is computed while the
//                                 softmax works on S_j)
//                 O  += P_j V_j   M = 128, N = 128 dims, K = 128 keys; P from
//                                 shared memory (K-major), V MN-major (the
//                                 cache's [key][dim] rows as they land)
//   warps 2..9  softmax, two threads per query row (its TMEM lane): warps
//               2-5 take key columns 0-63 of S (and dims 0-63 of O), warps 6-9
//               columns 64-127; masked row maximum (halves combined through
//               shared memory), then (once O += P_{j-1} V_{j-1} is done) the
//               rescale of O in TMEM when the maximum grew, P = exp2(S * scale
//               * log2 e - m) rounded to bf16 into shared memory (the operand
//               rounding of flash attention), running sums in fp32; at the end
//               O / l -> bf16 rows.
// TMEM: O in columns [0, 128), the S buffers in [128, 384).  Every wait is
// bounded and records an error bit instead of hanging.
#pragma once
#include "common.cuh"

namespace b200 {

constexpr int kPtBM = 128;       // queries per CTA
constexpr int kPtBN = 128;       // keys per tile
constexpr int kPtThreads = 320;  // producer, MMA issuer, 8 softmax warps
// shared memory (1024-byte aligned): Q | 2 x (K | V) | P | barriers
constexpr int kPtQ = 0;
constexpr int kPtStage = 32768;  // stage s: K at kPtStage + s * 65536, V 32 KB after it
constexpr int kPtP = kPtStage + 2 * 65536;
constexpr int kPtBar = kPtP + 32768;
constexpr int kPtRed = kPtBar + 128;  // float [2 halves][128 rows]: row maxima, then row sums
constexpr int kPtSmemBytes = 1024 + kPtRed + 1024;

struct PrefillTcArgs {
  const int* cu_q;
  const int* cu_k;
  const int* block_tables;  // null: K / V per token
  int bt_stride, bt_width;
  long long num_slots;      // paged: rows of the cache
  int B, Hq, Hkv, G, page;
  float scale_log2;
  __nv_bfloat16* out;
  long long out_stride;
  unsigned* err;
};

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Descriptor of an MN-major operand with the 128-byte swizzle: atoms of 64
// contiguous elements (one 128-byte row) x 8 rows along K; `lbo` bytes
// between atoms along MN, 1024 bytes between 8-row groups along K.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void pt_bar_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// The first cache row of key tile `key0` of sequence b (paged), or -1 when
// the block table has no valid block for it.
__device__ __forceinline__ long long pt_tile_row(const PrefillTcArgs& a, int b, int key0) {
  const int col = key0 / a.page;
  const long long blk = col < a.bt_width ? a.block_tables[(size_t)b * a.bt_stride + col] : -1;
  const long long row = blk * a.page + (key0 - col * a.page);
  return (blk >= 0 && row + kPtBN <= a.num_slots) ? row : -1;
}

__global__ void __launch_bounds__(kPtThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const PrefillTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPtBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* o_done = bars + 10;
  uint64_t* mma_drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  int* s_abort = reinterpret_cast<int*>(bars + 13);

  griddep_wait();
  griddep_launch_dependents();
  const int b = blockIdx.z, hq = blockIdx.y, h = hq / a.G;
  const int q0 = a.cu_q[b];
  const int Lq = a.cu_q[b + 1] - q0;
  const int i0 = blockIdx.x * kPtBM;
  if (Lq <= 0 || i0 >= Lq) return;  // the whole CTA, before any barrier or TMEM
  const int k0 = a.cu_k[b];
  const int Lk = a.cu_k[b + 1] - k0;
  const int off = Lk - Lq;
  const int key_end = max(0, min(Lk, i0 + kPtBM + off));  // keys any row of the tile sees
  const int ntiles = (key_end + kPtBN - 1) / kPtBN;
  const bool paged = a.block_tables != nullptr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 12; ++i) mbar_init(&bars[i], 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t smem_base = smem_u32(smem);

  if (warp == 0) {
    // ---- producer
    if (lane == 0 && ntiles > 0) {
      mbar_arrive_expect_tx(q_full, 32768);
      tma_load_3d(smem_base + kPtQ, &tmQ, smem_u32(q_full), 0, hq, q0 + i0);
      tma_load_3d(smem_base + kPtQ + 16384, &tmQ, smem_u32(q_full), 64, hq, q0 + i0);
      for (int j = 0; j < ntiles; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[s], (uint32_t)((j >> 1) & 1) ^ 1u, a.err)) break;
        const int key0 = j * kPtBN;
        long long row;
        if (paged) {
          row = pt_tile_row(a, b, key0);
          if (row < 0) {
            raise_error(a.err, ERR_BAD_INDEX);
            row = 0;  // loads rows 0..; the softmax masks the whole tile
          }
        } else {
          row = (long long)k0 + key0;
        }
        const uint32_t st = smem_base + kPtStage + (uint32_t)s * 65536u;
        const uint32_t bar = smem_u32(&kv_full[s]);
        mbar_arrive_expect_tx(&kv_full[s], 65536);
        tma_load_3d(st, &tmK, bar, 0, h, (int)row);
        tma_load_3d(st + 16384, &tmK, bar, 64, h, (int)row);
        tma_load_3d(st + 32768, &tmV, bar, 0, h, (int)row);
        tma_load_3d(st + 49152, &tmV, bar, 64, h, (int)row);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0 && ntiles > 0) {
      const uint32_t idesc_s = umma_idesc_bf16(kPtBM, kPtBN);
      const uint32_t idesc_o = umma_idesc_bf16(kPtBM, 128) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(q_full, 0u, a.err);
      for (int j = 0; ok && j <= ntiles; ++j) {
        if (j < ntiles) {
          const int s = j & 1;
          if (!mbar_wait(&kv_full[s], (uint32_t)(j >> 1) & 1u, a.err)) break;
          if (j >= 2 && !mbar_wait(&s_free[s], (uint32_t)((j >> 1) & 1) ^ 1u, a.err)) break;
          tc_fence_after();
          const uint32_t d = tmem_base + 128u + (uint32_t)s * 128u;
          const uint32_t kb = smem_base + kPtStage + (uint32_t)s * 65536u;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t o = (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u;
            tc_mma_f16(d, umma_desc_sw128(smem_base + kPtQ + o), umma_desc_sw128(kb + o), idesc_s,
                       kk > 0 ? 1u : 0u);
          }
          tc_commit(&s_full[s]);
        }
        if (j >= 1) {
          const int jj = j - 1, ss = jj & 1;
          if (!mbar_wait(p_full, (uint32_t)jj & 1u, a.err)) break;
          tc_fence_after();
          const uint32_t vb = smem_base + kPtStage + (uint32_t)ss * 65536u + 32768u;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t pa = smem_base + kPtP + (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u;
            tc_mma_f16(tmem_base, umma_desc_sw128(pa), umma_desc_sw128_mn(vb + (uint32_t)kk * 2048u, 16384u),
                       idesc_o, (jj > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(o_done);
          tc_commit(&kv_empty[ss]);
        }
      }
      // every MMA issued has completed before TMEM can be released
      tc_commit(mma_drain);
      mbar_wait(mma_drain, 0u, a.err);
    }
  } else {
    // ---- softmax / correction / epilogue: two threads per query row (its
    // TMEM lane), one per half of the columns
    const int sw = warp - 2;           // 0..7
    const int q = warp & 3;            // TMEM lane quarter of this warp
    const int hf = sw >> 2;            // 0: S columns / O dims 0-63, 1: 64-127
    const int row = q * 32 + lane;
    const int i = i0 + row;            // query index inside the sequence
    const int vis = i + off;           // last key this row sees (inclusive)
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    const bool lead = sw == 0 && lane == 0;
    float* red = reinterpret_cast<float*>(smem + kPtRed);  // [2][128]
    float m = -INFINITY, l = 0.f;      // l: this half's share of the row sum
    bool ok = true;
    // A wait that runs out sets s_abort; every softmax warp still reaches the
    // named barriers of the iteration, and all of them leave the loop after it.
    for (int j = 0; j < ntiles; ++j) {
      const int s = j & 1;
      bool fail = !mbar_wait(&s_full[s], (uint32_t)(j >> 1) & 1u, a.err);
      tc_fence_after();
      const int key0 = j * kPtBN;
      const bool tile_ok = !paged || pt_tile_row(a, b, key0) >= 0;
      const int lim = tile_ok ? min(Lk - 1, vis) - key0 : -1;  // last valid key of the tile, local index
      // every row of the CTA sees the whole tile: no masking
      const bool whole = tile_ok && key0 + kPtBN - 1 <= min(Lk - 1, i0 + off);
      const uint32_t sa = tmem_base + lane_addr + 128u + (uint32_t)s * 128u + (uint32_t)(hf * 64);
      // pass 1: masked maximum of this half (log2 domain), then the row's
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(sa + (uint32_t)(c * 32), r);
        tmem_ld_wait();
        const int col0 = hf * 64 + c * 32;
        if (whole) {
#pragma unroll
          for (int t = 0; t < 32; ++t) mt = fmaxf(mt, __uint_as_float(r[t]));
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) mt = fmaxf(mt, col0 + t <= lim ? __uint_as_float(r[t]) : -INFINITY);
        }
      }
      mt *= a.scale_log2;  // the scale is positive: max commutes with it
      red[hf * 128 + row] = mt;
      pt_bar_sync();
      mt = fmaxf(red[row], red[128 + row]);
      const float m_new = fmaxf(m, mt);
      const float alpha = (m == -INFINITY) ? 0.f : fast_exp2(m - m_new);
      // O += P_{j-1} V_{j-1} must be done before P is rewritten or O rescaled
      if (j >= 1) {
        fail |= !mbar_wait(o_done, (uint32_t)(j - 1) & 1u, a.err);
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t oa = tmem_base + lane_addr + (uint32_t)(hf * 64 + c * 32);
            uint32_t r[32];
            tmem_ld_32x32b_x32(oa, r);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < 32; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * alpha);
            tmem_st_32x32b_x32(oa, r);
          }
          tmem_st_wait();
        }
      }
      // pass 2: P = exp2(S' - m) as bf16 into this half's region of the
      // K-major, 128-byte swizzled P tile ([2 key halves][128 rows][128 B])
      float rs = 0.f;
      uint8_t* prow = smem + kPtP + hf * 16384 + row * 128;
      const bool live = m_new != -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(sa + (uint32_t)(c * 32), r);
        tmem_ld_wait();
        const int col0 = hf * 64 + c * 32;
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          float p0 = fast_exp2(__uint_as_float(r[t]) * a.scale_log2 - m_new);
          float p1 = fast_exp2(__uint_as_float(r[t + 1]) * a.scale_log2 - m_new);
          if (!whole) {
            p0 = (col0 + t <= lim && live) ? p0 : 0.f;
            p1 = (col0 + t + 1 <= lim && live) ? p1 : 0.f;
          }
          rs += p0 + p1;
          pk[t >> 1] = pack_bf16x2(p0, p1);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int chunk = (c * 4 + u) ^ (row & 7);
          *reinterpret_cast<uint4*>(prow + chunk * 16) =
              make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      l = l * alpha + rs;
      m = m_new;
      // keys past the sequence (or a whole tile without a valid block) may hold
      // stale cache bits: zero those V rows (P is 0 there, and 0 * NaN = NaN);
      // each half zeroes its 64 dims
      if (paged && (!tile_ok || key0 + row >= Lk)) {
        uint8_t* v = smem + kPtStage + s * 65536 + 32768 + hf * 16384 + row * 128;
#pragma unroll
        for (int u = 0; u < 8; ++u) *reinterpret_cast<uint4*>(v + u * 16) = make_uint4(0u, 0u, 0u, 0u);
      }
      if (fail) *s_abort = 1;
      fence_proxy_async_smem();
      tc_fence_before();
      pt_bar_sync();
      const bool abort_now = *reinterpret_cast<volatile int*>(s_abort) != 0;
      if (abort_now) {
        ok = false;
        break;
      }
      if (lead) {
        mbar_arrive(&s_free[s]);
        mbar_arrive(p_full);
      }
    }
    // ---- epilogue: O / l -> bf16 rows of this query head, each half its dims
    red[hf * 128 + row] = l;
    pt_bar_sync();
    const float lt = red[row] + red[128 + row];
    bool have = ntiles > 0 && ok;
    if (have) {
      have = mbar_wait(o_done, (uint32_t)(ntiles - 1) & 1u, a.err);
      tc_fence_after();
    }
    const float f = have && lt > 0.f ? 1.f / lt : 0.f;
    __nv_bfloat16* dst = a.out + (size_t)(q0 + i) * a.out_stride + (size_t)hq * 128 + hf * 64;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      uint32_t r[32];
#pragma unroll
      for (int t = 0; t < 32; ++t) r[t] = 0u;
      if (ntiles > 0) {
        tmem_ld_32x32b_x32(tmem_base + lane_addr + (uint32_t)(hf * 64 + c * 32), r);
        tmem_ld_wait();
      }
      if (i < Lq) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(r[8 * u]) * f, __uint_as_float(r[8 * u + 1]) * f);
          w.y = pack_bf16x2(__uint_as_float(r[8 * u + 2]) * f, __uint_as_float(r[8 * u + 3]) * f);
          w.z = pack_bf16x2(__uint_as_float(r[8 * u + 4]) * f, __uint_as_float(r[8 * u + 5]) * f);
          w.w = pack_bf16x2(__uint_as_float(r[8 * u + 6]) * f, __uint_as_float(r[8 * u + 7]) * f);
          *reinterpret_cast<uint4*>(dst + c * 32 + u * 8) = w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace b200
