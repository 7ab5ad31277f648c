// Paged decode attention (q_len == 1 per live sequence), head_dim 128.
//
// Device side of src/layers/attention.py:93-104 for the pure-decode batches
// that ModelRunner replays from a CUDA graph (model_runner.py:241-259):
// flash_attn_varlen_func with a block table, causal (for q_len == 1 every
// cached key is visible), GQA (q head n reads kv head n / G).
//
// Work decomposition (HBM-bound: every K/V byte is read exactly once):
//   item  = (512-token group of one sequence, kv head); an item may span
//           pages (their block-table entries are read once per item).  The
//           G = Hq / Hkv query heads that share the kv head are the columns
//           of the MMAs (tokens are the rows: S^T = K Q^T, O^T = V^T P^T).
//   warp  = owns whole items, taken from a global atomic counter (dynamic
//           scheduling: no tail from uneven sequence lengths).  Each warp
//           runs its own 3-stage ring of 32-token K/V tiles (+ the item's Q
//           rows with its first tile) loaded by TMA (cp.async.bulk.tensor,
//           128-byte swizzle, one mbarrier per stage, issued by lane 0), so
//           the ring keeps streaming across item boundaries and no CTA-wide
//           barrier is taken in the main loop.
//   merge = a sequence spanning several items writes per-item fp32 partials
//           (m, l, o) and bumps the completion counter of its (sequence, kv
//           head) unit.  A warp whose item queue has run dry takes the split
//           units, in sequence order, from a second queue, waits (bounded)
//           for the unit's items and merges them in one online-softmax pass,
//           so the merges overlap the other warps' last items instead of
//           following a grid-wide barrier.  A single-item sequence writes its
//           output directly.  (The launch is cooperative: every CTA is
//           resident, and a unit's items are all taken by running warps
//           before any warp waits on it.)
// The launch shape depends only on the SM count; context lengths are read
// from cu_seqlens_k on the device (CUDA-graph safe; rows with q length <= 0
// are graph padding and are skipped).
#pragma once
#include "common.cuh"

namespace b200 {

constexpr int kDecHD = 128;
constexpr int kDecItem = 512;        // tokens per work item (may span pages); sizes the workspace
constexpr int kDecItemLong = 1024;   // tokens per item when the batch's mean context is long
constexpr int kDecLongMean = 2048;   // mean context (keys per sequence) from which items are long
constexpr int kDecItemPages = 4;     // block-table entries an item can touch (pages >= 256 tokens)
constexpr int kDecTile = 32;      // tokens per pipeline stage
constexpr int kDecStages = 3;
constexpr int kDecWarps = 4;
constexpr int kDecMaxSeqs = 1024;       // plan capacity (prefix sums in shared memory)
constexpr int kDecMaxKvHeads = 64;
// stage: K [2 halves][32 rows][128 B] | V same | Q [2 halves][8 rows][128 B]
constexpr int kDecStK = 0, kDecStV = 8192, kDecStQ = 16384;
constexpr int kDecStageBytes = 18432;
constexpr int kDecWarpBytes = kDecStages * kDecStageBytes;
// workspace head: the scheduler words {next item, warps out of the item
// queue, (unused), next merge unit, warps out of the merge queue} in the first
// 256 bytes, then the per-(sequence, kv head) completion counters
// [kDecMaxSeqs][kDecMaxKvHeads]; all zero between calls (the last warp out of
// each queue resets its words, a merge zeroes its counter)
constexpr int kDecSchedBytes = 256 + kDecMaxSeqs * kDecMaxKvHeads * 4;

struct DecodeArgs {
  const int* block_tables;
  int bt_stride, bt_width;
  const int* cu_q;
  const int* cu_k;
  int B, Hq, Hkv, G, page, q_box_rows;
  long long num_slots;
  float scale_log2;      // softmax_scale * log2(e)
  int* sched;            // workspace head (kDecSchedBytes): scheduler words, then unit counters
  float* part_ml;        // [cap_items][Hq][2]
  float* part_o;         // [cap_items][Hq][128]
  long long cap_items;
  __nv_bfloat16* out;
  long long out_stride;
  unsigned* err;
};

struct DecTile {
  int b, h, c, npages, qrow;
  int ntok;     // valid tokens in the tile (the item's, in the iterator)
  int first, last;
  long long row;  // cache row (slot) of the tile's first token
  int j0;         // iterator: the item's first token in the sequence
};

// Release-ordered increment: this thread's earlier writes, and those of the
// lanes ordered before it by __syncwarp, are visible to whoever acquires the
// new value (no separate fence instruction).
__device__ __forceinline__ void red_release_gpu_add_s32(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_gpu_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__host__ __device__ constexpr int dec_smem_bytes() {
  return 1024 + kDecWarps * kDecWarpBytes + kDecWarps * kDecStages * 8 +
         kDecWarps * kDecStages * (int)sizeof(DecTile) + (8 + kDecMaxSeqs + 1) * (int)sizeof(int);
}

// byte offset of 16-byte chunk `ch` (0..15 over 128 dims) of row `r` in a
// [2 halves][rows][128 B] TMA tile with the 128-byte swizzle
__device__ __forceinline__ uint32_t tswz(int half_bytes, int r, int ch) {
  return (uint32_t)((ch >> 3) * half_bytes + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(128, 1)
    decode_attn_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmQ, const DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // layout: [warp rings][mbarriers][tile descriptors][scan scratch][plan]
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(smem + kDecWarps * kDecWarpBytes) + warp * kDecStages;
  DecTile* s_desc = reinterpret_cast<DecTile*>(smem + kDecWarps * kDecWarpBytes + kDecWarps * kDecStages * 8) +
                    warp * kDecStages;
  int* s_scan = reinterpret_cast<int*>(smem + kDecWarps * kDecWarpBytes + kDecWarps * kDecStages * 8 +
                                       kDecWarps * kDecStages * sizeof(DecTile));
  int* s_start = s_scan + 8;
  int* sched = a.sched;
  int* unit_done = a.sched + 64;  // [b * Hkv + h]: items of the unit published

  if (lane == 0) {
    for (int i = 0; i < kDecStages; ++i) mbar_init(&s_bar[i], 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmQ);
  }
  // the barrier setup above overlaps the previous kernel's tail
  // (programmatic dependent launch); sequence lengths, Q and the cache below
  griddep_wait();
  griddep_launch_dependents();

  // ---- plan: exclusive prefix sum of items per sequence (identical in every
  // CTA).  Item length: 512 keys, or 1024 when the batch's mean context is at
  // least kDecLongMean (half the per-item fixed work on long contexts; on
  // short ones the longer last items would lengthen the tail).
  int item_len = kDecItem;
  {
    const int tid = threadIdx.x;
    const int per = (a.B + 127) / 128;
    const int beg = min(a.B, tid * per), end = min(a.B, beg + per);
    long long keys = 0;
    int active = 0;
    for (int b = beg; b < end; ++b) {
      const int nq = a.cu_q[b + 1] - a.cu_q[b];
      const int nk = a.cu_k[b + 1] - a.cu_k[b];
      if (nq >= 1 && nk > 0) {
        keys += nk;
        ++active;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      keys += __shfl_xor_sync(0xffffffffu, keys, o);
      active += __shfl_xor_sync(0xffffffffu, active, o);
    }
    __shared__ long long s_keys[kDecWarps];
    if (lane == 0) {
      s_keys[warp] = keys;
      s_scan[warp] = active;
    }
    __syncthreads();
    long long all_keys = 0;
    int all_active = 0;
    for (int w = 0; w < kDecWarps; ++w) {
      all_keys += s_keys[w];
      all_active += s_scan[w];
    }
    if (all_active > 0 && all_keys >= (long long)kDecLongMean * all_active) item_len = kDecItemLong;
    __syncthreads();  // s_scan is reused by the scan below
    int local = 0;
    for (int b = beg; b < end; ++b) {
      const int nq = a.cu_q[b + 1] - a.cu_q[b];
      const int nk = a.cu_k[b + 1] - a.cu_k[b];
      const int cnt = (nq >= 1 && nk > 0) ? (nk + item_len - 1) / item_len : 0;
      s_start[b] = cnt;
      local += cnt;
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) s_scan[warp] = incl;
    __syncthreads();
    int run = incl - local;
    for (int w = 0; w < warp; ++w) run += s_scan[w];
    for (int b = beg; b < end; ++b) {
      const int cnt = s_start[b];
      s_start[b] = run;
      run += cnt;
    }
    if (tid == 127) s_start[a.B] = run;
    __syncthreads();
  }
  const int total_chunks = s_start[a.B];
  if ((long long)total_chunks > a.cap_items) {
    if (blockIdx.x == 0 && threadIdx.x == 0) raise_error(a.err, ERR_BAD_INDEX);
    return;
  }
  const int items = total_chunks * a.Hkv;
  const int nwarps = gridDim.x * kDecWarps;
  const uint32_t wsmem = smem_u32(smem + warp * kDecWarpBytes);

  // ---- tile iterator (uniform across the warp)
  bool more = true;       // the warp may still take items
  int it_k = 0, it_tiles = 0;
  DecTile cur{};
  long long blk0 = -1, blk1 = -1, blk2 = -1, blk3 = -1;  // the current item's pages
  auto grab_item = [&]() {
    int w = 0;
    if (lane == 0) w = atomicAdd(&sched[0], 1);
    w = __shfl_sync(0xffffffffu, w, 0);
    if (w >= items) {
      more = false;
      if (lane == 0 && atomicAdd(&sched[1], 1) == nwarps - 1) {
        // every warp has left the queue: reset it for the next call
        atomicExch(&sched[0], 0);
        atomicExch(&sched[1], 0);
      }
      return;
    }
    const int c = w / a.Hkv;
    const int h = w - c * a.Hkv;
    int lo = 0, hi = a.B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_start[mid] <= c) lo = mid; else hi = mid - 1;
    }
    const int b = lo;
    const int j0 = (c - s_start[b]) * item_len;
    const int nk = a.cu_k[b + 1] - a.cu_k[b];
    const int ntok_item = min(item_len, nk - j0);
    // the block-table entries of the item's pages (one per lane 0..3)
    const int col0 = j0 / a.page;
    long long e = -1;
    if (lane < kDecItemPages && col0 + lane < a.bt_width)
      e = a.block_tables[(size_t)b * a.bt_stride + col0 + lane];
    blk0 = __shfl_sync(0xffffffffu, e, 0);
    blk1 = __shfl_sync(0xffffffffu, e, 1);
    blk2 = __shfl_sync(0xffffffffu, e, 2);
    blk3 = __shfl_sync(0xffffffffu, e, 3);
    cur.b = b; cur.h = h; cur.c = c;
    cur.npages = s_start[b + 1] - s_start[b];
    cur.qrow = a.cu_q[b];
    cur.ntok = ntok_item;
    cur.j0 = j0;
    it_tiles = (ntok_item + kDecTile - 1) / kDecTile;
    it_k = 0;
  };
  grab_item();

  int issued = 0, valid_issued = 0;
  unsigned zeroed = 0;
  auto issue_next = [&]() {
    if (more) {
      const int s = issued % kDecStages;
      DecTile d = cur;
      // the tile's page and cache row; an invalid block loads rows 0.. of
      // the cache and masks every token
      const int tok0 = cur.j0 + it_k * kDecTile;
      const int pi = tok0 / a.page - cur.j0 / a.page;
      const long long blk = pi == 0 ? blk0 : pi == 1 ? blk1 : pi == 2 ? blk2 : pi == 3 ? blk3 : -1;
      const int ntile = min(kDecTile, cur.ntok - it_k * kDecTile);
      const long long row = blk * a.page + (tok0 % a.page);
      const bool valid = blk >= 0 && row + ntile <= a.num_slots;
      if (!valid && lane == 0) raise_error(a.err, ERR_BAD_INDEX);
      d.ntok = valid ? ntile : 0;
      d.first = it_k == 0;
      d.last = it_k == it_tiles - 1;
      d.row = valid ? row : 0;
      if (lane == 0) {
        s_desc[s] = d;
        const uint32_t st = wsmem + s * kDecStageBytes;
        const uint32_t bar = smem_u32(&s_bar[s]);
        if (zeroed & (1u << s)) fence_proxy_async_smem();
        mbar_arrive_expect_tx(&s_bar[s], 4 * 4096 + (d.first ? 2 * 128 * a.q_box_rows : 0));
        const int r = (int)d.row;
        tma_load_3d(st + kDecStK, &tmK, bar, 0, d.h, r);
        tma_load_3d(st + kDecStK + 4096, &tmK, bar, 64, d.h, r);
        tma_load_3d(st + kDecStV, &tmV, bar, 0, d.h, r);
        tma_load_3d(st + kDecStV + 4096, &tmV, bar, 64, d.h, r);
        if (d.first) {
          tma_load_3d(st + kDecStQ, &tmQ, bar, 0, d.h * a.G, d.qrow);
          tma_load_3d(st + kDecStQ + 1024, &tmQ, bar, 64, d.h * a.G, d.qrow);
        }
      }
      ++valid_issued;
      if (++it_k == it_tiles) grab_item();
    }
    ++issued;
  };

  issue_next();
  issue_next();

  // Tokens are the MMA rows: S^T = K Q^T (m16n8k16: 16 tokens x 8 head
  // columns, k over the head dim) and O^T = V^T P^T (16 dims x 8 head
  // columns, k over tokens).  The G query heads of the kv head are columns
  // 0..G-1; columns >= G carry unrelated rows and are never stored (every
  // column is independent of the others).
  const int g = lane >> 2, tq = lane & 3;  // fragment row group / column pair
  uint32_t qb[8][2];                        // B fragments of Q^T, 8 k-steps of 16 dims
  float ot[8][4];                            // O^T: 8 tiles of 16 dims
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};  // head columns 2tq, 2tq+1
  int consumed = 0;
  // the unit whose partial this warp wrote last and has not yet published:
  // its counter is bumped just before the warp's next item stores (or when
  // the warp leaves the item loop), so the release finds those stores long
  // completed instead of stalling on fresh ones
  int pending_unit = -1;
  auto publish_pending = [&]() {
    if (pending_unit >= 0) {
      __syncwarp();
      if (lane == 0) red_release_gpu_add_s32(&unit_done[pending_unit], 1);
      pending_unit = -1;
    }
  };

  for (int t = 0; t < valid_issued; ++t) {
    __syncwarp();
    issue_next();  // refills the stage of tile t - 1
    const int s = t % kDecStages;
    const uint32_t ph = (uint32_t)(t / kDecStages) & 1u;
    int ok = 1;
    if (lane == 0) ok = mbar_wait(&s_bar[s], ph, a.err) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) break;
    consumed = t + 1;
    mbar_wait(&s_bar[s], ph, a.err);  // every lane observes the completed phase
    const DecTile d = s_desc[s];
    const uint32_t sK = wsmem + s * kDecStageBytes + kDecStK;
    const uint32_t sV = wsmem + s * kDecStageBytes + kDecStV;
    const uint32_t sQ = wsmem + s * kDecStageBytes + kDecStQ;
    if (d.ntok < kDecTile) {
      // rows past the sequence hold other data of the block (possibly never
      // written): zero V there so that P = 0 cannot meet a NaN
      uint8_t* vrow = smem + warp * kDecWarpBytes + s * kDecStageBytes + kDecStV;
      for (int idx = lane; idx < (kDecTile - d.ntok) * 16; idx += 32) {
        const int r = d.ntok + (idx >> 4), ch = idx & 15;
        *reinterpret_cast<uint4*>(vrow + tswz(4096, r, ch)) = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
      zeroed |= 1u << s;
    } else {
      zeroed &= ~(1u << s);
    }

    if (d.first) {
      // B fragments of Q^T = ldmatrix of the Q rows (heads) per 8-dim chunk
#pragma unroll
      for (int p4 = 0; p4 < 4; ++p4)
        ldmatrix_x4(sQ + tswz(1024, lane & 7, 4 * p4 + (lane >> 3)), qb[2 * p4][0], qb[2 * p4][1],
                    qb[2 * p4 + 1][0], qb[2 * p4 + 1][1]);
#pragma unroll
      for (int md = 0; md < 8; ++md) ot[md][0] = ot[md][1] = ot[md][2] = ot[md][3] = 0.f;
      m_run[0] = m_run[1] = -INFINITY;
      l_run[0] = l_run[1] = 0.f;
    }

    // S^T over the tile's 32 tokens: 2 token tiles of 16
    float sc[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t ka[4];
        ldmatrix_x4(sK + tswz(4096, 16 * mt + (lane & 7) + 8 * ((lane >> 3) & 1), 2 * kk + (lane >> 4)),
                    ka[0], ka[1], ka[2], ka[3]);
        mma_bf16_16816(sc[mt], ka, qb[kk][0], qb[kk][1]);
      }
    }
    // online softmax per head column (its 32 tokens live in the 8 lanes
    // that share tq: reduce over lane bits 2..4)
    float cm[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tok = 16 * mt + g + 8 * (i >> 1);
        const float v = tok < d.ntok ? sc[mt][i] * a.scale_log2 : -INFINITY;
        sc[mt][i] = v;
        cm[i & 1] = fmaxf(cm[i & 1], v);
      }
    }
    float alpha[2], m_new[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      cm[e] = fmaxf(cm[e], __shfl_xor_sync(0xffffffffu, cm[e], 4));
      cm[e] = fmaxf(cm[e], __shfl_xor_sync(0xffffffffu, cm[e], 8));
      cm[e] = fmaxf(cm[e], __shfl_xor_sync(0xffffffffu, cm[e], 16));
      m_new[e] = fmaxf(m_run[e], cm[e]);
      alpha[e] = m_run[e] == -INFINITY ? 0.f : fast_exp2(m_run[e] - m_new[e]);
      m_run[e] = m_new[e];
    }
    // P (bf16, as the PV operand of the reference's flash attention) ->
    // B fragments of P^T through 8x8 transposes
    float ls[2] = {0.f, 0.f};
    uint32_t pb[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      float pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        pv[i] = m_new[i & 1] == -INFINITY ? 0.f : fast_exp2(sc[mt][i] - m_new[i & 1]);
        ls[i & 1] += pv[i];
      }
      pb[mt][0] = movmatrix_trans(pack_bf16x2(pv[0], pv[1]));  // tokens 16mt + 2tq, +1
      pb[mt][1] = movmatrix_trans(pack_bf16x2(pv[2], pv[3]));  // tokens 16mt + 8 + 2tq, +1
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      ls[e] += __shfl_xor_sync(0xffffffffu, ls[e], 4);
      ls[e] += __shfl_xor_sync(0xffffffffu, ls[e], 8);
      ls[e] += __shfl_xor_sync(0xffffffffu, ls[e], 16);
      l_run[e] = l_run[e] * alpha[e] + ls[e];
    }
#pragma unroll
    for (int md = 0; md < 8; ++md) {
      ot[md][0] *= alpha[0]; ot[md][1] *= alpha[1];
      ot[md][2] *= alpha[0]; ot[md][3] *= alpha[1];
    }
    // O^T += V^T P^T: 8 dim tiles x 2 token steps
#pragma unroll
    for (int md = 0; md < 8; ++md) {
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        uint32_t va[4];
        ldmatrix_x4_trans(sV + tswz(4096, 16 * ks + (lane & 7) + 8 * (lane >> 4), 2 * md + ((lane >> 3) & 1)),
                          va[0], va[1], va[2], va[3]);
        mma_bf16_16816(ot[md], va, pb[ks][0], pb[ks][1]);
      }
    }

    if (!d.last) continue;
    // ---- item done: output (single item) or split-KV partial
    publish_pending();
    if (d.npages == 1) {
      // O / l, transposed back to [head][dim] rows: 4-byte stores of dim pairs
      const float inv0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f;
      const float inv1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
      // (the transposes are warp-wide: every lane runs them, then the lanes
      // of the G live heads store)
      __nv_bfloat16* dst = a.out + (size_t)d.qrow * a.out_stride + (size_t)(d.h * a.G + g) * kDecHD;
#pragma unroll
      for (int md = 0; md < 8; ++md) {
        const uint32_t lo = movmatrix_trans(pack_bf16x2(ot[md][0] * inv0, ot[md][1] * inv1));
        const uint32_t hi = movmatrix_trans(pack_bf16x2(ot[md][2] * inv0, ot[md][3] * inv1));
        if (g < a.G) {
          *reinterpret_cast<uint32_t*>(dst + 16 * md + 2 * tq) = lo;
          *reinterpret_cast<uint32_t*>(dst + 16 * md + 8 + 2 * tq) = hi;
        }
      }
      continue;
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int col = 2 * tq + e;
      if (col < a.G) {
        const size_t hq = (size_t)d.h * a.G + col;
        float* po = a.part_o + ((size_t)d.c * a.Hq + hq) * kDecHD;
#pragma unroll
        for (int md = 0; md < 8; ++md) {
          po[16 * md + g] = ot[md][e];
          po[16 * md + 8 + g] = ot[md][2 + e];
        }
        if (g == 0)
          *reinterpret_cast<float2*>(a.part_ml + ((size_t)d.c * a.Hq + hq) * 2) = make_float2(m_run[e], l_run[e]);
      }
    }
    pending_unit = d.b * a.Hkv + d.h;
  }
  publish_pending();
  // drain: every issued tile has landed before the CTA's shared memory is released
  if (lane == 0) {
    for (int t = consumed; t < valid_issued; ++t)
      mbar_wait(&s_bar[t % kDecStages], (uint32_t)(t / kDecStages) & 1u, a.err);
  }
  __syncwarp();

  // ---- merge phase: (sequence, kv head) units of sequences split into
  // several items, from a second queue in sequence order.  Each lane owns 4
  // of the 128 dims of every head of the group; one online-softmax pass over
  // the items, loads batched over 2 items x every head.
  const int units = a.B * a.Hkv;
  while (true) {
    int u = 0;
    if (lane == 0) u = atomicAdd(&sched[3], 1);
    u = __shfl_sync(0xffffffffu, u, 0);
    if (u >= units) break;
    const int b = u / a.Hkv, h = u - b * a.Hkv;
    const int c0 = s_start[b], np = s_start[b + 1] - c0;
    if (np <= 1) continue;  // written directly (or an empty row)
    if (lane == 0) {
      // the unit's items were all taken before this queue opened: wait
      // (bounded) until they are published, then zero the counter
      const unsigned long long t0 = globaltimer_ns();
      while (ld_acquire_gpu_s32(&unit_done[u]) < np) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          raise_error(a.err, ERR_PEER_TIMEOUT);
          break;
        }
        __nanosleep(128);
      }
      unit_done[u] = 0;
    }
    __syncwarp();
    const int G = a.G;
    float M[8], L[8];
    float4 acc[8];
#pragma unroll
    for (int gg = 0; gg < 8; ++gg) {
      M[gg] = -INFINITY;
      L[gg] = 0.f;
      acc[gg] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int p0 = 0; p0 < np; p0 += 2) {
      float2 ml[2][8];
      float4 ov[2][8];
#pragma unroll
      for (int uu = 0; uu < 2; ++uu)
#pragma unroll
        for (int gg = 0; gg < 8; ++gg) {
          const bool live = gg < G && p0 + uu < np;
          const size_t row = (size_t)(c0 + p0 + uu) * a.Hq + (size_t)h * G + gg;
          ml[uu][gg] = live ? __ldcg(reinterpret_cast<const float2*>(a.part_ml + row * 2))
                            : make_float2(-INFINITY, 0.f);
          ov[uu][gg] = live ? __ldcg(reinterpret_cast<const float4*>(a.part_o + row * kDecHD) + lane)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
      for (int uu = 0; uu < 2; ++uu)
#pragma unroll
        for (int gg = 0; gg < 8; ++gg) {
          const float mi = ml[uu][gg].x;
          if (mi == -INFINITY) continue;  // padding or an empty item
          const float mn = fmaxf(M[gg], mi);
          const float sc = fast_exp2(M[gg] - mn);  // 0 while M is -inf
          const float w = fast_exp2(mi - mn);
          L[gg] = L[gg] * sc + w * ml[uu][gg].y;
          acc[gg].x = acc[gg].x * sc + w * ov[uu][gg].x;
          acc[gg].y = acc[gg].y * sc + w * ov[uu][gg].y;
          acc[gg].z = acc[gg].z * sc + w * ov[uu][gg].z;
          acc[gg].w = acc[gg].w * sc + w * ov[uu][gg].w;
          M[gg] = mn;
        }
    }
    const int qrow = a.cu_q[b];
#pragma unroll
    for (int gg = 0; gg < 8; ++gg) {
      if (gg >= G) continue;
      const float inv = L[gg] > 0.f ? 1.f / L[gg] : 0.f;
      uint2 packed;
      packed.x = pack_bf16x2(acc[gg].x * inv, acc[gg].y * inv);
      packed.y = pack_bf16x2(acc[gg].z * inv, acc[gg].w * inv);
      *reinterpret_cast<uint2*>(a.out + (size_t)qrow * a.out_stride + ((size_t)h * G + gg) * kDecHD + lane * 4) =
          packed;
    }
  }
  // the last warp out of the merge queue resets it for the next call
  if (lane == 0 && atomicAdd(&sched[4], 1) == nwarps - 1) {
    atomicExch(&sched[3], 0);
    atomicExch(&sched[4], 0);
  }
}

}  // namespace b200
