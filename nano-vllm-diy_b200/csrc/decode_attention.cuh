// Paged decode attention (q_len == 1 per live sequence), head_dim 128.
//
// Device side of src/layers/attention.py:93-104 for the pure-decode batches
// that ModelRunner replays from a CUDA graph (model_runner.py:241-259):
// flash_attn_varlen_func with a block table, causal (for q_len == 1 every
// cached key is visible), GQA (q head n reads kv head n / G).
//
// Work decomposition (HBM-bound: every K/V byte is read exactly once):
//   item  = (256-token group of one sequence, kv head).  256 divides the
//           reference's block size (runner_config.py:39), so an item lies in
//           one physical block.  The G = Hq / Hkv query heads that share the
//           kv head are the rows of one m16n8k16 MMA.
//   warp  = owns whole items, taken from a global atomic counter (dynamic
//           scheduling: no tail from uneven sequence lengths).  Each warp
//           runs its own 3-stage ring of 32-token K/V tiles (+ the item's Q
//           rows with its first tile) loaded by TMA (cp.async.bulk.tensor,
//           128-byte swizzle, one mbarrier per stage, issued by lane 0), so
//           the ring keeps streaming across item boundaries and no CTA-wide
//           barrier is taken after the start.
//   merge = a sequence spanning several items writes per-item partials
//           (m, l, o); the warp that finishes the last item of (sequence,
//           kv head) -- found with an atomic ticket -- merges them and writes
//           the output, then resets the ticket.  A single-item sequence
//           writes its output directly.
// The launch shape depends only on the SM count; context lengths are read
// from cu_seqlens_k on the device (CUDA-graph safe; rows with q length <= 0
// are graph padding and are skipped).
#pragma once
#include "common.cuh"

namespace b200 {

constexpr int kDecHD = 128;
constexpr int kDecItem = 256;     // tokens per work item
constexpr int kDecTile = 32;      // tokens per pipeline stage
constexpr int kDecStages = 3;
constexpr int kDecWarps = 4;
constexpr int kDecMaxSeqs = 1024;       // plan / ticket capacity
constexpr int kDecMaxKvHeads = 64;
// stage: K [2 halves][32 rows][128 B] | V same | Q [2 halves][8 rows][128 B]
constexpr int kDecStK = 0, kDecStV = 8192, kDecStQ = 16384;
constexpr int kDecStageBytes = 18432;
constexpr int kDecWarpBytes = kDecStages * kDecStageBytes;
// workspace head: tickets [kDecMaxSeqs * kDecMaxKvHeads] ints, then the
// scheduler words {next item, warps done}; all zero between calls
constexpr int kDecSchedOffset = kDecMaxSeqs * kDecMaxKvHeads * 4;
constexpr int kDecTicketBytes = kDecSchedOffset + 256;

struct DecodeArgs {
  const int* block_tables;
  int bt_stride, bt_width;
  const int* cu_q;
  const int* cu_k;
  int B, Hq, Hkv, G, page, q_box_rows;
  long long num_slots;
  float scale_log2;      // softmax_scale * log2(e)
  int* tickets;          // workspace head (see kDecTicketBytes)
  float* part_ml;        // [cap_items][Hq][2]
  float* part_o;         // [cap_items][Hq][128]
  long long cap_items;
  __nv_bfloat16* out;
  long long out_stride;
  unsigned* err;
};

struct DecTile {
  int b, h, c, npages, qrow;
  int ntok;     // valid tokens in the tile
  int first, last;
  long long row;  // cache row (slot) of the tile's first token
};

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
  int* sched = a.tickets + kDecSchedOffset / 4;   // {next item, warps done}

  if (lane == 0) {
    for (int i = 0; i < kDecStages; ++i) mbar_init(&s_bar[i], 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmQ);
  }

  // ---- plan: exclusive prefix sum of items per sequence (identical in every CTA)
  {
    const int tid = threadIdx.x;
    const int per = (a.B + 127) / 128;
    const int beg = min(a.B, tid * per), end = min(a.B, beg + per);
    int local = 0;
    for (int b = beg; b < end; ++b) {
      const int nq = a.cu_q[b + 1] - a.cu_q[b];
      const int nk = a.cu_k[b + 1] - a.cu_k[b];
      const int cnt = (nq >= 1 && nk > 0) ? (nk + kDecItem - 1) / kDecItem : 0;
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
    const int j0 = (c - s_start[b]) * kDecItem;
    const int nk = a.cu_k[b + 1] - a.cu_k[b];
    const int ntok_item = min(kDecItem, nk - j0);
    const int col = j0 / a.page;
    const long long blk = col < a.bt_width ? a.block_tables[(size_t)b * a.bt_stride + col] : -1;
    const long long row = blk * a.page + (j0 % a.page);
    cur.b = b; cur.h = h; cur.c = c;
    cur.npages = s_start[b + 1] - s_start[b];
    cur.qrow = a.cu_q[b];
    cur.ntok = ntok_item;
    cur.row = (blk < 0 || row + ntok_item > a.num_slots) ? -1 : row;
    if (cur.row < 0 && lane == 0) raise_error(a.err, ERR_BAD_INDEX);
    it_tiles = (ntok_item + kDecTile - 1) / kDecTile;
    it_k = 0;
  };
  grab_item();

  int issued = 0, valid_issued = 0;
  auto issue_next = [&]() {
    if (more) {
      const int s = issued % kDecStages;
      DecTile d = cur;
      // an invalid block loads rows 0.. of the cache and masks every token
      d.ntok = cur.row < 0 ? 0 : min(kDecTile, cur.ntok - it_k * kDecTile);
      d.first = it_k == 0;
      d.last = it_k == it_tiles - 1;
      d.row = cur.row < 0 ? 0 : cur.row + (long long)it_k * kDecTile;
      if (lane == 0) {
        s_desc[s] = d;
        const uint32_t st = wsmem + s * kDecStageBytes;
        const uint32_t bar = smem_u32(&s_bar[s]);
        fence_proxy_async_smem();
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

  const int g = lane >> 2;           // MMA row = query head inside the group
  const bool live_row = g < a.G;
  const int mi = lane >> 3, rin = lane & 7;
  uint32_t qa[8][4];
  float o[16][4];
  float m_run = -INFINITY, l_run = 0.f;
  int consumed = 0;

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
    }

    if (d.first) {
      // A fragments of Q: rows 0-7 = heads (rows >= G unused), rows 8-15 zero
#pragma unroll
      for (int kp = 0; kp < 4; ++kp) {
        ldmatrix_x4(sQ + tswz(1024, rin, 4 * kp + mi), qa[2 * kp][0], qa[2 * kp][2],
                    qa[2 * kp + 1][0], qa[2 * kp + 1][2]);
        qa[2 * kp][1] = qa[2 * kp][3] = qa[2 * kp + 1][1] = qa[2 * kp + 1][3] = 0u;
      }
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
      m_run = -INFINITY;
      l_run = 0.f;
    }

    // S = Q K^T over the tile's 32 tokens (4 n-tiles of 8)
    float sc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
    for (int kp = 0; kp < 4; ++kp) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(sK + tswz(4096, nt * 8 + rin, 4 * kp + mi), b0, b1, b2, b3);
        mma_bf16_16816(sc[nt], qa[2 * kp], b0, b1);
        mma_bf16_16816(sc[nt], qa[2 * kp + 1], b2, b3);
      }
    }
    float mt = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tok = nt * 8 + 2 * (lane & 3) + e;
        const float v = tok < d.ntok ? sc[nt][e] * a.scale_log2 : -INFINITY;
        sc[nt][e] = v;
        mt = fmaxf(mt, v);
      }
    }
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
    const float m_new = fmaxf(m_run, mt);
    const float alpha = m_run == -INFINITY ? 0.f : fast_exp2(m_run - m_new);
    m_run = m_new;
    float ls = 0.f;
    // P enters the PV MMA as bf16 hi + lo parts (hi = bf16(p), lo = bf16(p - hi)):
    // ~16 significant bits of p instead of 8.
    uint32_t ph2[2][4], pl[2][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const float p0 = m_new == -INFINITY ? 0.f : fast_exp2(sc[nt][0] - m_new);
      const float p1 = m_new == -INFINITY ? 0.f : fast_exp2(sc[nt][1] - m_new);
      ls += p0 + p1;
      const uint32_t hk = pack_bf16x2(p0, p1);
      const float2 hf = unpack_bf16x2(hk);
      const uint32_t lk = pack_bf16x2(p0 - hf.x, p1 - hf.y);
      const int kp = nt >> 1, hiw = (nt & 1) * 2;
      ph2[kp][hiw] = hk; ph2[kp][hiw + 1] = 0u;
      pl[kp][hiw] = lk; pl[kp][hiw + 1] = 0u;
    }
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    l_run = l_run * alpha + ls;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      o[dt][0] *= alpha;
      o[dt][1] *= alpha;
    }
    // O += P V (16 dim tiles of 8)
#pragma unroll
    for (int kp = 0; kp < 2; ++kp) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t v0, v1, v2, v3;
        ldmatrix_x4_trans(sV + tswz(4096, kp * 16 + 8 * (mi & 1) + rin, 2 * dp + (mi >> 1)), v0, v1, v2, v3);
        mma_bf16_16816(o[2 * dp], ph2[kp], v0, v1);
        mma_bf16_16816(o[2 * dp + 1], ph2[kp], v2, v3);
        mma_bf16_16816(o[2 * dp], pl[kp], v0, v1);
        mma_bf16_16816(o[2 * dp + 1], pl[kp], v2, v3);
      }
    }

    if (!d.last) continue;
    // ---- item done: output (single item) or partial + ticket
    const int hq = d.h * a.G + g;
    if (d.npages == 1) {
      if (live_row) {
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        __nv_bfloat16* dst = a.out + (size_t)d.qrow * a.out_stride + (size_t)hq * kDecHD;
#pragma unroll
        for (int dt = 0; dt < 16; ++dt)
          *reinterpret_cast<uint32_t*>(dst + dt * 8 + 2 * (lane & 3)) =
              pack_bf16x2(o[dt][0] * inv, o[dt][1] * inv);
      }
      continue;
    }
    if (live_row) {
      float* po = a.part_o + ((size_t)d.c * a.Hq + hq) * kDecHD;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt)
        *reinterpret_cast<float2*>(po + dt * 8 + 2 * (lane & 3)) = make_float2(o[dt][0], o[dt][1]);
      if ((lane & 3) == 0)
        *reinterpret_cast<float2*>(a.part_ml + ((size_t)d.c * a.Hq + hq) * 2) = make_float2(m_run, l_run);
    }
    __threadfence();
    __syncwarp();
    int ticket = 0;
    if (lane == 0) ticket = atomicAdd(a.tickets + (size_t)d.b * a.Hkv + d.h, 1);
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket != d.npages - 1) continue;
    __threadfence();
    // this warp merges the npages partials of (b, h): every lane loads the
    // (m, l) of one item at a time and the partial rows are read 8 items per
    // batch, so the merge is not a chain of dependent L2 round trips
    const int c0 = s_start[d.b];
    const int np = d.npages;
    for (int gg = 0; gg < a.G; ++gg) {
      const size_t hqq = (size_t)d.h * a.G + gg;
      float M = -INFINITY;
      for (int p0 = 0; p0 < np; p0 += 32) {
        if (p0 + lane < np) M = fmaxf(M, __ldcg(a.part_ml + ((size_t)(c0 + p0 + lane) * a.Hq + hqq) * 2));
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      float L = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int p0 = 0; p0 < np; p0 += 32) {
        float w = 0.f;
        if (p0 + lane < np) {
          const float2 ml = __ldcg(reinterpret_cast<const float2*>(a.part_ml + ((size_t)(c0 + p0 + lane) * a.Hq + hqq) * 2));
          w = fast_exp2(ml.x - M);
          L += w * ml.y;
        }
        const int cnt = min(32, np - p0);
        for (int j = 0; j < cnt; j += 8) {
          float4 ov[8];
          float wj[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            wj[u] = __shfl_sync(0xffffffffu, w, j + u);
            ov[u] = j + u < cnt
                        ? __ldcg(reinterpret_cast<const float4*>(a.part_o + ((size_t)(c0 + p0 + j + u) * a.Hq + hqq) * kDecHD) + lane)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            acc.x += wj[u] * ov[u].x; acc.y += wj[u] * ov[u].y;
            acc.z += wj[u] * ov[u].z; acc.w += wj[u] * ov[u].w;
          }
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
      const float inv = L > 0.f ? 1.f / L : 0.f;
      uint2 packed;
      packed.x = pack_bf16x2(acc.x * inv, acc.y * inv);
      packed.y = pack_bf16x2(acc.z * inv, acc.w * inv);
      *reinterpret_cast<uint2*>(a.out + (size_t)d.qrow * a.out_stride + hqq * kDecHD + lane * 4) = packed;
    }
    if (lane == 0) atomicExch(a.tickets + (size_t)d.b * a.Hkv + d.h, 0);
  }
  // drain: every issued tile has landed before the CTA's shared memory is released
  if (lane == 0) {
    for (int t = consumed; t < valid_issued; ++t)
      mbar_wait(&s_bar[t % kDecStages], (uint32_t)(t / kDecStages) & 1u, a.err);
  }
  __syncwarp();
}

}  // namespace b200
