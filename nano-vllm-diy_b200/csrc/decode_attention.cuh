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
//   warp  = owns whole items; a persistent grid (one 4-warp CTA per SM)
//           hands items to warps round-robin.  Each warp runs its own
//           3-stage cp.async ring of 32-token K/V tiles (+ the item's Q rows
//           with its first tile) that keeps streaming across item
//           boundaries, so loads stay in flight while the warp computes and
//           no CTA-wide barrier is ever taken.
//   combine = a sequence spanning several items writes per-item partials
//           (m, l, o); the warp that finishes the last item of (sequence,
//           kv head) -- found with an atomic ticket -- merges them and writes
//           the output, then resets the ticket for the next call.  A
//           single-item sequence writes its output directly.
// The launch shape depends only on B and the SM count, never on the context
// lengths, which are read from cu_seqlens_k on the device (CUDA-graph safe;
// rows with q length <= 0 are graph padding and are skipped).
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
constexpr int kDecStageBytes = 2 * kDecTile * 256 + 8 * 256;   // K + V + Q rows
constexpr int kDecWarpBytes = kDecStages * kDecStageBytes;
constexpr int kDecTicketBytes = kDecMaxSeqs * kDecMaxKvHeads * 4;  // workspace head

struct DecTile;
__host__ __device__ constexpr int dec_smem_bytes();

struct DecodeArgs {
  const __nv_bfloat16* q;
  long long q_stride;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  const int* block_tables;
  int bt_stride, bt_width;
  const int* cu_q;
  const int* cu_k;
  int B, Hq, Hkv, G, page;
  long long num_slots;
  float scale_log2;      // softmax_scale * log2(e)
  int* tickets;          // [kDecMaxSeqs * kDecMaxKvHeads], zero between calls
  float* part_ml;        // [cap_items][Hq][2]
  float* part_o;         // [cap_items][Hq][128]
  long long cap_items;
  __nv_bfloat16* out;
  long long out_stride;
  unsigned* err;
};

struct DecTile {
  int b, h, c, npages, qrow;
  int tok0;     // first token of the tile inside the sequence
  int ntok;     // valid tokens in the tile
  int first, last;
  long long row0;  // cache row (slot) of token tok0, -1 if the block is invalid
};

__host__ __device__ constexpr int dec_smem_bytes() {
  return kDecWarps * kDecWarpBytes + kDecWarps * kDecStages * (int)sizeof(DecTile) +
         (8 + kDecMaxSeqs + 1) * (int)sizeof(int);
}

__device__ __forceinline__ uint32_t dswz(int r, int ch) {
  return (uint32_t)(r * 256 + ((ch ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(128, 1) decode_attn_kernel(const DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // layout: [warp rings][tile descriptors][scan scratch][plan]
  DecTile* s_desc = reinterpret_cast<DecTile*>(smem + kDecWarps * kDecWarpBytes) + warp * kDecStages;
  int* s_scan = reinterpret_cast<int*>(smem + kDecWarps * kDecWarpBytes +
                                       kDecWarps * kDecStages * sizeof(DecTile));
  int* s_start = s_scan + 8;

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
  const int gwarp = blockIdx.x * kDecWarps + warp;
  const int nwarps = gridDim.x * kDecWarps;

  uint8_t* wbase = smem + warp * kDecWarpBytes;
  const uint32_t wsmem = smem_u32(wbase);

  // ---- tile iterator (uniform across the warp)
  int it_w = gwarp;       // current item
  int it_k = 0;           // next tile inside it
  int it_tiles = 0;
  DecTile cur{};
  auto decode_item = [&](int w) {
    const int c = w / a.Hkv;
    const int h = w - c * a.Hkv;
    int lo = 0, hi = a.B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_start[mid] <= c) lo = mid; else hi = mid - 1;
    }
    const int b = lo;
    const int p = c - s_start[b];
    const int nk = a.cu_k[b + 1] - a.cu_k[b];
    cur.b = b; cur.h = h; cur.c = c;
    cur.npages = s_start[b + 1] - s_start[b];
    cur.qrow = a.cu_q[b];
    const int j0 = p * kDecItem;
    const int ntok_item = min(kDecItem, nk - j0);
    const int col = j0 / a.page;
    const long long blk = col < a.bt_width ? a.block_tables[(size_t)b * a.bt_stride + col] : -1;
    const long long row = blk * a.page + (j0 % a.page);
    cur.row0 = (blk < 0 || row + ntok_item > a.num_slots) ? -1 : row;
    if (cur.row0 < 0 && lane == 0) raise_error(a.err, ERR_BAD_INDEX);
    cur.tok0 = j0;
    cur.ntok = ntok_item;  // item-level for now
    it_tiles = (ntok_item + kDecTile - 1) / kDecTile;
    it_k = 0;
  };
  if (it_w < items) decode_item(it_w);

  int issued = 0, valid_issued = 0;
  auto issue_next = [&]() {
    if (it_w < items) {
      const int s = issued % kDecStages;
      DecTile d = cur;
      d.tok0 = cur.tok0 + it_k * kDecTile;
      d.ntok = min(kDecTile, cur.ntok - it_k * kDecTile);
      d.first = it_k == 0;
      d.last = it_k == it_tiles - 1;
      if (lane == 0) s_desc[s] = d;
      const uint32_t sK = wsmem + s * kDecStageBytes;
      const uint32_t sV = sK + kDecTile * 256;
      const uint32_t sQ = sV + kDecTile * 256;
      const long long row_tile = d.row0 < 0 ? -1 : d.row0 + (long long)it_k * kDecTile;
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int idx = lane + 32 * i;
        const int r = idx >> 4, ch = idx & 15;
        const bool valid = r < d.ntok && row_tile >= 0;
        const size_t off = valid ? ((size_t)(row_tile + r) * a.Hkv + d.h) * kDecHD + ch * 8 : 0;
        cp_async_16_zfill(sK + dswz(r, ch), a.k_cache + off, valid);
        cp_async_16_zfill(sV + dswz(r, ch), a.v_cache + off, valid);
      }
      if (d.first) {
        for (int idx = lane; idx < a.G * 16; idx += 32) {
          const int g = idx >> 4, ch = idx & 15;
          cp_async_16(sQ + g * 256 + ch * 16,
                      a.q + (size_t)d.qrow * a.q_stride + (size_t)(d.h * a.G + g) * kDecHD + ch * 8);
        }
      }
      ++valid_issued;
      if (++it_k == it_tiles) {
        it_w += nwarps;
        if (it_w < items) decode_item(it_w);
      }
    }
    cp_async_commit();
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

  for (int t = 0; t < valid_issued; ++t) {
    cp_async_wait<1>();
    __syncwarp();
    issue_next();
    const int s = t % kDecStages;
    const DecTile d = s_desc[s];
    const uint32_t sK = wsmem + s * kDecStageBytes;
    const uint32_t sV = sK + kDecTile * 256;
    const uint8_t* sQp = wbase + s * kDecStageBytes + 2 * kDecTile * 256;

    if (d.first) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int dd = ks * 16 + 2 * (lane & 3);
        qa[ks][0] = live_row ? *reinterpret_cast<const uint32_t*>(sQp + g * 256 + dd * 2) : 0u;
        qa[ks][1] = 0u;
        qa[ks][2] = live_row ? *reinterpret_cast<const uint32_t*>(sQp + g * 256 + (dd + 8) * 2) : 0u;
        qa[ks][3] = 0u;
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
        ldmatrix_x4(sK + dswz(nt * 8 + rin, 4 * kp + mi), b0, b1, b2, b3);
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
    uint32_t ph[2][4], pl[2][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const float p0 = fast_exp2(sc[nt][0] - m_new);
      const float p1 = fast_exp2(sc[nt][1] - m_new);
      ls += p0 + p1;
      const uint32_t hk = pack_bf16x2(p0, p1);
      const float2 hf = unpack_bf16x2(hk);
      const uint32_t lk = pack_bf16x2(p0 - hf.x, p1 - hf.y);
      const int kp = nt >> 1, hiw = (nt & 1) * 2;
      ph[kp][hiw] = hk; ph[kp][hiw + 1] = 0u;
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
        ldmatrix_x4_trans(sV + dswz(kp * 16 + 8 * (mi & 1) + rin, 2 * dp + (mi >> 1)), v0, v1, v2, v3);
        mma_bf16_16816(o[2 * dp], ph[kp], v0, v1);
        mma_bf16_16816(o[2 * dp + 1], ph[kp], v2, v3);
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
    // this warp merges the npages partials of (b, h)
    const int c0 = s_start[d.b];
    for (int gg = 0; gg < a.G; ++gg) {
      const size_t hqq = (size_t)d.h * a.G + gg;
      float M = -INFINITY;
      for (int p = lane; p < d.npages; p += 32)
        M = fmaxf(M, __ldcg(a.part_ml + ((size_t)(c0 + p) * a.Hq + hqq) * 2));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      float L = 0.f;
      for (int p = lane; p < d.npages; p += 32) {
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(a.part_ml + ((size_t)(c0 + p) * a.Hq + hqq) * 2));
        L += fast_exp2(ml.x - M) * ml.y;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int p = 0; p < d.npages; ++p) {
        const float w = fast_exp2(__ldcg(a.part_ml + ((size_t)(c0 + p) * a.Hq + hqq) * 2) - M);
        const float4 ov = __ldcg(reinterpret_cast<const float4*>(a.part_o + ((size_t)(c0 + p) * a.Hq + hqq) * kDecHD) + lane);
        acc.x += w * ov.x; acc.y += w * ov.y; acc.z += w * ov.z; acc.w += w * ov.w;
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      uint2 packed;
      packed.x = pack_bf16x2(acc.x * inv, acc.y * inv);
      packed.y = pack_bf16x2(acc.z * inv, acc.w * inv);
      *reinterpret_cast<uint2*>(a.out + (size_t)d.qrow * a.out_stride + hqq * kDecHD + lane * 4) = packed;
    }
    if (lane == 0) atomicExch(a.tickets + (size_t)d.b * a.Hkv + d.h, 0);
  }
  cp_async_wait<0>();
}

}  // namespace b200
