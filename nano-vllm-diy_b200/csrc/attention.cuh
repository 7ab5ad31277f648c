// Paged, varlen, causal GQA attention for head_dim 128.
//
// Device side of src/layers/attention.py:79-104 (Attention.forward ->
// flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
// max_seqlen_k, softmax_scale, causal=True, block_table)).  Semantics kept:
//   * query i of a sequence (0-based inside its q chunk of length Lq) sees
//     keys j <= i + Lk - Lq (causal, bottom-right aligned);
//   * q head n reads kv head n / (Hq / Hkv);
//   * with a block table, key j of sequence b lives in cache row
//     block_table[b][j / page] * page + j % page of a [num_blocks, page,
//     Hkv, 128] cache; without one, in row cu_seqlens_k[b] + j of k / v;
//   * lengths are read on the device from cu_seqlens_*; a sequence whose
//     query length is <= 0 (CUDA-graph padding) is skipped.
//
// This file holds prefill_attn_kernel (prefill, chunked prefill, prefix
// hits and mixed batches): FA2-style, 64 queries x 1 head per CTA, K/V tiles
// of 64 keys double-buffered with cp.async, online softmax in registers, P
// fed to the PV MMA as bf16 hi + lo parts.  Pure-decode batches use
// decode_attention.cuh.
#pragma once
#include "common.cuh"

namespace b200 {

constexpr int kHD = 128;          // head_dim

// Swizzled byte offset of 16-byte chunk `ch` of row `r` in a [rows][256 B]
// tile: chunk index XOR (row % 8) makes every ldmatrix phase conflict-free.
__device__ __forceinline__ uint32_t swz(int r, int ch) {
  return (uint32_t)(r * 256 + ((ch ^ (r & 7)) << 4));
}

// ---------------------------------------------------------------------------
// prefill / mixed batches
// ---------------------------------------------------------------------------
struct PrefillArgs {
  const __nv_bfloat16* q;
  long long q_stride;
  const __nv_bfloat16* k;  // contiguous K/V source when block_tables == nullptr
  const __nv_bfloat16* v;
  long long k_stride, v_stride;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  const int* block_tables;
  int bt_stride;
  int bt_width;
  long long num_slots;
  const int* cu_q;
  const int* cu_k;
  int B, Hq, Hkv, G, page;
  float scale_log2;
  __nv_bfloat16* out;
  long long out_stride;
  unsigned* err;
};

constexpr int kPfBM = 64;  // queries per CTA
constexpr int kPfBN = 64;  // keys per tile

__global__ void __launch_bounds__(128) prefill_attn_kernel(const PrefillArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;                    // 64 x 256 B
  uint8_t* sK = smem + 16384;            // 2 stages x 64 x 256 B
  uint8_t* sV = smem + 16384 + 32768;    // 2 stages

  const int b = blockIdx.z, hq = blockIdx.y, h = hq / a.G;
  const int q0 = a.cu_q[b];
  const int Lq = a.cu_q[b + 1] - q0;
  const int i0 = blockIdx.x * kPfBM;
  if (Lq <= 0 || i0 >= Lq) return;
  const int Lk = a.cu_k[b + 1] - a.cu_k[b];
  const int off = Lk - Lq;
  const int key_end = max(0, min(Lk, i0 + kPfBM + off));  // exclusive
  const int ntiles = (key_end + kPfBN - 1) / kPfBN;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int* bt = a.block_tables ? a.block_tables + (size_t)b * a.bt_stride : nullptr;

  // Q tile (rows >= Lq zero-filled)
  for (int idx = tid; idx < kPfBM * 16; idx += 128) {
    const int r = idx >> 4, ch = idx & 15;
    const bool valid = i0 + r < Lq;
    const __nv_bfloat16* src = valid ? a.q + (size_t)(q0 + i0 + r) * a.q_stride + (size_t)hq * kHD + ch * 8 : a.q;
    cp_async_16_zfill(smem_u32(sQ) + swz(r, ch), src, valid);
  }
  cp_async_commit();

  auto load_kv = [&](int tile, int stage) {
    const int jb = tile * kPfBN;
    for (int idx = tid; idx < kPfBN * 16; idx += 128) {
      const int r = idx >> 4, ch = idx & 15;
      const int j = jb + r;
      bool valid = j < key_end;
      const __nv_bfloat16* ks = a.k_cache ? a.k_cache : a.k;
      const __nv_bfloat16* vs = ks;
      if (valid) {
        if (bt) {
          const int col = j / a.page;
          const long long blk = col < a.bt_width ? bt[col] : -1;
          const long long slot = blk * a.page + (j % a.page);
          if (blk < 0 || slot >= a.num_slots) {
            raise_error(a.err, ERR_BAD_INDEX);
            valid = false;
          } else {
            ks = a.k_cache + ((size_t)slot * a.Hkv + h) * kHD + ch * 8;
            vs = a.v_cache + ((size_t)slot * a.Hkv + h) * kHD + ch * 8;
          }
        } else {
          const size_t row = (size_t)(a.cu_k[b] + j);
          ks = a.k + row * a.k_stride + (size_t)h * kHD + ch * 8;
          vs = a.v + row * a.v_stride + (size_t)h * kHD + ch * 8;
        }
      }
      cp_async_16_zfill(smem_u32(sK + stage * 16384) + swz(r, ch), ks, valid);
      cp_async_16_zfill(smem_u32(sV + stage * 16384) + swz(r, ch), vs, valid);
    }
    cp_async_commit();
  };

  if (ntiles > 0) load_kv(0, 0);

  float o[16][4];
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY};
  float l_r[2] = {0.f, 0.f};
  uint32_t qa[8][4];
  const int mi = lane >> 3, rin = lane & 7;
  const int row_a = i0 + warp * 16 + (lane >> 2);  // rows held by this thread: row_a, row_a + 8

  for (int t = 0; t < ntiles; ++t) {
    if (t + 1 < ntiles) {
      load_kv(t + 1, (t + 1) & 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (t == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int r = warp * 16 + 8 * (mi & 1) + rin;
        ldmatrix_x4(smem_u32(sQ) + swz(r, 2 * ks + (mi >> 1)), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
      }
    }
    const uint32_t sKs = smem_u32(sK + (t & 1) * 16384);
    const uint32_t sVs = smem_u32(sV + (t & 1) * 16384);

    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int kp = 0; kp < 4; ++kp) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(sKs + swz(nt * 8 + rin, 4 * kp + mi), b0, b1, b2, b3);
        mma_bf16_16816(s[nt], qa[2 * kp], b0, b1);
        mma_bf16_16816(s[nt], qa[2 * kp + 1], b2, b3);
      }
    }
    // mask + online softmax; c-frag: [0,1] row_a, [2,3] row_a + 8
    float mt[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = row_a + (e >> 1) * 8;
        const int j = t * kPfBN + nt * 8 + 2 * (lane & 3) + (e & 1);
        const bool ok = j < Lk && j <= i + off;
        const float v = ok ? s[nt][e] * a.scale_log2 : -INFINITY;
        s[nt][e] = v;
        mt[e >> 1] = fmaxf(mt[e >> 1], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      mt[rr] = fmaxf(mt[rr], __shfl_xor_sync(0xffffffffu, mt[rr], 1));
      mt[rr] = fmaxf(mt[rr], __shfl_xor_sync(0xffffffffu, mt[rr], 2));
      const float mnew = fmaxf(m_r[rr], mt[rr]);
      alpha[rr] = (m_r[rr] == -INFINITY) ? 0.f : fast_exp2(m_r[rr] - mnew);
      m_r[rr] = mnew;
    }
    float ls[2] = {0.f, 0.f};
    uint32_t pa[4][4], pl[4][4];  // bf16 hi / lo parts of P (see decode kernel)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        p[e] = (mm == -INFINITY) ? 0.f : fast_exp2(s[nt][e] - mm);
        ls[e >> 1] += p[e];
      }
      const uint32_t h01 = pack_bf16x2(p[0], p[1]);
      const uint32_t h23 = pack_bf16x2(p[2], p[3]);
      const float2 f01 = unpack_bf16x2(h01), f23 = unpack_bf16x2(h23);
      const uint32_t l01 = pack_bf16x2(p[0] - f01.x, p[1] - f01.y);
      const uint32_t l23 = pack_bf16x2(p[2] - f23.x, p[3] - f23.y);
      const int kp = nt >> 1;
      if ((nt & 1) == 0) {
        pa[kp][0] = h01; pa[kp][1] = h23;
        pl[kp][0] = l01; pl[kp][1] = l23;
      } else {
        pa[kp][2] = h01; pa[kp][3] = h23;
        pl[kp][2] = l01; pl[kp][3] = l23;
      }
    }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      ls[rr] += __shfl_xor_sync(0xffffffffu, ls[rr], 1);
      ls[rr] += __shfl_xor_sync(0xffffffffu, ls[rr], 2);
      l_r[rr] = l_r[rr] * alpha[rr] + ls[rr];
    }
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      o[dt][0] *= alpha[0]; o[dt][1] *= alpha[0];
      o[dt][2] *= alpha[1]; o[dt][3] *= alpha[1];
    }
#pragma unroll
    for (int kp = 0; kp < 4; ++kp) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t v0, v1, v2, v3;
        const int r = kp * 16 + 8 * (mi & 1) + rin;
        ldmatrix_x4_trans(sVs + swz(r, 2 * dp + (mi >> 1)), v0, v1, v2, v3);
        mma_bf16_16816(o[2 * dp], pa[kp], v0, v1);
        mma_bf16_16816(o[2 * dp + 1], pa[kp], v2, v3);
        mma_bf16_16816(o[2 * dp], pl[kp], v0, v1);
        mma_bf16_16816(o[2 * dp + 1], pl[kp], v2, v3);
      }
    }
    __syncthreads();  // stage (t & 1) is refilled two iterations later
  }

  // epilogue: rows with no visible key (l == 0) are written as zeros
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int i = row_a + rr * 8;
    if (i >= Lq) continue;
    const float inv = l_r[rr] > 0.f ? 1.f / l_r[rr] : 0.f;
    __nv_bfloat16* dst = a.out + (size_t)(q0 + i) * a.out_stride + (size_t)hq * kHD;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      const int d = dt * 8 + 2 * (lane & 3);
      *reinterpret_cast<uint32_t*>(dst + d) = pack_bf16x2(o[dt][rr * 2] * inv, o[dt][rr * 2 + 1] * inv);
    }
  }
}

}  // namespace b200
