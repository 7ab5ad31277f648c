// Memory-bound kernels of the decoder path: RMSNorm (+ fused residual add),
// q/k RMSNorm + neox RoPE + KV-cache store, the slot_mapping scatter,
// SiLU-and-mul, vocab-parallel embedding rows and greedy argmax.
//
// Rounding points follow the reference modules exactly (fp32 math, bf16
// results at the module boundaries), and multiply/add pairs use explicit
// round-to-nearest intrinsics where the reference evaluates them as separate
// fp32 operations, so that no FMA contraction changes the result.
#pragma once
#include "common.cuh"

namespace b200 {

constexpr int kHeadDimEW = 128;

// ---------------------------------------------------------------------------
// RMSNorm  (src/layers/layernorm.py:10-28)
//   normal:   out = bf16(w * (x * 1/sqrt(mean(x^2) + eps)))
//   residual: s = x + res (fp32); res_out = bf16(s); out = bf16(w * (s * ...))
// One CTA per row, 8 bf16 per vector, up to VPT vectors per thread.
// ---------------------------------------------------------------------------
template <int VPT, bool RESIDUAL>
__global__ void __launch_bounds__(256) rms_norm_kernel(const __nv_bfloat16* __restrict__ x,
                                                       long long x_stride,
                                                       const __nv_bfloat16* __restrict__ res,
                                                       const __nv_bfloat16* __restrict__ w,
                                                       __nv_bfloat16* __restrict__ out,
                                                       long long out_stride,
                                                       __nv_bfloat16* __restrict__ res_out,
                                                       int dim, float eps) {
  __shared__ float s_red[8];
  const int row = blockIdx.x;
  const int nvec = dim / 8;
  // the norm weights are parameters (no kernel of the step writes them): their
  // loads are issued first and overlap the previous kernel and the row loads
  uint4 wv[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    wv[i] = vi < nvec ? *reinterpret_cast<const uint4*>(w + vi * 8) : make_uint4(0u, 0u, 0u, 0u);
  }
  griddep_wait();
  griddep_launch_dependents();
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      const uint4 raw = *reinterpret_cast<const uint4*>(x + (size_t)row * x_stride + vi * 8);
      const uint32_t* rw = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(rw[k]);
        v[i][2 * k] = f.x;
        v[i][2 * k + 1] = f.y;
      }
      if (RESIDUAL) {
        const uint4 rr = *reinterpret_cast<const uint4*>(res + (size_t)row * dim + vi * 8);
        const uint32_t* rp = reinterpret_cast<const uint32_t*>(&rr);
        uint4 packed;
        uint32_t* pk = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_bf16x2(rp[k]);
          v[i][2 * k] = __fadd_rn(v[i][2 * k], f.x);
          v[i][2 * k + 1] = __fadd_rn(v[i][2 * k + 1], f.y);
          pk[k] = pack_bf16x2(v[i][2 * k], v[i][2 * k + 1]);
        }
        *reinterpret_cast<uint4*>(res_out + (size_t)row * dim + vi * 8) = packed;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += v[i][k] * v[i][k];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += s_red[i];
  const float var = __fadd_rn(tot / (float)dim, eps);
  const float inv = 1.0f / sqrtf(var);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      const uint32_t* wp = reinterpret_cast<const uint32_t*>(&wv[i]);
      uint4 packed;
      uint32_t* pk = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 wf = unpack_bf16x2(wp[k]);
        const float a0 = __fmul_rn(wf.x, __fmul_rn(v[i][2 * k], inv));
        const float a1 = __fmul_rn(wf.y, __fmul_rn(v[i][2 * k + 1], inv));
        pk[k] = pack_bf16x2(a0, a1);
      }
      *reinterpret_cast<uint4*>(out + (size_t)row * out_stride + vi * 8) = packed;
    }
  }
}

// ---------------------------------------------------------------------------
// q/k RMSNorm + neox RoPE + K/V cache store for one token row of the fused
// qkv projection (src/models/qwen3.py:80-89, src/layers/pos_embedding.py:30-52,
// src/layers/attention.py:10-34).  One warp per (token, head); lane l holds
// dims {2l, 2l+1} and {2l+64, 2l+65}, i.e. both halves of its RoPE pairs.
//   heads [0, Hq)            q: norm -> rope -> q_out
//   heads [Hq, Hq+Hkv)       k: norm -> rope -> k_out and cache[slot]
//   heads [Hq+Hkv, Hq+2Hkv)  v: copy          -> v_out and cache[slot]
// ---------------------------------------------------------------------------
struct QKNormRopeArgs {
  const __nv_bfloat16* q_in;   // [T] rows of Hq heads, token stride q_in_stride
  const __nv_bfloat16* k_in;   // [T] rows of Hkv heads
  const __nv_bfloat16* v_in;   // [T] rows of Hkv heads, or nullptr (rope only)
  long long q_in_stride, k_in_stride, v_in_stride;
  int T, Hq, Hkv;
  const __nv_bfloat16* q_w;  // [128] or nullptr (no q/k norm: qkv_bias models)
  const __nv_bfloat16* k_w;
  float eps;
  const float* cos_sin;      // [max_pos][128] = [cos(64) | sin(64)]
  const long long* positions;
  long long max_pos;
  const int* slot_mapping;   // [T] or nullptr
  __nv_bfloat16* k_cache;    // [num_slots][Hkv][128] or nullptr
  __nv_bfloat16* v_cache;
  long long num_slots;
  __nv_bfloat16* q_out;      // [T][Hq][128]
  __nv_bfloat16* k_out;      // [T][Hkv][128] or nullptr
  __nv_bfloat16* v_out;
  unsigned* err;
};

__global__ void __launch_bounds__(256) qk_norm_rope_store_kernel(const QKNormRopeArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = a.Hq + (a.v_in ? 2 : 1) * a.Hkv;
  const long long total = (long long)a.T * heads;
  for (long long wi = (long long)blockIdx.x * warps + (threadIdx.x >> 5); wi < total;
       wi += (long long)gridDim.x * warps) {
    const int t = (int)(wi / heads);
    const int hh = (int)(wi - (long long)t * heads);
    const __nv_bfloat16* src;
    if (hh < a.Hq) src = a.q_in + (size_t)t * a.q_in_stride + (size_t)hh * kHeadDimEW;
    else if (hh < a.Hq + a.Hkv) src = a.k_in + (size_t)t * a.k_in_stride + (size_t)(hh - a.Hq) * kHeadDimEW;
    else src = a.v_in + (size_t)t * a.v_in_stride + (size_t)(hh - a.Hq - a.Hkv) * kHeadDimEW;
    uint32_t lo = *reinterpret_cast<const uint32_t*>(src + 2 * lane);
    uint32_t hi = *reinterpret_cast<const uint32_t*>(src + 64 + 2 * lane);
    const int slot = a.slot_mapping ? a.slot_mapping[t] : -1;
    const bool store = a.k_cache != nullptr && slot >= 0;
    if (a.k_cache != nullptr && (slot < -1 || (long long)slot >= a.num_slots)) {
      if (lane == 0 && hh == a.Hq) raise_error(a.err, ERR_BAD_INDEX);
    }
    const bool slot_ok = store && (long long)slot < a.num_slots;
    if (hh >= a.Hq + a.Hkv) {
      const int vh = hh - a.Hq - a.Hkv;
      if (a.v_out) {
        __nv_bfloat16* d = a.v_out + ((size_t)t * a.Hkv + vh) * kHeadDimEW;
        *reinterpret_cast<uint32_t*>(d + 2 * lane) = lo;
        *reinterpret_cast<uint32_t*>(d + 64 + 2 * lane) = hi;
      }
      if (slot_ok) {
        __nv_bfloat16* d = a.v_cache + ((size_t)slot * a.Hkv + vh) * kHeadDimEW;
        *reinterpret_cast<uint32_t*>(d + 2 * lane) = lo;
        *reinterpret_cast<uint32_t*>(d + 64 + 2 * lane) = hi;
      }
      continue;
    }
    const bool is_q = hh < a.Hq;
    float2 x0 = unpack_bf16x2(lo), x1 = unpack_bf16x2(hi);
    const __nv_bfloat16* nw = is_q ? a.q_w : a.k_w;
    if (nw != nullptr) {
      float ss = x0.x * x0.x + x0.y * x0.y + x1.x * x1.x + x1.y * x1.y;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv = 1.0f / sqrtf(__fadd_rn(ss / 128.0f, a.eps));
      const float2 w0 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(nw + 2 * lane));
      const float2 w1 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(nw + 64 + 2 * lane));
      x0.x = bf16_round(__fmul_rn(w0.x, __fmul_rn(x0.x, inv)));
      x0.y = bf16_round(__fmul_rn(w0.y, __fmul_rn(x0.y, inv)));
      x1.x = bf16_round(__fmul_rn(w1.x, __fmul_rn(x1.x, inv)));
      x1.y = bf16_round(__fmul_rn(w1.y, __fmul_rn(x1.y, inv)));
    }
    long long pos = a.positions[t];
    if (pos < 0 || pos >= a.max_pos) {
      if (lane == 0) raise_error(a.err, ERR_BAD_INDEX);
      pos = pos < 0 ? 0 : a.max_pos - 1;
    }
    const float* cs = a.cos_sin + (size_t)pos * kHeadDimEW;
    const float2 c = *reinterpret_cast<const float2*>(cs + 2 * lane);
    const float2 s = *reinterpret_cast<const float2*>(cs + 64 + 2 * lane);
    // t1' = t1*cos - t2*sin ; t2' = t1*sin + t2*cos
    const float r0x = __fsub_rn(__fmul_rn(x0.x, c.x), __fmul_rn(x1.x, s.x));
    const float r0y = __fsub_rn(__fmul_rn(x0.y, c.y), __fmul_rn(x1.y, s.y));
    const float r1x = __fadd_rn(__fmul_rn(x0.x, s.x), __fmul_rn(x1.x, c.x));
    const float r1y = __fadd_rn(__fmul_rn(x0.y, s.y), __fmul_rn(x1.y, c.y));
    lo = pack_bf16x2(r0x, r0y);
    hi = pack_bf16x2(r1x, r1y);
    if (is_q) {
      __nv_bfloat16* d = a.q_out + ((size_t)t * a.Hq + hh) * kHeadDimEW;
      *reinterpret_cast<uint32_t*>(d + 2 * lane) = lo;
      *reinterpret_cast<uint32_t*>(d + 64 + 2 * lane) = hi;
    } else {
      const int kh = hh - a.Hq;
      if (a.k_out) {
        __nv_bfloat16* d = a.k_out + ((size_t)t * a.Hkv + kh) * kHeadDimEW;
        *reinterpret_cast<uint32_t*>(d + 2 * lane) = lo;
        *reinterpret_cast<uint32_t*>(d + 64 + 2 * lane) = hi;
      }
      if (slot_ok) {
        __nv_bfloat16* d = a.k_cache + ((size_t)slot * a.Hkv + kh) * kHeadDimEW;
        *reinterpret_cast<uint32_t*>(d + 2 * lane) = lo;
        *reinterpret_cast<uint32_t*>(d + 64 + 2 * lane) = hi;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// store_kvcache  (src/layers/attention.py:10-61)
// cache.view(-1, D)[slot[i]] = key[i] (and value), slot -1 skipped.
// 16-byte vectors; a grid-stride loop over (token, vector).
// ---------------------------------------------------------------------------
__global__ void store_kvcache_kernel(const __nv_bfloat16* __restrict__ key, long long key_stride,
                                     const __nv_bfloat16* __restrict__ value,
                                     long long value_stride, __nv_bfloat16* __restrict__ k_cache,
                                     __nv_bfloat16* __restrict__ v_cache,
                                     const int* __restrict__ slot_mapping, int T, int D,
                                     long long num_slots, unsigned* err) {
  griddep_wait();
  griddep_launch_dependents();
  const int vpt = D / 8;  // 16-byte vectors per token row
  const long long total = (long long)T * vpt;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / vpt);
    const int v = (int)(i - (long long)t * vpt);
    const int slot = slot_mapping[t];
    if (slot == -1) continue;
    if (slot < -1 || (long long)slot >= num_slots) {
      if (v == 0) raise_error(err, ERR_BAD_INDEX);
      continue;
    }
    const uint4 kv = *reinterpret_cast<const uint4*>(key + (size_t)t * key_stride + v * 8);
    const uint4 vv = *reinterpret_cast<const uint4*>(value + (size_t)t * value_stride + v * 8);
    *reinterpret_cast<uint4*>(k_cache + (size_t)slot * D + v * 8) = kv;
    *reinterpret_cast<uint4*>(v_cache + (size_t)slot * D + v * 8) = vv;
  }
}

// ---------------------------------------------------------------------------
// SiLU-and-mul (src/layers/activation.py:6-10): out = silu(x[:, :I]) * x[:, I:]
// ---------------------------------------------------------------------------
__global__ void silu_and_mul_kernel(const __nv_bfloat16* __restrict__ x, long long x_stride,
                                    __nv_bfloat16* __restrict__ out, long long out_stride, int T,
                                    int I) {
  griddep_wait();
  griddep_launch_dependents();
  const int vpr = I / 8;
  const long long total = (long long)T * vpr;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / vpr);
    const int c = (int)(i - (long long)t * vpr) * 8;
    const uint4 g = *reinterpret_cast<const uint4*>(x + (size_t)t * x_stride + c);
    const uint4 u = *reinterpret_cast<const uint4*>(x + (size_t)t * x_stride + I + c);
    const uint32_t* gp = reinterpret_cast<const uint32_t*>(&g);
    const uint32_t* up = reinterpret_cast<const uint32_t*>(&u);
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 gf = unpack_bf16x2(gp[k]);
      const float2 uf = unpack_bf16x2(up[k]);
      const float s0 = bf16_round(gf.x / (1.0f + expf(-gf.x)));
      const float s1 = bf16_round(gf.y / (1.0f + expf(-gf.y)));
      op[k] = pack_bf16x2(__fmul_rn(s0, uf.x), __fmul_rn(s1, uf.y));
    }
    *reinterpret_cast<uint4*>(out + (size_t)t * out_stride + c) = o;
  }
}

// ---------------------------------------------------------------------------
// VocabParallelEmbedding local part (src/layers/llm_head.py:38-49):
// out[t] = W[id - start] if start <= id < end else 0.
// ---------------------------------------------------------------------------
__global__ void embedding_kernel(const long long* __restrict__ ids,
                                 const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                 int T, int H, long long start, long long end, unsigned* err) {
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
    if (id >= start && id < end) v = *reinterpret_cast<const uint4*>(w + (size_t)(id - start) * H + c);
    *reinterpret_cast<uint4*>(out + (size_t)t * H + c) = v;
  }
}

// ---------------------------------------------------------------------------
// Greedy argmax over the vocabulary (first index of the maximum, like
// torch.argmax).  One CTA per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) argmax_kernel(const __nv_bfloat16* __restrict__ logits,
                                                      long long stride, int V,
                                                      long long* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float s_v[32];
  __shared__ int s_i[32];
  const int row = blockIdx.x;
  const __nv_bfloat16* lp = logits + (size_t)row * stride;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  auto take = [&](float v, int i) {
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
  };
  int scalar_from = 0;
  if ((reinterpret_cast<uintptr_t>(lp) & 15) == 0) {
    // 16-byte loads (8 logits), four in flight per thread
    const int nv = V >> 3;
    const uint4* vp = reinterpret_cast<const uint4*>(lp);
    for (int j = threadIdx.x; j < nv; j += 4 * blockDim.x) {
      uint4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int jj = j + u * (int)blockDim.x;
        q[u] = jj < nv ? __ldg(vp + jj) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int jj = j + u * (int)blockDim.x;
        if (jj >= nv) continue;
        const uint32_t w[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          take(__uint_as_float(w[k] << 16), jj * 8 + 2 * k);
          take(__uint_as_float(w[k] & 0xffff0000u), jj * 8 + 2 * k + 1);
        }
      }
    }
    scalar_from = nv << 3;
  }
  for (int i = scalar_from + (int)threadIdx.x; i < V; i += blockDim.x) take(__bfloat162float(lp[i]), i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { s_v[warp] = best; s_i[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? s_v[lane] : -INFINITY;
    bi = lane < nw ? s_i[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) out[row] = bi == 0x7fffffff ? 0 : bi;
  }
}

}  // namespace b200
