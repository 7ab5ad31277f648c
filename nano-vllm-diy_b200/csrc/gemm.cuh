// Y[T, N] = X[T, K] * W[N, K]^T  (+ bias) on 5th-generation tensor cores.
//
// This is the device side of the reference's F.linear calls
// (src/layers/linear.py:75 ColumnParallelLinear.forward, :170
// RowParallelLinear.forward, src/layers/llm_head.py:64 ParallelLMHead).
//
// Tiling ("swap-AB"): the weight is the M operand (128 output features per
// CTA) and the tokens are the N operand (BN = 32..256 tokens per CTA), so a
// decode batch of B <= 256 tokens is a single N tile and every CTA streams a
// disjoint 128-row slab of W from HBM exactly once.  Both operands are
// K-major in global memory (W is [out, in] row-major, X is [T, in]), which is
// what the tcgen05 K-major shared-memory descriptors want.
//
// Roles (192 threads):
//   warp 0      TMA producer (one lane): W box 64x128, X box 64xBN, 128-byte
//               swizzle, into an S-stage ring guarded by full/empty mbarriers
//   warp 1      TMEM allocator + MMA issuer (one lane): 4 x tcgen05.mma
//               (M=128, N=BN, K=16) per 64-wide K block, accumulators in TMEM
//   warps 2..5  epilogue: tcgen05.ld 32x32b -> registers -> global
//
// Epilogues:
//   EPI_BF16     y = bf16(acc + bias)                       (split == 1)
//   EPI_F32      ws[split] = acc (fp32 partials, reduced by splitk_reduce)
//   EPI_SILU     gate/up interleaved tiles: out = bf16(silu(bf16 g) * bf16 u)
//                (src/layers/activation.py:6-10 fused into the gate_up GEMM)
#pragma once
#include "common.cuh"

namespace b200 {

enum GemmEpilogue : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_SILU = 2 };

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;
constexpr int kGemmMaxStages = 8;

struct GemmArgs {
  int T, N, K;         // tokens, output features (rows of W), reduction dim
  int BN;              // token tile (multiple of 32, <= 256)
  int stages;          // smem ring depth
  int num_kb;          // ceil(K / 64)
  int kb_per_split;    // K blocks per split (blockIdx.z)
  int tmem_cols;       // power of two >= BN
  int epi;             // GemmEpilogue
  __nv_bfloat16* y;    // EPI_BF16 / EPI_SILU output
  long long ldy;       // row stride of y (elements)
  float* ws;           // EPI_F32 partials [splits][T][N]
  const __nv_bfloat16* bias;  // [N] or nullptr (EPI_BF16 only)
  int silu_inter;      // EPI_SILU: I (rows of W are [gate(I) ; up(I)])
  unsigned* err;
};

__device__ __forceinline__ float silu_mul_ref(float g, float u) {
  // F.silu on a bf16 tensor rounds its result to bf16, the product rounds
  // again (eager semantics of src/layers/activation.py:9-10).
  const float s = bf16_round(g / (1.0f + expf(-g)));
  return bf16_round(__fmul_rn(s, u));
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

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kGemmBM;  // feature tile (EPI_SILU: gate row 64*blockIdx.x)
  const int t0 = blockIdx.y * p.BN;
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
  const int nk = kb1 - kb0;

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

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        const int s = i % S;
        const uint32_t ph = (uint32_t)(i / S) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, p.err)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], kABytes + b_bytes);
        const int kc = (kb0 + i) * kGemmBK;
        if (p.epi == EPI_SILU) {
          // rows [64 gate | 64 up] of the interleaved tile
          const int g0 = blockIdx.x * 64;
          tma_load_2d(a_smem + (size_t)s * kABytes, &tmW, &full[s], kc, g0);
          tma_load_2d(a_smem + (size_t)s * kABytes + kABytes / 2, &tmW, &full[s], kc,
                      p.silu_inter + g0);
        } else {
          tma_load_2d(a_smem + (size_t)s * kABytes, &tmW, &full[s], kc, n0);
        }
        tma_load_2d(b_smem + (size_t)s * b_bytes, &tmX, &full[s], kc, t0);
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
    // ---------------- epilogue: warps 2..5 -> TMEM lane quarters 2,3,0,1
    const int q = warp & 3;
    const int row = q * 32 + lane;  // accumulator row inside the 128-row tile
    const bool have = mbar_wait(tmem_full, 0, p.err);
    tc_fence_after();
    if (p.epi == EPI_SILU) {
      // lanes 0..63 hold gate rows, 64..127 the matching up rows.  The loop
      // runs even after a timed-out wait so every epilogue warp reaches the
      // same named barriers; only the stores are skipped.
      float* xch = reinterpret_cast<float*>(a_smem);  // 64 x 33 floats
      const int feat = blockIdx.x * 64 + (row & 63);
      for (int c = 0; c < p.BN; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)c, r);
        tmem_ld_wait();
        if (q >= 2) {
#pragma unroll
          for (int j = 0; j < 32; ++j) xch[(row - 64) * 33 + j] = __uint_as_float(r[j]);
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (have && q < 2 && feat < p.silu_inter) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int t = t0 + c + j;
            if (t < p.T) {
              const float g = bf16_round(__uint_as_float(r[j]));
              const float u = bf16_round(xch[row * 33 + j]);
              p.y[(size_t)t * p.ldy + feat] = __float2bfloat16_rn(silu_mul_ref(g, u));
            }
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
    } else if (have) {
      {
        const int n = n0 + row;
        float bias_v = 0.f;
        if (p.epi == EPI_BF16 && p.bias != nullptr && n < p.N) bias_v = __bfloat162float(p.bias[n]);
        for (int c = 0; c < p.BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)c, r);
          tmem_ld_wait();
          if (n < p.N) {
            if (p.epi == EPI_BF16) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int t = t0 + c + j;
                if (t < p.T)
                  p.y[(size_t)t * p.ldy + n] = __float2bfloat16_rn(__uint_as_float(r[j]) + bias_v);
              }
            } else {
              float* dst = p.ws + (size_t)blockIdx.z * p.T * p.N;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int t = t0 + c + j;
                if (t < p.T) dst[(size_t)t * p.N + n] = __uint_as_float(r[j]);
              }
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, (uint32_t)p.tmem_cols);
  }
}

// Sum the fp32 split-K partials [splits][T][N] and apply the epilogue.
//   EPI_BF16: y[t][n] = bf16(sum + bias[n])
//   EPI_SILU: y[t][j] = silu(bf16 g) * bf16 u with g = col j, u = col j + N/2
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int T, int N,
                                     __nv_bfloat16* __restrict__ y, long long ldy,
                                     const __nv_bfloat16* __restrict__ bias, int epi) {
  const int outN = (epi == EPI_SILU) ? N / 2 : N;
  const int vecs = outN / 4;
  const size_t total = (size_t)T * vecs;
  const size_t plane = (size_t)T * N;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(idx / vecs);
    const int c = (int)(idx % vecs) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 acc2 = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < splits; ++s) {
      const float4 v = *reinterpret_cast<const float4*>(ws + s * plane + (size_t)t * N + c);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      if (epi == EPI_SILU) {
        const float4 u = *reinterpret_cast<const float4*>(ws + s * plane + (size_t)t * N + outN + c);
        acc2.x += u.x; acc2.y += u.y; acc2.z += u.z; acc2.w += u.w;
      }
    }
    float o[4] = {acc.x, acc.y, acc.z, acc.w};
    if (epi == EPI_SILU) {
      const float u[4] = {acc2.x, acc2.y, acc2.z, acc2.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = silu_mul_ref(bf16_round(o[i]), bf16_round(u[i]));
    } else if (bias != nullptr) {
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] += __bfloat162float(bias[c + i]);
    }
    uint2 packed;
    packed.x = pack_bf16x2(o[0], o[1]);
    packed.y = pack_bf16x2(o[2], o[3]);
    *reinterpret_cast<uint2*>(y + (size_t)t * ldy + c) = packed;
  }
}

}  // namespace b200
