// CUDA-core GEMM for projection shapes the TMA path cannot address (row strides
// that are not 16-byte multiples, e.g. d_model % 4 != 0 in FP32). FP32 FMA
// accumulation; A/B given as FP32 (optionally as TF32 hi+lo pairs, summed
// exactly on load) or BF16. Same output conventions as the tensor-core GEMM,
// without the fused RoPE / KV scatter (the host applies those separately).
#include "common.cuh"
#include "kernels.h"

namespace wv {
namespace {

constexpr int TM = 64, TN = 64, TK = 16;

__device__ __forceinline__ float ld_op(const void* p, const void* lo, size_t i, bool bf16) {
  if (bf16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  float v = static_cast<const float*>(p)[i];
  if (lo) v += static_cast<const float*>(lo)[i];
  return v;
}

__global__ void __launch_bounds__(256) gemm_simt_kernel(GemmArgs g) {
  __shared__ float As[TK][TM + 1];
  __shared__ float Bs[TK][TN + 1];
  const bool bf16 = g.kind == kGemmBF16;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < g.K; k0 += TK) {
    for (int i = threadIdx.x; i < TM * TK; i += 256) {
      const int r = i / TK, c = i % TK;
      const int m = m0 + r, k = k0 + c;
      As[c][r] = (m < g.M && k < g.K) ? ld_op(g.a, g.a_lo, (size_t)m * g.lda + k, bf16) : 0.f;
      const int n = n0 + r;
      Bs[c][r] = (n < g.N && k < g.K) ? ld_op(g.b, g.b_lo, (size_t)n * g.ldb + k, bf16) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < TK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[k][ty + 16 * i];
        b[i] = Bs[k][tx + 16 * i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + ty + 16 * i, n = n0 + tx + 16 * j;
      if (m >= g.M || n >= g.N) continue;
      float v = acc[i][j];
      if (g.b_scale && g.kind == kGemmFP8) v *= g.b_scale[n];
      const size_t off = (size_t)m * g.ldo + n;
      if (g.out_bf16) {
        static_cast<__nv_bfloat16*>(g.out)[off] = __float2bfloat16_rn(v);
      } else {
        if (!(g.split_only && g.out_hi)) static_cast<float*>(g.out)[off] = v;
        if (g.out_hi) {
          const float h = to_tf32(v);
          g.out_hi[off] = h;
          g.out_lo[off] = v - h;
        }
      }
    }
}

} // namespace

cudaError_t gemm_simt(const GemmArgs& g, cudaStream_t stream) {
  if (g.kind != kGemmBF16 && g.kind != kGemmTF32x3) return cudaErrorInvalidValue;
  dim3 grid((g.N + TN - 1) / TN, (g.M + TM - 1) / TM);
  gemm_simt_kernel<<<grid, 256, 0, stream>>>(g);
  return cudaGetLastError();
}

} // namespace wv
