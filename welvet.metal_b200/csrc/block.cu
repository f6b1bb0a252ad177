// Transformer-block kernels around the MHA: RMSNorm / LayerNorm forward, the
// embedding gather with its activation, and the operand packing of the SwiGLU
// feed-forward (whose Gate|Up GEMM applies SiLU(gate) * up in the tcgen05 GEMM
// epilogue, gemm_tc.cu). All of them are HBM-bound passes.
#include "common.cuh"
#include "kernels.h"

#include <cuda_bf16.h>

namespace wv {
namespace {

inline int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

__device__ __forceinline__ float load_elem(const void* p, size_t i, int bf16) {
  return bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]) : __ldg(static_cast<const float*>(p) + i);
}
__device__ __forceinline__ void store_elem(void* p, size_t i, float v, int bf16) {
  if (bf16)
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    static_cast<float*>(p)[i] = v;
}

// Sum over the TPR threads of a row group (a warp, or the whole 256-thread CTA).
template <int TPR>
__device__ __forceinline__ double group_sum(double v, double* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (TPR == 32) return v;
  const int w = threadIdx.x >> 5;
  __syncthreads();  // red is reused by the next call
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  double t = 0;
#pragma unroll
  for (int i = 0; i < TPR / 32; ++i) t += red[i];
  return t;
}

// RMSNorm (LN = false) / LayerNorm (LN = true) forward of op_norm_forward
// (shaders/ops_norm.metal:2-26): sum and sum of squares of the row, mean (LayerNorm
// only), var = E[x^2] - mean^2, inv = 1/sqrt(var + eps); pre = x-hat = (x - mean) *
// inv, post = x-hat * gamma (+ beta). The reference evaluates this in float2
// soft-double and rounds pre/post once; here the statistics and both outputs are
// computed in FP64 and rounded once (E[x^2] - mean^2 cancels badly in FP32 when
// |mean| >> std). TPR threads own a row: a warp for dim <= 1024, else the CTA.
// The row is read twice; the second read hits L1/L2.
template <int TPR, bool LN>
__global__ void __launch_bounds__(256) norm_fwd_kernel(NormArgs a) {
  __shared__ double red[8];
  const int rows_per_cta = 256 / TPR;
  const int lane = threadIdx.x % TPR;
  const int dim = a.dim;
  const bool vec = a.vec4;
  for (int64_t row = (int64_t)blockIdx.x * rows_per_cta + threadIdx.x / TPR; row < a.rows;
       row += (int64_t)gridDim.x * rows_per_cta) {
    const size_t base = (size_t)row * dim;
    double s = 0, q = 0;
    if (vec && !a.x_bf16) {
      const float4* x4 = reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + base);
      for (int i = lane; i < dim / 4; i += TPR) {
        const float4 v = __ldg(x4 + i);
        s += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
        q += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
      }
    } else {
      for (int i = lane; i < dim; i += TPR) {
        const double v = load_elem(a.x, base + i, a.x_bf16);
        s += v;
        q += v * v;
      }
    }
    s = group_sum<TPR>(s, red);
    q = group_sum<TPR>(q, red);
    const double mean = LN ? s / dim : 0.0;
    const double var = q / dim - mean * mean;
    const double inv = 1.0 / sqrt(var + a.eps);
    if (vec && !a.x_bf16 && !a.out_bf16) {
      const float4* x4 = reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + base);
      float4* pre4 = a.pre ? reinterpret_cast<float4*>(static_cast<float*>(a.pre) + base) : nullptr;
      float4* post4 = reinterpret_cast<float4*>(static_cast<float*>(a.post) + base);
      const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
      const float4* b4 = reinterpret_cast<const float4*>(a.beta);
      for (int i = lane; i < dim / 4; i += TPR) {
        const float4 v = __ldg(x4 + i), g = __ldg(g4 + i);
        const float4 b = LN ? __ldg(b4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        const double h0 = ((double)v.x - mean) * inv, h1 = ((double)v.y - mean) * inv;
        const double h2 = ((double)v.z - mean) * inv, h3 = ((double)v.w - mean) * inv;
        if (pre4) __stcs(pre4 + i, make_float4((float)h0, (float)h1, (float)h2, (float)h3));
        float4 y;
        y.x = (float)(LN ? h0 * g.x + b.x : h0 * g.x);
        y.y = (float)(LN ? h1 * g.y + b.y : h1 * g.y);
        y.z = (float)(LN ? h2 * g.z + b.z : h2 * g.z);
        y.w = (float)(LN ? h3 * g.w + b.w : h3 * g.w);
        __stcs(post4 + i, y);
      }
    } else {
      for (int i = lane; i < dim; i += TPR) {
        const double h = ((double)load_elem(a.x, base + i, a.x_bf16) - mean) * inv;
        if (a.pre) store_elem(a.pre, base + i, (float)h, a.out_bf16);
        const double y = LN ? h * a.gamma[i] + a.beta[i] : h * a.gamma[i];
        store_elem(a.post, base + i, (float)y, a.out_bf16);
      }
    }
  }
}

// act_value (shaders/ops_common.metal:83-105) in FP32 with correctly rounded
// basics and CUDA's expf/tanhf (a few ulp; the reference's soft-double is exact
// to FP32 rounding). LeakyReLU multiplies by 0.01 in double as the reference's
// float2 constant does.
__device__ __forceinline__ float act_apply(float v, int act) {
  switch (act) {
  case 0: return v > 0.f ? v : 0.f;
  case 1: return __fdiv_rn(v, 1.f + expf(-v));
  case 2: {
    const float u = 0.7978845608f * (v + 0.044715f * v * v * v);
    return 0.5f * v * (1.f + (u > 18.f ? 1.f : (u < -18.f ? -1.f : tanhf(u))));
  }
  case 3: return v > 18.f ? 1.f : (v < -18.f ? -1.f : tanhf(v));
  case 4: return __fdiv_rn(1.f, 1.f + expf(-v));
  case 5: return v < 0.f ? (float)((double)v * 0.01) : v;
  case 6: return v < 0.f ? 0.f : v * v;
  default: return v;
  }
}

// Row id of op_embedding_forward (shaders/ops_embedding.metal:4): abs(int(x)) % vocab.
// The conversion truncates toward zero; beyond +-2^31 it saturates here (the
// reference's is undefined there), and the magnitude is taken in 64 bits, so
// the row is always inside the table.
__device__ __forceinline__ int embed_row(float x, int vocab) {
  const long long t = (long long)__float2int_rz(x);
  return (int)((t < 0 ? -t : t) % vocab);
}

__global__ void __launch_bounds__(256) embedding_kernel(EmbedArgs a) {
  const int per_row = a.vec4 ? a.emb / 4 : a.emb;
  const int64_t total = a.tokens * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_row;
    const int c = (int)(i % per_row);
    const int id = embed_row(__ldg(a.x + t * a.in_last), a.vocab);
    if (a.vec4) {
      float4 v = __ldg(reinterpret_cast<const float4*>(a.W + (size_t)id * a.emb) + c);
      v = make_float4(act_apply(v.x, a.act), act_apply(v.y, a.act), act_apply(v.z, a.act), act_apply(v.w, a.act));
      if (a.out_bf16) {
        __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.out) + (size_t)t * a.emb + 4 * c;
        o[0] = __float2bfloat16_rn(v.x), o[1] = __float2bfloat16_rn(v.y);
        o[2] = __float2bfloat16_rn(v.z), o[3] = __float2bfloat16_rn(v.w);
      } else {
        __stcs(reinterpret_cast<float4*>(static_cast<float*>(a.out) + (size_t)t * a.emb) + c, v);
      }
    } else {
      store_elem(a.out, (size_t)t * a.emb + c, act_apply(__ldg(a.W + (size_t)id * a.emb + c), a.act), a.out_bf16);
    }
  }
}

// SwiGLU operand packing. Gate and Up [inter, in] go into one [2 * inter_p, in_p]
// matrix whose rows alternate in groups of 32 (gate rows 32g..32g+31, then the
// same up rows), so that every 64-column group of the fused GEMM's output holds
// 32 gate and the matching 32 up values for the epilogue; padding rows and
// columns are zero. Down [in, inter] goes to [in, inter_p] with zero columns.
__global__ void pack_gate_up_kernel(const float* gate, const float* up, float* out, int inter, int in,
                                    int inter_p, int in_p) {
  const int64_t total = (int64_t)2 * inter_p * in_p;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / in_p), c = (int)(i % in_p);
    const int grp = r / 64, within = r % 64;
    const bool is_up = within >= 32;
    const int src = grp * 32 + (within & 31);
    float v = 0.f;
    if (src < inter && c < in) v = (is_up ? up : gate)[(size_t)src * in + c];
    out[i] = v;
  }
}
__global__ void pad_cols_kernel(const float* src, float* dst, int64_t rows, int cols, int cols_p) {
  const int64_t total = rows * cols_p;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols_p;
    const int c = (int)(i % cols_p);
    dst[i] = c < cols ? src[r * cols + c] : 0.f;
  }
}
// x [rows, cols] (FP32 or BF16) -> zero-padded [rows, cols_p] as TF32 hi/lo pairs
// (hi != null) or BF16 (b != null).
__global__ void pad_operand_kernel(const void* x, int x_bf16, int64_t rows, int cols, int cols_p, float* hi,
                                   float* lo, __nv_bfloat16* b) {
  const int64_t total = rows * cols_p;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols_p;
    const int c = (int)(i % cols_p);
    const float v = c < cols ? load_elem(x, (size_t)r * cols + c, x_bf16) : 0.f;
    if (hi) {
      const float h = to_tf32(v);
      hi[i] = h;
      lo[i] = v - h;
    } else {
      b[i] = __float2bfloat16_rn(v);
    }
  }
}

int grid_of(int64_t work, int per_thread = 1) {
  const int64_t blocks = (work / per_thread + 255) / 256;
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sm_count() * 8));
}

} // namespace

cudaError_t norm_forward(const NormArgs& a0, int layernorm, cudaStream_t s) {
  if (a0.rows <= 0 || a0.dim <= 0) return cudaSuccess;
  NormArgs a = a0;
  auto al16 = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  a.vec4 = a.dim % 4 == 0 && al16(a.x) && al16(a.pre) && al16(a.post) && al16(a.gamma) && al16(a.beta);
  const int sms = sm_count();
  if (a.dim <= 1024) {
    const int grid = (int)std::min<int64_t>((a.rows + 7) / 8, (int64_t)sms * 8);
    if (layernorm)
      norm_fwd_kernel<32, true><<<grid, 256, 0, s>>>(a);
    else
      norm_fwd_kernel<32, false><<<grid, 256, 0, s>>>(a);
  } else {
    const int grid = (int)std::min<int64_t>(a.rows, (int64_t)sms * 8);
    if (layernorm)
      norm_fwd_kernel<256, true><<<grid, 256, 0, s>>>(a);
    else
      norm_fwd_kernel<256, false><<<grid, 256, 0, s>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t embedding_forward(const EmbedArgs& a0, cudaStream_t s) {
  if (a0.tokens <= 0 || a0.emb <= 0) return cudaSuccess;
  EmbedArgs a = a0;
  a.vec4 = a.emb % 4 == 0 && (reinterpret_cast<uintptr_t>(a.W) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(a.out) & (a.out_bf16 ? 7 : 15)) == 0;
  const int64_t work = a.tokens * (a.vec4 ? a.emb / 4 : a.emb);
  embedding_kernel<<<grid_of(work), 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t swiglu_pack_gate_up(const float* gate, const float* up, float* out, int inter, int in, int inter_p,
                                int in_p, cudaStream_t s) {
  pack_gate_up_kernel<<<grid_of((int64_t)2 * inter_p * in_p), 256, 0, s>>>(gate, up, out, inter, in, inter_p, in_p);
  return cudaGetLastError();
}

cudaError_t pad_cols(const float* src, float* dst, int64_t rows, int cols, int cols_p, cudaStream_t s) {
  pad_cols_kernel<<<grid_of(rows * cols_p), 256, 0, s>>>(src, dst, rows, cols, cols_p);
  return cudaGetLastError();
}

cudaError_t pad_operand(const void* x, int x_bf16, int64_t rows, int cols, int cols_p, float* hi, float* lo,
                        void* b, cudaStream_t s) {
  pad_operand_kernel<<<grid_of(rows * cols_p), 256, 0, s>>>(x, x_bf16, rows, cols, cols_p, hi, lo,
                                                           static_cast<__nv_bfloat16*>(b));
  return cudaGetLastError();
}

} // namespace wv
