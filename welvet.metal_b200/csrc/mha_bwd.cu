// MHA NormalBP leaf on the B200: the reference's backward of the attention with
// its stream semantics (shaders/ops_mha.metal:31-175, back = 1), MSE loss and
// gradient (welvet_dense.metal:193-215), FP32 SGD (welvet_dense.metal:263-281) and
// the operand preparation of the dense-gradient GEMMs (3xTF32 on the tensor
// cores, host/normalbp.cpp). The attention backward works in FP64 like the
// reference's float2 soft-double and rounds to FP32 where it does.
#include "common.cuh"
#include "kernels.h"

namespace wv {
namespace {

inline int sm_count_dev() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}
inline int grid_n(int64_t n) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sm_count_dev() * 8));
}

#define GSTRIDE(i, n) \
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (n); i += (int64_t)gridDim.x * blockDim.x)

// src [rows, cols] (ld = cols) -> dst [cols, rows_p] transposed, TF32 hi/lo,
// zero-padded rows_p >= rows.
__global__ void transpose_split_kernel(const float* src, int64_t rows, int cols, int64_t rows_p, float* hi,
                                       float* lo) {
  GSTRIDE(i, (int64_t)cols * rows_p) {
    const int c = (int)(i / rows_p);
    const int64_t r = i % rows_p;
    const float v = r < rows ? src[r * cols + c] : 0.f;
    const float h = to_tf32(v);
    hi[i] = h;
    lo[i] = v - h;
  }
}

// rope_gpu (ops_mha.metal:13-30) on one head-major row in FP64; reverse applies
// the transposed rotation. The exponent 2i/hd is an FP32 division, as there.
__device__ void rope_row(double* v, int pos, int nh, int hd, double theta, bool reverse) {
  const int half = hd / 2;
  if (half < 1 || (float)theta <= 0.0f) return;
  const double lt = log(theta);
  for (int head = 0; head < nh; ++head)
    for (int i = 0; i < half; ++i) {
      const float e = __fdiv_rn((float)(2 * i), (float)hd);
      const double angle = (double)pos / exp(lt * (double)e);
      double sn, cs;
      sincos(angle, &sn, &cs);
      double* a = v + (size_t)head * hd + i;
      double* b = a + half;
      const double x = *a, y = *b;
      if (reverse) {
        *a = x * cs + y * sn;
        *b = -x * sn + y * cs;
      } else {
        *a = x * cs - y * sn;
        *b = x * sn + y * cs;
      }
    }
}

// Batch b's ring: every slot cleared, then the slots of positions base..base+T-1
// hold that batch's keys/values (the last position written wins when T > MSL),
// keys rotated at their position; and the batch's q rows, rotated.
__global__ void ring_fill_kernel(BwdArgs a, int b) {
  const int base = b * a.T;
  const int rows = a.msl + a.T;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    if (r < a.msl) {
      const int s = r;
      double* kd = a.ck + (size_t)s * a.kd;
      double* vd = a.cv + (size_t)s * a.kd;
      const int t0 = ((s - base) % a.msl + a.msl) % a.msl;
      if (t0 >= a.T) {
        for (int i = 0; i < a.kd; ++i) kd[i] = vd[i] = 0.0;
        continue;
      }
      const int t = t0 + a.msl * ((a.T - 1 - t0) / a.msl);
      const int64_t tok = (int64_t)base + t;
      for (int i = 0; i < a.kd; ++i) {
        kd[i] = a.qkv[tok * a.ld_qkv + a.qd + i];
        vd[i] = a.qkv[tok * a.ld_qkv + a.qd + a.kd + i];
      }
      if (a.rope) rope_row(kd, base + t, a.nk, a.hd, a.theta, false);
    } else {
      const int t = r - a.msl;
      const int64_t tok = (int64_t)base + t;
      double* qd = a.qb + (size_t)t * a.qd;
      for (int i = 0; i < a.qd; ++i) qd[i] = a.qkv[tok * a.ld_qkv + i];
      if (a.rope) rope_row(qd, base + t, a.nh, a.hd, a.theta, false);
    }
  }
}

__device__ __forceinline__ bool allowed(const BwdArgs& a, int q, int k) {
  if (a.mask == 2) return true;
  if (a.mask == 3) {
    const int w = a.window > 0 ? a.window : a.msl;
    return a.window_causal ? (k <= q && k >= q - w + 1) : (abs(q - k) < w);
  }
  if (a.mask == 4 && q < a.prefix && k < a.prefix) return true;
  return k <= q;
}

__device__ __forceinline__ double block_sum(double v, double* red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  double t = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
  return t;
}
__device__ __forceinline__ double block_max(double v, double* red) {
  for (int o = 16; o; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  double t = -1e300;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t = fmax(t, red[i]);
  return t;
}

// One (head, query t) of batch b per block: scores over keys [0, base+T) (earlier
// positions read the cleared ring, i.e. zero keys), softmax or sigmoid, then
// dw_k = v_k . gy, delta_k, gq (this query, no contention) and gk / gv (ring
// slots, FP64 atomics). score / delta per key live in the scratch row of the block.
__global__ void __launch_bounds__(256) attn_bwd_query_kernel(BwdArgs a, int b) {
  __shared__ double red[8];
  const int head = blockIdx.x, t = blockIdx.y;
  const int base = b * a.T, pos = base + t, kvlen = base + a.T;
  const int kh = head / (a.nh / a.nk);
  const double* q = a.qb + (size_t)t * a.qd + (size_t)head * a.hd;
  double* sc = a.scratch + ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * (size_t)(2 * a.kvmax);
  double* dl = sc + a.kvmax;
  const float* gy = a.grad_attn + (size_t)pos * a.qd + (size_t)head * a.hd;
  const double gscale = a.shift ? 18446744073709551616.0 : 1.0;  // 2^64
  double mx = -1e300;
  int cnt = 0;
  for (int k = threadIdx.x; k < kvlen; k += blockDim.x) {
    if (!allowed(a, pos, k)) {
      sc[k] = 0.0;
      continue;
    }
    const double* kr = a.ck + (size_t)(k % a.msl) * a.kd + (size_t)kh * a.hd;
    double dot = 0;
    for (int z = 0; z < a.hd; ++z) dot += q[z] * kr[z];
    double s = dot * a.scale;
    if (a.alibi) s -= exp2((double)(-(float)(head + 1) * 8.0f / (float)a.nh)) * (double)(float)abs(pos - k);
    sc[k] = s;
    mx = fmax(mx, s);
    ++cnt;
  }
  const int count = (int)block_sum((double)cnt, red);
  if (count == 0) return;
  mx = block_max(mx, red);
  double part = 0;
  for (int k = threadIdx.x; k < kvlen; k += blockDim.x)
    if (allowed(a, pos, k)) {
      const double e = a.sigmoid ? 1.0 / (1.0 + exp(-sc[k])) : exp(sc[k] - mx);
      sc[k] = e;
      part += e;
    }
  const double sum = block_sum(part, red);
  double sdw = 0;
  for (int k = threadIdx.x; k < kvlen; k += blockDim.x) {
    if (!allowed(a, pos, k)) {
      dl[k] = 0.0;
      continue;
    }
    const double p = a.sigmoid ? sc[k] : sc[k] / sum;
    sc[k] = p;
    const double* vr = a.cv + (size_t)(k % a.msl) * a.kd + (size_t)kh * a.hd;
    double* gvr = a.gv + (size_t)(k % a.msl) * a.kd + (size_t)kh * a.hd;
    double dw = 0;
    for (int z = 0; z < a.hd; ++z) {
      const double g = (double)gy[z] * gscale;
      atomicAdd(gvr + z, p * g);
      dw += vr[z] * g;
    }
    dl[k] = dw;
    sdw += dw * p;
  }
  const double sumdw = block_sum(sdw, red);
  for (int k = threadIdx.x; k < kvlen; k += blockDim.x) {
    if (!allowed(a, pos, k)) continue;
    const double p = sc[k];
    const double delta = (a.sigmoid ? dl[k] * p * (1.0 - p) : p * (dl[k] - sumdw)) * a.scale;
    dl[k] = delta;
    double* gkr = a.gk + (size_t)(k % a.msl) * a.kd + (size_t)kh * a.hd;
    for (int z = 0; z < a.hd; ++z) atomicAdd(gkr + z, delta * q[z]);
  }
  __syncthreads();
  double* gq = a.gq + (size_t)t * a.qd + (size_t)head * a.hd;
  for (int z = threadIdx.x; z < a.hd; z += blockDim.x) {
    double acc = 0;
    for (int k = 0; k < kvlen; ++k)
      if (allowed(a, pos, k)) acc += dl[k] * a.ck[(size_t)(k % a.msl) * a.kd + (size_t)kh * a.hd + z];
    gq[z] = acc;
  }
}

// End of batch b: q gradients rotated back and written (FP32, scaled back), then
// the key-gradient slots of the batch's positions rotated back, each slot by its
// positions in order (a slot shared by several positions turns once per position).
__global__ void batch_end_kernel(BwdArgs a, int b) {
  const int base = b * a.T;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < a.T + a.msl; r += gridDim.x * blockDim.x) {
    if (r < a.T) {
      double* gq = a.gq + (size_t)r * a.qd;
      if (a.rope) rope_row(gq, base + r, a.nh, a.hd, a.theta, true);
      float* out = a.g_q + (size_t)(base + r) * a.ld_g;
      for (int i = 0; i < a.qd; ++i) out[i] = ldexpf((float)gq[i], -a.shift);
    } else if (a.rope) {
      const int s = r - a.T;
      const int t0 = ((s - base) % a.msl + a.msl) % a.msl;
      for (int t = t0; t < a.T; t += a.msl) rope_row(a.gk + (size_t)s * a.kd, base + t, a.nk, a.hd, a.theta, true);
    }
  }
}

__global__ void final_kv_kernel(BwdArgs a) {
  GSTRIDE(i, a.M * a.kd) {
    const int64_t tok = i / a.kd;
    const int c = (int)(i % a.kd);
    const size_t s = (size_t)(tok % a.msl) * a.kd + c;
    a.g_k[tok * a.ld_g + c] = ldexpf((float)a.gk[s], -a.shift);
    a.g_v[tok * a.ld_g + c] = ldexpf((float)a.gv[s], -a.shift);
  }
}

// welvet_mse_grad: g = fl32(2 (p - t) / n) with the difference exact.
__global__ void mse_kernel(const float* pred, const float* target, float* grad, double* partial, int64_t n) {
  __shared__ double red[8];
  double s = 0;
  GSTRIDE(i, n) {
    const double d = (double)pred[i] - (double)target[i];
    grad[i] = (float)(2.0 * d / (double)n);
    s += d * d;
  }
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    partial[blockIdx.x] = t;
  }
}

// welvet_sgd_f32_f64_grad, normal range: step = fl32(lr * g), w - step in FP32
// (gradients below 1e-20 scaled by 2^64 around the product, as there).
__global__ void sgd_kernel(const float* w, const float* g, float* out, int64_t n, double lr) {
  GSTRIDE(i, n) {
    const float gv = g[i];
    const float step = fabsf(gv) < 1e-20f ? ldexpf((float)(lr * ldexp((double)gv, 64)), -64) : (float)(lr * (double)gv);
    out[i] = w[i] - step;
  }
}

}  // namespace

cudaError_t transpose_split(const float* src, int64_t rows, int cols, int64_t rows_p, float* hi, float* lo,
                            cudaStream_t s) {
  transpose_split_kernel<<<grid_n((int64_t)cols * rows_p), 256, 0, s>>>(src, rows, cols, rows_p, hi, lo);
  return cudaGetLastError();
}

cudaError_t attn_backward(const BwdArgs& a, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(a.gk, 0, (size_t)a.msl * a.kd * sizeof(double), s);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(a.gv, 0, (size_t)a.msl * a.kd * sizeof(double), s);
  if (e != cudaSuccess) return e;
  for (int b = 0; b < a.B; ++b) {
    ring_fill_kernel<<<std::max(1, (a.msl + a.T + 127) / 128), 128, 0, s>>>(a, b);
    e = cudaMemsetAsync(a.gq, 0, (size_t)a.T * a.qd * sizeof(double), s);
    if (e != cudaSuccess) return e;
    attn_bwd_query_kernel<<<dim3(a.nh, a.T), 256, 0, s>>>(a, b);
    batch_end_kernel<<<std::max(1, (a.msl + a.T + 127) / 128), 128, 0, s>>>(a, b);
  }
  final_kv_kernel<<<grid_n(a.M * a.kd), 256, 0, s>>>(a);
  return cudaGetLastError();
}

int mse_grid(int64_t n) { return std::min(grid_n(n), 1024); }

cudaError_t mse_grad(const float* pred, const float* target, float* grad, double* partial, int64_t n,
                     cudaStream_t s) {
  mse_kernel<<<mse_grid(n), 256, 0, s>>>(pred, target, grad, partial, n);
  return cudaGetLastError();
}

cudaError_t sgd_f32(const float* w, const float* g, float* out, int64_t n, double lr, cudaStream_t s) {
  sgd_kernel<<<grid_n(n), 256, 0, s>>>(w, g, out, n, lr);
  return cudaGetLastError();
}

}  // namespace wv
