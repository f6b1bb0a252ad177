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

// One rotation pair of rope_gpu (ops_mha.metal:13-30) in FP64: elements i and
// i + hd/2 of a head row, at position pos; reverse applies the transposed
// rotation. The exponent 2i/hd is an FP32 division, as there.
__device__ __forceinline__ void rope_pair(double* a, double* b, int pos, int i, int hd, double theta, bool reverse) {
  const float e = __fdiv_rn((float)(2 * i), (float)hd);
  const double angle = (double)pos / exp(log(theta) * (double)e);
  double sn, cs;
  sincos(angle, &sn, &cs);
  const double x = *a, y = *b;
  if (reverse) {
    *a = x * cs + y * sn;
    *b = -x * sn + y * cs;
  } else {
    *a = x * cs - y * sn;
    *b = x * sn + y * cs;
  }
}
__device__ __forceinline__ bool rope_on(const BwdArgs& a) {
  return a.rope && a.hd / 2 >= 1 && (float)a.theta > 0.0f;
}

// The element unit of the per-pair kernels: unit u of a row's `heads` x P units
// (P = ceil(hd / 2)) is head u / P, pair i = u % P; i < hd/2 covers elements i and
// i + hd/2, i == hd/2 (odd hd) the last element, hd - 1, alone.
struct PairIdx {
  int head, i, e0, e1;  // row offsets; e1 < 0: a single element
};
__device__ __forceinline__ PairIdx pair_idx(int u, int hd) {
  const int P = (hd + 1) / 2, half = hd / 2;
  PairIdx r;
  r.head = u / P;
  r.i = u % P;
  if (r.i < half) {
    r.e0 = r.head * hd + r.i;
    r.e1 = r.e0 + half;
  } else {
    r.e0 = r.head * hd + hd - 1;
    r.e1 = -1;
  }
  return r;
}

// Batch b's ring: every slot cleared, then the slots of positions base..base+T-1
// hold that batch's keys/values (T <= MSL, so one position per slot), keys rotated
// at their position; the batch's q rows, rotated; and its attention gradient rows
// in FP64, times 2^64 when the shift is on. One thread per element pair.
__global__ void ring_fill_kernel(BwdArgs a, int b) {
  const int base = b * a.T;
  const int P = (a.hd + 1) / 2;
  const int64_t n_slot = (int64_t)a.msl * a.nk * P, n_q = (int64_t)a.T * a.nh * P;
  const double gscale = a.shift ? 18446744073709551616.0 : 1.0;  // 2^64
  const bool rope = rope_on(a);
  GSTRIDE(u, n_slot + n_q) {
    if (u < n_slot) {
      const int s = (int)(u / ((int64_t)a.nk * P));
      const PairIdx x = pair_idx((int)(u % ((int64_t)a.nk * P)), a.hd);
      double* kd = a.ck + (size_t)s * a.kd;
      double* vd = a.cv + (size_t)s * a.kd;
      const int t = ((s - base) % a.msl + a.msl) % a.msl;
      if (t >= a.T) {
        kd[x.e0] = vd[x.e0] = 0.0;
        if (x.e1 >= 0) kd[x.e1] = vd[x.e1] = 0.0;
        continue;
      }
      const float* src = a.qkv + (int64_t)(base + t) * a.ld_qkv + a.qd;
      kd[x.e0] = src[x.e0];
      vd[x.e0] = src[a.kd + x.e0];
      if (x.e1 >= 0) {
        kd[x.e1] = src[x.e1];
        vd[x.e1] = src[a.kd + x.e1];
        if (rope) rope_pair(kd + x.e0, kd + x.e1, base + t, x.i, a.hd, a.theta, false);
      }
    } else {
      const int64_t v = u - n_slot;
      const int t = (int)(v / ((int64_t)a.nh * P));
      const PairIdx x = pair_idx((int)(v % ((int64_t)a.nh * P)), a.hd);
      const int64_t tok = (int64_t)base + t;
      const float* src = a.qkv + tok * a.ld_qkv;
      const float* gsrc = a.grad_attn + tok * a.qd;
      double* qd = a.qb + (size_t)t * a.qd;
      double* gd = a.gyb + (size_t)t * a.qd;
      qd[x.e0] = src[x.e0];
      gd[x.e0] = (double)gsrc[x.e0] * gscale;
      if (x.e1 >= 0) {
        qd[x.e1] = src[x.e1];
        gd[x.e1] = (double)gsrc[x.e1] * gscale;
        if (rope) rope_pair(qd + x.e0, qd + x.e1, base + t, x.i, a.hd, a.theta, false);
      }
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

// FP64 tiled GEMM, one (query head, k split) per blockIdx.z:
//   C_h[m, n] = sum_k A_h[m, k] * B_h(k, n)
// A_h[m, k] = a[h * a_hs + m * lda + k]; B's rows are ring slots taken modulo `mod`
// (key positions past the ring wrap onto it): with B_NK, B_h(k, n) =
// b[kvh * b_hs + (n % mod) * ldb + k], else b[kvh * b_hs + (k % mod) * ldb + n], for
// the KV head kvh = h / group. 64 x 64 tiles, k-steps of 16, 256 threads of 4 x 4
// outputs; operands outside M / N / K read as zero.
struct DgemmArgs {
  int M = 0, N = 0, K = 0, mod = 1, group = 1;
  int heads = 1, ksplit = 1;  // blockIdx.z = head + heads * split; split s sums k in its chunk
  int64_t c_split = 0;        // output offset of split s: s * c_split
  const double* a = nullptr;
  int64_t lda = 0, a_hs = 0;
  const double* b = nullptr;
  int64_t ldb = 0, b_hs = 0;
  double* c = nullptr;
  int64_t ldc = 0, c_hs = 0;
};
template <bool B_NK>
__global__ void __launch_bounds__(256) dgemm_kernel(DgemmArgs g) {
  __shared__ double As[16][65], Bs[16][65];
  const int h = blockIdx.z % g.heads, split = blockIdx.z / g.heads;
  const double* A = g.a + (int64_t)h * g.a_hs;
  const double* B = g.b + (int64_t)(h / g.group) * g.b_hs;
  double* C = g.c + (int64_t)h * g.c_hs + (int64_t)split * g.c_split;
  const int kchunk = (g.K + g.ksplit * 16 - 1) / (g.ksplit * 16) * 16;
  const int kbeg = split * kchunk, kend = min(g.K, kbeg + kchunk);
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  double acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
  for (int k0 = kbeg; k0 < kend; k0 += 16) {
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      const int idx = tid + 256 * l;
      const int r = idx >> 4, kk = idx & 15, m = m0 + r, k = k0 + kk;
      As[kk][r] = (m < g.M && k < kend) ? A[(int64_t)m * g.lda + k] : 0.0;
      if (B_NK) {
        const int n = n0 + r;
        Bs[kk][r] = (n < g.N && k < kend) ? B[(int64_t)(n % g.mod) * g.ldb + k] : 0.0;
      } else {
        const int kb = idx >> 6, n = n0 + (idx & 63), kr = k0 + kb;
        Bs[kb][idx & 63] = (kr < kend && n < g.N) ? B[(int64_t)(kr % g.mod) * g.ldb + n] : 0.0;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      double av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n < g.N) C[(int64_t)m * g.ldc + n] = acc[i][j];
    }
  }
}

// One (head, query t) of batch b per block, on its scratch row: the first half
// holds q.k per key (dgemm, keys of earlier positions read the cleared ring as zero
// vectors), the second v.gy per key. Scores scaled (ALiBi subtracted), softmax or
// sigmoid over the keys the mask allows, then delta_k = p_k (dw_k - sum p dw) scale
// (sigmoid: dw_k p_k (1 - p_k) scale). The row is left holding p_k and delta_k,
// zero for keys the mask excludes.
__global__ void __launch_bounds__(256) attn_bwd_row_kernel(BwdArgs a, int b) {
  __shared__ double red[8];
  const int head = blockIdx.x, t = blockIdx.y;
  const int base = b * a.T, pos = base + t, kvlen = base + a.T;
  double* sc = a.scratch + ((size_t)t * a.nh + head) * (size_t)(2 * a.kvmax);
  double* dl = sc + a.kvmax;
  double mx = -1e300;
  int cnt = 0;
  for (int k = threadIdx.x; k < kvlen; k += blockDim.x) {
    if (!allowed(a, pos, k)) {
      sc[k] = 0.0;
      continue;
    }
    double s = sc[k] * a.scale;
    if (a.alibi) s -= exp2((double)(-(float)(head + 1) * 8.0f / (float)a.nh)) * (double)(float)abs(pos - k);
    sc[k] = s;
    mx = fmax(mx, s);
    ++cnt;
  }
  const int count = (int)block_sum((double)cnt, red);
  if (count == 0) {
    for (int k = threadIdx.x; k < kvlen; k += blockDim.x) dl[k] = 0.0;
    return;
  }
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
    sdw += dl[k] * p;
  }
  const double sumdw = block_sum(sdw, red);
  for (int k = threadIdx.x; k < kvlen; k += blockDim.x) {
    if (!allowed(a, pos, k)) continue;
    const double p = sc[k];
    dl[k] = (a.sigmoid ? dl[k] * p * (1.0 - p) : p * (dl[k] - sumdw)) * a.scale;
  }
}


// Key / value gradients of batch b from the scratch rows of attn_bwd_row_kernel.
// For KV head kh and ring slot s (keys k = s, s + msl, ... below base + T, in
// that order), over the group's query heads h and the batch's queries t:
//   gv[s] += p[h,t,k] * gy[t,h] * 2^shift,   gk[s] += delta[h,t,k] * q[t,h]
// (q rotated, as the scores used it) — the same products the reference adds per
// (query, key), summed here without atomics in a fixed order. One block per (32
// slots, KV head): lane = slot, warp = head-dimension residue mod 8, so each thread
// keeps 8 + 8 FP64 sums per 64-dimension chunk; rows (t, h) are staged 16 at a time
// in shared memory, and under the causal mask the rows of queries before the
// tile's first key (all zero) are skipped.
constexpr int kKvSlots = 32, kKvRows = 16, kKvDims = 64;
__global__ void __launch_bounds__(256) kv_grad_kernel(BwdArgs a, int b) {
  __shared__ double ps[kKvRows][kKvSlots], ds[kKvRows][kKvSlots];
  __shared__ double gs[kKvRows][kKvDims], qs[kKvRows][kKvDims];
  const int base = b * a.T, kvlen = base + a.T;
  const int kh = blockIdx.y, G = a.nh / a.nk;
  const int s0 = blockIdx.x * kKvSlots;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rows = G * a.T;  // row r: query t = r / G, head kh * G + r % G
  const size_t ldr = 2 * (size_t)a.kvmax;
  // split blockIdx.z of gridDim.z takes rows [r_lo, r_hi) (whole 16-row chunks)
  const int per = (rows + (int)gridDim.z * kKvRows - 1) / ((int)gridDim.z * kKvRows) * kKvRows;
  const int r_lo = (int)blockIdx.z * per, r_hi = min(rows, r_lo + per);
  for (int z0 = 0; z0 < a.hd; z0 += kKvDims) {
    double av[8], ak[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) av[i] = ak[i] = 0.0;
    for (int k0 = s0; k0 < kvlen; k0 += a.msl) {
      int r_begin = r_lo;
      if (a.mask == 1) r_begin = max(r_lo, max(0, k0 - base) * G / kKvRows * kKvRows);
      for (int r0 = r_begin; r0 < r_hi; r0 += kKvRows) {
        __syncthreads();
        for (int i = threadIdx.x; i < kKvRows * kKvSlots; i += blockDim.x) {
          const int rr = i / kKvSlots, j = i % kKvSlots, r = r0 + rr, k = k0 + j;
          double pv = 0.0, dv = 0.0;
          if (r < r_hi && k < kvlen && s0 + j < a.msl) {
            const int t = r / G, h = kh * G + r % G;
            const double* row = a.scratch + ((size_t)t * a.nh + h) * ldr;
            pv = row[k];
            dv = row[a.kvmax + k];
          }
          ps[rr][j] = pv;
          ds[rr][j] = dv;
        }
        for (int i = threadIdx.x; i < kKvRows * kKvDims; i += blockDim.x) {
          const int rr = i / kKvDims, zz = i % kKvDims, r = r0 + rr, z = z0 + zz;
          double gv = 0.0, qv = 0.0;
          if (r < r_hi && z < a.hd) {
            const int t = r / G, h = kh * G + r % G;
            gv = a.gyb[(size_t)t * a.qd + (size_t)h * a.hd + z];
            qv = a.qb[(size_t)t * a.qd + (size_t)h * a.hd + z];
          }
          gs[rr][zz] = gv;
          qs[rr][zz] = qv;
        }
        __syncthreads();
#pragma unroll 4
        for (int rr = 0; rr < kKvRows; ++rr) {
          const double p = ps[rr][lane], d = ds[rr][lane];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            av[i] += p * gs[rr][warp + 8 * i];
            ak[i] += d * qs[rr][warp + 8 * i];
          }
        }
      }
    }
    const int s = s0 + lane;
    if (s < a.msl && s < kvlen) {
      // one split: add into the ring; several: this split's partial sums, which
      // sum_parts_kernel adds into the ring in split order
      const size_t ring = (size_t)a.msl * a.kd, off = (size_t)s * a.kd + (size_t)kh * a.hd;
      double* gvr = gridDim.z == 1 ? a.gv + off : a.part_kv + (2 * (size_t)blockIdx.z) * ring + off;
      double* gkr = gridDim.z == 1 ? a.gk + off : a.part_kv + (2 * (size_t)blockIdx.z + 1) * ring + off;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int z = z0 + warp + 8 * i;
        if (z < a.hd) {
          if (gridDim.z == 1) {
            gvr[z] += av[i];
            gkr[z] += ak[i];
          } else {
            gvr[z] = av[i];
            gkr[z] = ak[i];
          }
        }
      }
    }
  }
}

// out[i] (+)= sum over p < nparts of part[p * stride + i], in order p = 0, 1, ...
// (accumulate: add to out; else overwrite). With the key/value partials the parts
// alternate v, k: out2 receives the odd parts.
__global__ void sum_parts_kernel(const double* part, int nparts, int64_t stride, int64_t n, double* out,
                                 double* out2, bool accumulate) {
  GSTRIDE(i, n) {
    if (out2) {
      double v = 0.0, k = 0.0;
      for (int p = 0; p < nparts; ++p) {
        v += part[(2 * (int64_t)p) * stride + i];
        k += part[(2 * (int64_t)p + 1) * stride + i];
      }
      out[i] += v;
      out2[i] += k;
    } else {
      double v = 0.0;
      for (int p = 0; p < nparts; ++p) v += part[(int64_t)p * stride + i];
      out[i] = accumulate ? out[i] + v : v;
    }
  }
}

// End of batch b: q gradients rotated back and written (FP32, scaled back), then
// the key-gradient slots of the batch's positions rotated back, each slot by its
// positions in order (a slot shared by several positions turns once per position).
// One thread per element pair.
__global__ void batch_end_kernel(BwdArgs a, int b) {
  const int base = b * a.T;
  const int P = (a.hd + 1) / 2;
  const bool rope = rope_on(a);
  const int64_t n_q = (int64_t)a.T * a.nh * P, n_slot = rope ? (int64_t)a.msl * a.nk * P : 0;
  GSTRIDE(u, n_q + n_slot) {
    if (u < n_q) {
      const int t = (int)(u / ((int64_t)a.nh * P));
      const PairIdx x = pair_idx((int)(u % ((int64_t)a.nh * P)), a.hd);
      double* gq = a.gq + (size_t)t * a.qd;
      float* out = a.g_q + (size_t)(base + t) * a.ld_g;
      if (x.e1 >= 0 && rope) rope_pair(gq + x.e0, gq + x.e1, base + t, x.i, a.hd, a.theta, true);
      out[x.e0] = ldexpf((float)gq[x.e0], -a.shift);
      if (x.e1 >= 0) out[x.e1] = ldexpf((float)gq[x.e1], -a.shift);
    } else {
      const int64_t v = u - n_q;
      const int s = (int)(v / ((int64_t)a.nk * P));
      const PairIdx x = pair_idx((int)(v % ((int64_t)a.nk * P)), a.hd);
      if (x.e1 < 0) continue;
      double* gk = a.gk + (size_t)s * a.kd;
      const int t0 = ((s - base) % a.msl + a.msl) % a.msl;
      for (int t = t0; t < a.T; t += a.msl) rope_pair(gk + x.e0, gk + x.e1, base + t, x.i, a.hd, a.theta, true);
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

int attn_backward_launches(const BwdArgs& a) {
  int n = 1;  // final_kv_kernel
  for (int b = 0; b < a.B; ++b) {
    const int kvlen = (b + 1) * a.T;
    n += 7 + ((kvlen + 511) / 512 > 1 ? 1 : 0) + (a.nh / a.nk * a.T >= 256 ? 1 : 0);
  }
  return n;
}

cudaError_t attn_backward(const BwdArgs& a, cudaStream_t s) {
  if (a.T > 65535 || a.nh > 65535 || a.nk <= 0 || a.nh % a.nk) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(a.gk, 0, (size_t)a.msl * a.kd * sizeof(double), s);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(a.gv, 0, (size_t)a.msl * a.kd * sizeof(double), s);
  if (e != cudaSuccess) return e;
  const int P = (a.hd + 1) / 2;
  const int64_t ldr = 2 * (int64_t)a.kvmax;
  for (int b = 0; b < a.B; ++b) {
    const int kvlen = (b + 1) * a.T;
    ring_fill_kernel<<<grid_n((int64_t)(a.msl * a.nk + a.T * a.nh) * P), 256, 0, s>>>(a, b);
    // S = q k^T and DW = (gy 2^shift) v^T into the two halves of each scratch row
    DgemmArgs g;
    g.M = a.T;
    g.N = kvlen;
    g.K = a.hd;
    g.mod = a.msl;
    g.group = a.nh / a.nk;
    g.lda = a.qd;
    g.a_hs = a.hd;
    g.ldb = a.kd;
    g.b_hs = a.hd;
    g.ldc = (int64_t)a.nh * ldr;
    g.c_hs = ldr;
    g.heads = a.nh;
    const dim3 grid_s((kvlen + 63) / 64, (a.T + 63) / 64, a.nh);
    g.a = a.qb;
    g.b = a.ck;
    g.c = a.scratch;
    dgemm_kernel<true><<<grid_s, 256, 0, s>>>(g);
    g.a = a.gyb;
    g.b = a.cv;
    g.c = a.scratch + a.kvmax;
    dgemm_kernel<true><<<grid_s, 256, 0, s>>>(g);
    attn_bwd_row_kernel<<<dim3(a.nh, a.T), 256, 0, s>>>(a, b);
    // gq = delta k, the keys split into chunks of up to 512 (partials summed in order)
    const int qsplit = std::min(kMaxSplit, (kvlen + 511) / 512);
    DgemmArgs q;
    q.M = a.T;
    q.N = a.hd;
    q.K = kvlen;
    q.mod = a.msl;
    q.group = a.nh / a.nk;
    q.a = a.scratch + a.kvmax;
    q.lda = (int64_t)a.nh * ldr;
    q.a_hs = ldr;
    q.b = a.ck;
    q.ldb = a.kd;
    q.b_hs = a.hd;
    q.c = qsplit > 1 ? a.part_q : a.gq;
    q.ldc = a.qd;
    q.c_hs = a.hd;
    q.heads = a.nh;
    q.ksplit = qsplit;
    q.c_split = (int64_t)a.T * a.qd;
    dgemm_kernel<false><<<dim3((a.hd + 63) / 64, (a.T + 63) / 64, a.nh * qsplit), 256, 0, s>>>(q);
    if (qsplit > 1)
      sum_parts_kernel<<<grid_n((int64_t)a.T * a.qd), 256, 0, s>>>(a.part_q, qsplit, (int64_t)a.T * a.qd,
                                                                  (int64_t)a.T * a.qd, a.gq, nullptr, false);
    const int nslot = std::min(a.msl, kvlen);
    const int kvsplit = a.nh / a.nk * a.T >= 256 ? kMaxSplit : 1;
    kv_grad_kernel<<<dim3((nslot + kKvSlots - 1) / kKvSlots, a.nk, kvsplit), 256, 0, s>>>(a, b);
    if (kvsplit > 1)
      sum_parts_kernel<<<grid_n((int64_t)nslot * a.kd), 256, 0, s>>>(a.part_kv, kvsplit, (int64_t)a.msl * a.kd,
                                                                    (int64_t)nslot * a.kd, a.gv, a.gk, true);
    batch_end_kernel<<<grid_n((int64_t)(a.T * a.nh + a.msl * a.nk) * P), 256, 0, s>>>(a, b);
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
