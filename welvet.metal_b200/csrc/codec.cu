// Weight codecs, TF32 splitting, RoPE tables and synthetic-data generation.
// These kernels are HBM-bound elementwise passes: grid-stride loops sized to a
// multiple of the SM count, 16-byte accesses where the layout allows.
#include "codec.cuh"
#include "common.cuh"
#include "formatnone.cuh"
#include "kernels.h"

#include <array>
#include <utility>

namespace wv {
namespace {

inline int grid_for(int64_t n, int per_thread = 1) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = (n / per_thread + 255) / 256;
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sms * 8));
}

#define GRID_STRIDE(i, n) \
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (n); i += (int64_t)gridDim.x * blockDim.x)

template <int DT>
__device__ __forceinline__ float4 rt_vec(float4 v, const RtStats& st, const float* t) {
  return make_float4(rt_elem<DT>(v.x, st, t), rt_elem<DT>(v.y, st, t), rt_elem<DT>(v.z, st, t),
                     rt_elem<DT>(v.w, st, t));
}

// One dtype per instantiation. stats = [absmax, min, max] of the tensor, or null
// for dtypes that need none. With 16-byte aligned pointers each thread streams
// two float4 per iteration (evict-first loads and stores; w may equal out, each
// element is read and then written by the same thread), the n % 4 tail by block
// 0; otherwise one element per thread.
template <int DT>
__global__ void __launch_bounds__(256) roundtrip_kernel(const float* w, float* out, int64_t n, const float* stats,
                                                        int vec) {
  __shared__ float t[17];
  if (DT == 26) nf4_table_init(t);
  RtStats st{1.f, 0.f, 1.f};
  if (stats) {
    st.amax = stats[0];
    st.mn = stats[1];
    const float span = __fsub_rn(stats[2], stats[1]);
    st.span = span == 0.f ? 1.f : span;
  }
  if (DT == 26) __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (!vec) {
    for (; i < n; i += stride) out[i] = rt_elem<DT>(w[i], st, t);
    return;
  }
  const int64_t n4 = n >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4* o4 = reinterpret_cast<float4*>(out);
  for (; i + stride < n4; i += 2 * stride) {
    const float4 a = __ldcs(w4 + i), b = __ldcs(w4 + i + stride);
    __stcs(o4 + i, rt_vec<DT>(a, st, t));
    __stcs(o4 + i + stride, rt_vec<DT>(b, st, t));
  }
  if (i < n4) __stcs(o4 + i, rt_vec<DT>(__ldcs(w4 + i), st, t));
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const int64_t j = (n4 << 2) + threadIdx.x;
    out[j] = rt_elem<DT>(w[j], st, t);
  }
}

using RoundtripFn = void (*)(const float*, float*, int64_t, const float*, int);
template <int... D>
constexpr std::array<RoundtripFn, sizeof...(D)> roundtrip_table(std::integer_sequence<int, D...>) {
  return {&roundtrip_kernel<D>...};
}
constexpr auto kRoundtrip = roundtrip_table(std::make_integer_sequence<int, 34>{});

__global__ void encode_kernel(int dtype, const float* w, void* codes, int64_t n, const float* nf4_scale) {
  if (dtype == 26) {
    __shared__ float t[17];
    nf4_table_init(t);
    __syncthreads();
    float s = *nf4_scale;
    if (s == 0.f) s = 1.f;
    uint8_t* out = static_cast<uint8_t*>(codes);
    GRID_STRIDE(j, (n + 1) / 2) {
      const int64_t i = 2 * j;
      const int lo = nf4_nearest(__fdiv_rn(w[i], s), t);
      const int hi = (i + 1 < n) ? nf4_nearest(__fdiv_rn(w[i + 1], s), t) : 0;
      out[j] = (uint8_t)(lo | (hi << 4));
    }
    return;
  }
  GRID_STRIDE(i, n) {
    switch (dtype) {
    case 0: static_cast<double*>(codes)[i] = (double)w[i]; break;
    case 1: static_cast<float*>(codes)[i] = w[i]; break;
    case 2: static_cast<uint16_t*>(codes)[i] = f16_encode(w[i]); break;
    case 3: static_cast<uint16_t*>(codes)[i] = bf16_encode_trunc(w[i]); break;
    case 4: static_cast<uint8_t*>(codes)[i] = e4m3_encode(w[i]); break;
    case 5: static_cast<uint8_t*>(codes)[i] = e5m2_encode(w[i]); break;
    default: break;
    }
  }
}

__global__ void decode_kernel(int dtype, const void* codes, float* out, int64_t n, const float* nf4_scale) {
  float s = 1.f;
  if (dtype == 26) {
    s = *nf4_scale;
    if (s == 0.f) s = 1.f;
  }
  GRID_STRIDE(i, n) {
    float v = 0.f;
    switch (dtype) {
    case 0: v = (float)static_cast<const double*>(codes)[i]; break;
    case 1: v = static_cast<const float*>(codes)[i]; break;
    case 2: v = f16_decode(static_cast<const uint16_t*>(codes)[i]); break;
    case 3: v = bf16_decode(static_cast<const uint16_t*>(codes)[i]); break;
    case 4: v = e4m3_decode(static_cast<const uint8_t*>(codes)[i]); break;
    case 5: v = e5m2_decode(static_cast<const uint8_t*>(codes)[i]); break;
    case 26: {
      const uint8_t b = static_cast<const uint8_t*>(codes)[i / 2];
      v = nf4_level((i & 1) ? (b >> 4) : (b & 0xf)) * s;
      break;
    }
    default: break;
    }
    out[i] = v;
  }
}

// max |w| — per-block partial maxima, then one block folds them.
__global__ void absmax_partial(const float* w, int64_t n, float* partial) {
  float m = 0.f;
  GRID_STRIDE(i, n) m = fmaxf(m, fabsf(w[i]));
  __shared__ float red[32];
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) partial[blockIdx.x] = m;
  }
}

// Block-level fold of (absmax, min, max); thread 0 writes out[blockIdx.x],
// out[stride + blockIdx.x], out[2 * stride + blockIdx.x].
__device__ __forceinline__ void stats_block_store(float m, float mn, float mx, float* out, int64_t out_stride) {
  __shared__ float red[3][32];
  for (int o = 16; o; o >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = m;
    red[1][threadIdx.x >> 5] = mn;
    red[2][threadIdx.x >> 5] = mx;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const bool live = threadIdx.x < (blockDim.x >> 5);
    m = live ? red[0][threadIdx.x] : 0.f;
    mn = live ? red[1][threadIdx.x] : INFINITY;
    mx = live ? red[2][threadIdx.x] : -INFINITY;
    for (int o = 16; o; o >>= 1) {
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (threadIdx.x == 0) {
      out[blockIdx.x] = m;
      out[out_stride + blockIdx.x] = mn;
      out[2 * out_stride + blockIdx.x] = mx;
    }
  }
}

// First pass of [absmax, min, max]: per-block partials into three arrays of
// gridDim.x floats. 16-byte loads when w is aligned (four in flight per thread),
// the n % 4 tail by block 0.
__global__ void __launch_bounds__(256) stats_first(const float* w, int64_t n, float* out, int vec) {
  float m = 0.f, mn = INFINITY, mx = -INFINITY;
  auto acc = [&](float v) {
    m = fmaxf(m, fabsf(v));
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  };
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (vec) {
    const int64_t n4 = n >> 2;
    const float4* w4 = reinterpret_cast<const float4*>(w);
    for (; i + 3 * stride < n4; i += 4 * stride) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldcs(w4 + i + u * stride);
#pragma unroll
      for (int u = 0; u < 4; ++u) acc(v[u].x), acc(v[u].y), acc(v[u].z), acc(v[u].w);
    }
    for (; i < n4; i += stride) {
      const float4 a = __ldcs(w4 + i);
      acc(a.x), acc(a.y), acc(a.z), acc(a.w);
    }
    if (blockIdx.x == 0 && threadIdx.x < (n & 3)) acc(w[(n4 << 2) + threadIdx.x]);
  } else {
    for (; i < n; i += stride) acc(w[i]);
  }
  stats_block_store(m, mn, mx, out, gridDim.x);
}

// Second pass: one block folds the three partial arrays of length n.
__global__ void stats_fold(const float* part, int64_t n, float* out3) {
  float m = 0.f, mn = INFINITY, mx = -INFINITY;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    m = fmaxf(m, part[i]);
    mn = fminf(mn, part[n + i]);
    mx = fmaxf(mx, part[2 * n + i]);
  }
  stats_block_store(m, mn, mx, out3, 1);
}

// One warp per row: absmax/448 (1 when 0), then E4M3 codes of w/scale.
__global__ void fp8_rowscale_encode_kernel(const float* w, int rows, int cols, uint8_t* codes, float* scales) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* r = w + (size_t)warp * cols;
  float m = 0.f;
  for (int c = lane; c < cols; c += 32) m = fmaxf(m, fabsf(r[c]));
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = __fdiv_rn(m, 448.0f);
  if (s == 0.f) s = 1.f;
  if (lane == 0) scales[warp] = s;
  for (int c = lane; c < cols; c += 32) codes[(size_t)warp * cols + c] = e4m3_encode(__fdiv_rn(r[c], s));
}

__global__ void fp8_rowscale_decode_kernel(const uint8_t* codes, const float* scales, int rows, int cols,
                                           void* out, int out_bf16) {
  GRID_STRIDE(i, (int64_t)rows * cols) {
    const float v = __fmul_rn(e4m3_decode(codes[i]), scales[i / cols]);
    if (out_bf16)
      static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
    else
      static_cast<float*>(out)[i] = v;
  }
}

// One warp per block of 64 elements (two per lane).
__global__ void nf4_block_encode_kernel(const float* w, int64_t n, uint8_t* packed, float* absmax) {
  __shared__ float t[17];
  nf4_table_init(t);
  __syncthreads();
  const int64_t blk = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (blk * 64 >= n) return;
  const int64_t i0 = blk * 64 + 2 * lane;
  const float a = i0 < n ? w[i0] : 0.f, b = i0 + 1 < n ? w[i0 + 1] : 0.f;
  float m = fmaxf(fabsf(a), fabsf(b));
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (m == 0.f) m = 1.f;
  if (lane == 0) absmax[blk] = m;
  if (i0 < n) {
    const int lo = nf4_nearest(__fdiv_rn(a, m), t);
    const int hi = i0 + 1 < n ? nf4_nearest(__fdiv_rn(b, m), t) : 0;
    packed[i0 / 2] = (uint8_t)(lo | (hi << 4));
  }
}

// Vectorised decodes for the aligned shapes (FP8: cols % 16 == 0; NF4: n % 32 ==
// 0): each step loads 16 code bytes (16 FP8 / 32 NF4 codes) with one scale, and
// stores the decoded values as 16-byte vectors; loads and stores are streaming
// (evict-first), two steps in flight per thread. Values are those of the scalar
// kernels (the same products, each rounded to BF16 alone).
__device__ __forceinline__ void store_decoded(void* out, int64_t first, const float* v, int count, bool bf16) {
  if (bf16) {
    uint4* o = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + first);
    for (int q = 0; q < count / 8; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[8 * q + 2 * j], v[8 * q + 2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
      __stcs(o + q, make_uint4(w[0], w[1], w[2], w[3]));
    }
  } else {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + first);
    for (int q = 0; q < count / 4; ++q) __stcs(o + q, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
  }
}

template <bool BF16>
__global__ void __launch_bounds__(256) fp8_rowscale_decode_vec_kernel(const uint4* codes, const float* scales,
                                                                      uint32_t n16, uint32_t cols16, void* out) {
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += 2 * stride) {
    const bool two = i + stride < n16;
    const uint4 c0 = __ldcs(codes + i);
    const uint4 c1 = two ? __ldcs(codes + i + stride) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h == 1 && !two) break;
      const uint32_t idx = h ? i + stride : i;
      const uint4 c = h ? c1 : c0;
      const float sc = __ldg(scales + idx / cols16);
      const uint32_t w[4] = {c.x, c.y, c.z, c.w};
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = __fmul_rn(e4m3_decode((uint8_t)(w[j >> 2] >> (8 * (j & 3)))), sc);
      store_decoded(out, (int64_t)idx * 16, v, 16, BF16);
    }
  }
}

template <bool BF16>
__global__ void __launch_bounds__(256) nf4_block_decode_vec_kernel(const uint4* packed, const float* absmax,
                                                                   uint32_t n32, void* out) {
  __shared__ float lv[16];
  if (threadIdx.x < 16) lv[threadIdx.x] = nf4_level(threadIdx.x);
  __syncthreads();
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n32; i += 2 * stride) {
    const bool two = i + stride < n32;
    const uint4 c0 = __ldcs(packed + i);
    const uint4 c1 = two ? __ldcs(packed + i + stride) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h == 1 && !two) break;
      const uint32_t idx = h ? i + stride : i;
      const uint4 c = h ? c1 : c0;
      const float am = __ldg(absmax + idx / 2);  // 32 codes of one 64-weight block
      const uint32_t w[4] = {c.x, c.y, c.z, c.w};
      float v[32];
#pragma unroll
      for (int j = 0; j < 16; ++j) {  // byte j: low nibble = even weight, high = odd
        const uint32_t b = (w[j >> 2] >> (8 * (j & 3))) & 0xffu;
        v[2 * j] = __fmul_rn(lv[b & 0xf], am);
        v[2 * j + 1] = __fmul_rn(lv[b >> 4], am);
      }
      store_decoded(out, (int64_t)idx * 32, v, 32, BF16);
    }
  }
}

__global__ void nf4_block_decode_kernel(const uint8_t* packed, const float* absmax, int64_t n, void* out,
                                        int out_bf16) {
  GRID_STRIDE(i, n) {
    const uint8_t b = packed[i / 2];
    const float v = __fmul_rn(nf4_level((i & 1) ? (b >> 4) : (b & 0xf)), absmax[i / 64]);
    if (out_bf16)
      static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
    else
      static_cast<float*>(out)[i] = v;
  }
}

// Codes whose reference decoding differs from IEEE-style E4M3 are rewritten to a
// code with the same reference value: subnormal codes (exponent 0, mantissa != 0)
// decode to +-0 in the reference, 0x7f/0xff decode to +-448 (= 0x7e/0xfe).
__global__ void fp8_normalize_kernel(uint8_t* codes, int64_t n) {
  GRID_STRIDE(i, n) {
    const uint8_t c = codes[i];
    if ((c & 0x78) == 0)
      codes[i] = c & 0x80;
    else if ((c & 0x7f) == 0x7f)
      codes[i] = c - 1;
  }
}

__global__ void split_tf32_kernel(const float* x, float* hi, float* lo, int64_t n) {
  GRID_STRIDE(i, n) {
    const float v = x[i];
    const float h = to_tf32(v);
    hi[i] = h;
    lo[i] = v - h;
  }
}

__global__ void cast_f32_bf16_kernel(const float* x, __nv_bfloat16* y, int64_t n) {
  GRID_STRIDE(i, n) y[i] = __float2bfloat16_rn(x[i]);
}
__global__ void cast_bf16_f32_kernel(const __nv_bfloat16* x, float* y, int64_t n) {
  GRID_STRIDE(i, n) y[i] = __bfloat162float(x[i]);
}

// rope_gpu (shaders/ops_mha.metal:13-30): power = theta^(fl32(2i/hd)),
// angle = pos / power, evaluated in double and rounded once to float.
__global__ void rope_table_kernel(float2* tab, int max_pos, int hd, double theta) {
  const int half = hd / 2;
  const double ltheta = log(theta);
  GRID_STRIDE(idx, (int64_t)max_pos * half) {
    const int pos = (int)(idx / half), i = (int)(idx % half);
    const float e = __fdiv_rn((float)(2 * i), (float)hd);
    const double power = exp(ltheta * (double)e);
    const double angle = (double)pos / power;
    double s, c;
    sincos(angle, &s, &c);
    tab[idx] = make_float2((float)c, (float)s);
  }
}

__global__ void rope_apply_kernel(void* x, int is_bf16, int64_t M, int ld, int cols, int hd,
                                  const float2* tab, int max_pos, const int* positions, int pos_mod) {
  const int half = hd / 2;
  const int pairs_per_row = (cols / hd) * half;
  GRID_STRIDE(idx, M * pairs_per_row) {
    const int64_t row = idx / pairs_per_row;
    const int r = (int)(idx % pairs_per_row);
    const int head = r / half, i = r % half;
    int pos = positions ? positions[row] : (pos_mod > 0 ? (int)(row % pos_mod) : (int)row);
    if (pos < 0 || pos >= max_pos) continue;
    const float2 cs = tab[(size_t)pos * half + i];
    const size_t ia = (size_t)row * ld + (size_t)head * hd + i, ib = ia + half;
    if (is_bf16) {
      __nv_bfloat16* p = static_cast<__nv_bfloat16*>(x);
      const float a = __bfloat162float(p[ia]), b = __bfloat162float(p[ib]);
      p[ia] = __float2bfloat16_rn(a * cs.x - b * cs.y);
      p[ib] = __float2bfloat16_rn(a * cs.y + b * cs.x);
    } else {
      float* p = static_cast<float*>(x);
      const float a = p[ia], b = p[ib];
      p[ia] = a * cs.x - b * cs.y;
      p[ib] = a * cs.y + b * cs.x;
    }
  }
}

// SplitMix64 finaliser on (seed * golden + index): a counter-based stream, so
// element i is the same wherever and in whatever order it is generated.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ double unif01(uint64_t seed, uint64_t i) {
  return (double)(mix64(seed * 0xD1B54A32D192ED03ull + i) >> 11) * 0x1.0p-53;
}

__global__ void fill_kernel(void* dst, int is_bf16, int64_t n, uint64_t seed, uint64_t offset, int kind,
                            double a) {
  GRID_STRIDE(i, n) {
    const uint64_t gi = offset + (uint64_t)i;
    double v;
    if (kind == 0) {
      v = a * (2.0 * unif01(seed, gi) - 1.0);
    } else {
      const double u1 = unif01(seed, 2 * gi), u2 = unif01(seed, 2 * gi + 1);
      v = a * sqrt(-2.0 * log(1.0 - u1)) * cos(6.283185307179586 * u2);
    }
    if (is_bf16)
      static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn((float)v);
    else
      static_cast<float*>(dst)[i] = (float)v;
  }
}

} // namespace

bool codec_dtype_supported(int dtype) { return dtype >= 0 && dtype <= 33; }
bool codec_needs_stats(int dtype) { return formatnone_needs_stats(dtype); }
cudaError_t codec_roundtrip_f32(int dtype, const float* w, float* out, int64_t n, const float* stats,
                                cudaStream_t s) {
  if (!codec_dtype_supported(dtype)) return cudaErrorInvalidValue;
  if (n <= 0) return cudaSuccess;
  const int vec = ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  const int grid = vec ? grid_for((n >> 2) + 1, 2) : grid_for(n);
  kRoundtrip[dtype]<<<grid, 256, 0, s>>>(w, out, n, stats, vec);
  return cudaGetLastError();
}
cudaError_t stats_f32(const float* w, int64_t n, float* out3, float* scratch, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const int vec = (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  const int g = std::min(vec ? grid_for((n >> 2) + 1, 4) : grid_for(n), 1024);
  stats_first<<<g, 256, 0, s>>>(w, n, scratch, vec);
  stats_fold<<<1, 1024, 0, s>>>(scratch, g, out3);
  return cudaGetLastError();
}
cudaError_t codec_encode(int dtype, const float* w, void* codes, int64_t n, const float* nf4_scale,
                         cudaStream_t s) {
  encode_kernel<<<grid_for(n), 256, 0, s>>>(dtype, w, codes, n, nf4_scale);
  return cudaGetLastError();
}
cudaError_t codec_decode(int dtype, const void* codes, float* out, int64_t n, const float* nf4_scale,
                         cudaStream_t s) {
  decode_kernel<<<grid_for(n), 256, 0, s>>>(dtype, codes, out, n, nf4_scale);
  return cudaGetLastError();
}
cudaError_t absmax_f32(const float* w, int64_t n, float* out, float* scratch, cudaStream_t s) {
  const int g = std::min(grid_for(n), 1024);
  absmax_partial<<<g, 256, 0, s>>>(w, n, scratch);
  absmax_partial<<<1, 1024, 0, s>>>(scratch, g, out);
  return cudaGetLastError();
}
cudaError_t fp8_rowscale_encode(const float* w, int rows, int cols, uint8_t* codes, float* scales,
                                cudaStream_t s) {
  fp8_rowscale_encode_kernel<<<(rows + 7) / 8, 256, 0, s>>>(w, rows, cols, codes, scales);
  return cudaGetLastError();
}
cudaError_t fp8_rowscale_decode(const uint8_t* codes, const float* scales, int rows, int cols, void* out,
                                int out_bf16, cudaStream_t s) {
  const int64_t n = (int64_t)rows * cols;
  if (cols % 16 == 0 && n / 16 < (int64_t{1} << 31) && reinterpret_cast<uintptr_t>(codes) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(out) % 16 == 0) {
    const uint32_t n16 = (uint32_t)(n / 16);
    if (out_bf16)
      fp8_rowscale_decode_vec_kernel<true><<<grid_for(n16), 256, 0, s>>>(reinterpret_cast<const uint4*>(codes),
                                                                          scales, n16, cols / 16, out);
    else
      fp8_rowscale_decode_vec_kernel<false><<<grid_for(n16), 256, 0, s>>>(reinterpret_cast<const uint4*>(codes),
                                                                           scales, n16, cols / 16, out);
    return cudaGetLastError();
  }
  fp8_rowscale_decode_kernel<<<grid_for((int64_t)rows * cols), 256, 0, s>>>(codes, scales, rows, cols, out,
                                                                             out_bf16);
  return cudaGetLastError();
}
// FormatNone codes of the reference quantisers kept resident for the dequantising
// GEMM (native_codec.cpp pack_native :189-560): Int8 (one byte, q = clamp(round(w /
// s), -128, 127), s = absmax / 127), Int4 (two per byte, low nibble first, s =
// absmax / 7, q in [-8, 7]) and FP4 (E2M1 code of fp4_roundtrip's value, no scale);
// the same float arithmetic as rt_signed / fp4_roundtrip, so code * scale is the
// reference's decoded weight. row_scale[r] = s for each of the n / cols rows (1 for
// FP4). stats = [absmax, min, max] of w (stats_f32).
__global__ void fn_codes_kernel(int dtype, const float* w, int64_t n, int cols, const float* stats, uint8_t* codes,
                                float* row_scale) {
  const int max_q = dtype == 9 ? 127 : 7;
  float sc = 1.f;
  if (dtype != 16) {
    sc = rn_div(stats[0], (float)max_q);
    if (sc == 0.f) sc = 1.f;
  }
  auto code_of = [&](float x) -> uint32_t {
    if (dtype == 16) {
      const float r = fp4_roundtrip(x);
      const float m = fabsf(r);
      const uint32_t c = m < 0.25f ? 0u : m < 0.75f ? 1u : m < 1.25f ? 2u : m < 1.75f ? 3u
                       : m < 2.5f ? 4u : m < 3.5f ? 5u : m < 5.f ? 6u : 7u;
      return (r < 0.f ? 8u : 0u) | c;
    }
    int q = (int)roundf(rn_div(x, sc));
    q = q > max_q ? max_q : (q < -max_q - 1 ? -max_q - 1 : q);
    return (uint32_t)q & (dtype == 9 ? 0xffu : 0xfu);
  };
  const int64_t nb = dtype == 9 ? n : (n + 1) / 2;  // code bytes
  GRID_STRIDE(i, nb) {
    if (dtype == 9) {
      codes[i] = (uint8_t)code_of(w[i]);
    } else {
      const uint32_t lo = code_of(w[2 * i]);
      const uint32_t hi = 2 * i + 1 < n ? code_of(w[2 * i + 1]) : 0u;
      codes[i] = (uint8_t)(lo | (hi << 4));
    }
    const int64_t e0 = dtype == 9 ? i : 2 * i;
    if (e0 % cols == 0) row_scale[e0 / cols] = sc;
    if (dtype != 9 && (e0 + 1) % cols == 0 && e0 + 1 < n) row_scale[(e0 + 1) / cols] = sc;
  }
}

cudaError_t formatnone_codes_encode(int dtype, const float* w, int64_t n, int cols, const float* stats,
                                    uint8_t* codes, float* row_scale, cudaStream_t s) {
  if (dtype != 9 && dtype != 14 && dtype != 16) return cudaErrorInvalidValue;
  fn_codes_kernel<<<grid_for(dtype == 9 ? n : (n + 1) / 2), 256, 0, s>>>(dtype, w, n, cols, stats, codes,
                                                                       row_scale);
  return cudaGetLastError();
}

cudaError_t nf4_block_encode(const float* w, int64_t n, uint8_t* packed, float* absmax, cudaStream_t s) {
  const int64_t blocks = (n + 63) / 64;
  nf4_block_encode_kernel<<<(int)((blocks + 7) / 8), 256, 0, s>>>(w, n, packed, absmax);
  return cudaGetLastError();
}
cudaError_t nf4_block_decode(const uint8_t* packed, const float* absmax, int64_t n, void* out, int out_bf16,
                             cudaStream_t s) {
  if (n % 32 == 0 && n / 32 < (int64_t{1} << 31) && reinterpret_cast<uintptr_t>(packed) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(out) % 16 == 0) {
    const uint32_t n32 = (uint32_t)(n / 32);
    if (out_bf16)
      nf4_block_decode_vec_kernel<true><<<grid_for(n32), 256, 0, s>>>(reinterpret_cast<const uint4*>(packed),
                                                                       absmax, n32, out);
    else
      nf4_block_decode_vec_kernel<false><<<grid_for(n32), 256, 0, s>>>(reinterpret_cast<const uint4*>(packed),
                                                                        absmax, n32, out);
    return cudaGetLastError();
  }
  nf4_block_decode_kernel<<<grid_for(n), 256, 0, s>>>(packed, absmax, n, out, out_bf16);
  return cudaGetLastError();
}
cudaError_t fp8_normalize(uint8_t* codes, int64_t n, cudaStream_t s) {
  fp8_normalize_kernel<<<grid_for(n), 256, 0, s>>>(codes, n);
  return cudaGetLastError();
}
cudaError_t split_tf32(const float* x, float* hi, float* lo, int64_t n, cudaStream_t s) {
  split_tf32_kernel<<<grid_for(n), 256, 0, s>>>(x, hi, lo, n);
  return cudaGetLastError();
}
cudaError_t cast_f32_bf16(const float* x, void* y, int64_t n, cudaStream_t s) {
  cast_f32_bf16_kernel<<<grid_for(n), 256, 0, s>>>(x, static_cast<__nv_bfloat16*>(y), n);
  return cudaGetLastError();
}
cudaError_t cast_bf16_f32(const void* x, float* y, int64_t n, cudaStream_t s) {
  cast_bf16_f32_kernel<<<grid_for(n), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), y, n);
  return cudaGetLastError();
}
cudaError_t rope_table(float2* tab, int max_pos, int head_dim, double theta, cudaStream_t s) {
  if (head_dim < 2) return cudaSuccess;
  rope_table_kernel<<<grid_for((int64_t)max_pos * (head_dim / 2)), 256, 0, s>>>(tab, max_pos, head_dim, theta);
  return cudaGetLastError();
}
cudaError_t rope_apply(void* x, int is_bf16, int64_t M, int ld, int cols, int head_dim, const float2* tab,
                       int max_pos, const int* positions, int pos_mod, cudaStream_t s) {
  if (head_dim < 2 || cols <= 0) return cudaSuccess;
  rope_apply_kernel<<<grid_for(M * (cols / head_dim) * (head_dim / 2)), 256, 0, s>>>(
      x, is_bf16, M, ld, cols, head_dim, tab, max_pos, positions, pos_mod);
  return cudaGetLastError();
}
cudaError_t fill_synthetic(void* dst, int is_bf16, int64_t n, uint64_t seed, uint64_t offset, int kind,
                           double a, cudaStream_t s) {
  fill_kernel<<<grid_for(n), 256, 0, s>>>(dst, is_bf16, n, seed, offset, kind, a);
  return cudaGetLastError();
}

} // namespace wv
