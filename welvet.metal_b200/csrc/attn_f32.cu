// FP32 attention forward on CUDA cores with register tiling (the FP32 path of
// op_attention, shaders/ops_mha.metal:31-127), for head_dim 64 and 128 and every
// mask / ALiBi / sigmoid variant of the reference, without the stream-mode ring
// wrap (attn_simt_kernel keeps that case).
//
// A CTA of 256 threads owns 64 query rows and walks the allowed keys in blocks of
// 64. Thread (ty, tx) = (t / 16, t % 16) holds the 4 x 4 scores of rows 4ty.. and
// keys 4tx.. of the block and the 4 x HD/16 outputs of rows 4ty.. (dims 4tx.. of
// every 64-dim half). Per block: S = Q K^T from Q^T and K^T tiles in shared memory
// (one 16-byte load of each per 16 FMAs), online softmax in the log2 domain with the
// row max reduced over the 16 threads of a row by shuffles, P^T to shared memory,
// then O += P V (again 16 FMAs per two 16-byte loads). FP32 throughout; exp2 by
// ex2.approx (relative error below 2^-22).
#include "common.cuh"
#include "kernels.h"

#include <math.h>

namespace wv {
namespace {

constexpr int kBQ = 64;        // query rows per CTA
constexpr int kBK = 64;        // keys per block
constexpr int kLd = kBK + 4;   // padded row of the transposed tiles (floats)
constexpr int kThreads = 256;
constexpr float kLog2e = 1.4426950408889634f;

struct MaskF {
  int mask, window, msl, prefix, window_causal;
};

__device__ __forceinline__ bool allow_f(const MaskF& m, int q, int k) {
  if (m.mask == 2) return true;
  if (m.mask == 3) {
    const int w = m.window > 0 ? m.window : m.msl;
    return m.window_causal ? (k <= q && k >= q - w + 1) : (abs(q - k) < w);
  }
  if (m.mask == 4 && q < m.prefix && k < m.prefix) return true;
  return k <= q;
}

__device__ __forceinline__ void key_range_f(const MaskF& m, int q0, int q1, int kv_end, int& lo, int& hi) {
  lo = 0;
  hi = kv_end - 1;
  if (m.mask == 2) return;
  if (m.mask == 3) {
    const int w = m.window > 0 ? m.window : m.msl;
    lo = max(0, q0 - w + 1);
    hi = m.window_causal ? min(hi, q1) : min(hi, q1 + w - 1);
    return;
  }
  int h = q1;
  if (m.mask == 4 && q0 < m.prefix) h = max(h, m.prefix - 1);
  hi = min(hi, h);
}

// True when every (query, key) of the block is allowed and the keys are in range.
__device__ __forceinline__ bool block_full_f(const MaskF& m, int q0, int q1, int k0, int k1, int kv_end) {
  if (k1 >= kv_end) return false;
  if (m.mask == 2) return true;
  if (m.mask == 3) {
    const int w = m.window > 0 ? m.window : m.msl;
    return m.window_causal ? (k1 <= q0 && k0 >= q1 - w + 1) : (q1 - k0 < w && k1 - q0 < w);
  }
  if (m.mask == 4 && q1 < m.prefix && k1 < m.prefix) return true;
  return k1 <= q0;
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int HD>
__global__ void __launch_bounds__(kThreads) attn_f32_kernel(AttnArgs a, MaskF mk) {
  constexpr int NH = HD / 64;  // 64-dim halves of a row
  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);
  float* qt = sm;                 // [HD][kLd]: Q^T, pre-scaled by scale*log2(e)
  float* kt = qt + HD * kLd;      // [HD][kLd]: K^T
  float* vs = kt + HD * kLd;      // [kBK][HD]
  float* pt = vs + kBK * HD;      // [kBK][kLd]: P^T

  const int head = blockIdx.y, b = blockIdx.z;
  const int group = a.num_heads / a.num_kv_heads, kh = head / group;
  const int Tq = a.seq;
  const int t0 = blockIdx.x * kBQ;
  const int64_t row_base = (int64_t)b * a.seq;
  const int pos0 = a.stream_mode ? b * a.seq : 0;
  const int kv_end = a.stream_mode ? (b + 1) * a.seq : a.seq;
  const int64_t key_base = a.stream_mode ? 0 : row_base;  // no ring wrap on this path
  const float* Q = static_cast<const float*>(a.q);
  const float* K = static_cast<const float*>(a.k);
  const float* V = static_cast<const float*>(a.v);
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const float qscale = a.scale * kLog2e;
  const float slope2 = a.alibi ? exp2f(-(float)(a.head_base + head + 1) * 8.0f / (float)a.total_heads) * kLog2e : 0.f;

  // Q^T tile (rows past the sequence are zero). Consecutive threads take
  // consecutive rows, so the transposed stores hit consecutive banks.
  for (int i = tid; i < kBQ * (HD / 4); i += kThreads) {
    const int r = i % kBQ, d4 = (i / kBQ) * 4, t = t0 + r;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < Tq) v = *reinterpret_cast<const float4*>(Q + (size_t)(row_base + t) * a.ldq + (size_t)head * HD + d4);
    qt[(d4 + 0) * kLd + r] = v.x * qscale;
    qt[(d4 + 1) * kLd + r] = v.y * qscale;
    qt[(d4 + 2) * kLd + r] = v.z * qscale;
    qt[(d4 + 3) * kLd + r] = v.w * qscale;
  }

  const int tl = min(t0 + kBQ, Tq) - 1;
  int lo, hi;
  key_range_f(mk, pos0 + t0, pos0 + tl, kv_end, lo, hi);

  float o[4][4 * NH];
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 4 * NH; ++j) o[i][j] = 0.f;
  }

  for (int kb = (lo / kBK) * kBK; kb <= hi; kb += kBK) {
    __syncthreads();  // previous block's K^T, V and P^T are consumed
    for (int i = tid; i < kBK * (HD / 4); i += kThreads) {  // K^T: consecutive threads, consecutive keys
      const int j = i % kBK, d4 = (i / kBK) * 4, kk = kb + j;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (kk <= hi) kv = *reinterpret_cast<const float4*>(K + (size_t)(key_base + kk) * a.ldk + (size_t)kh * HD + d4);
      kt[(d4 + 0) * kLd + j] = kv.x;
      kt[(d4 + 1) * kLd + j] = kv.y;
      kt[(d4 + 2) * kLd + j] = kv.z;
      kt[(d4 + 3) * kLd + j] = kv.w;
    }
    for (int i = tid; i < kBK * (HD / 4); i += kThreads) {  // V: row-major, coalesced
      const int j = i / (HD / 4), d4 = (i % (HD / 4)) * 4, kk = kb + j;
      float4 vv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (kk <= hi) vv = *reinterpret_cast<const float4*>(V + (size_t)(key_base + kk) * a.ldk + (size_t)kh * HD + d4);
      *reinterpret_cast<float4*>(vs + j * HD + d4) = vv;
    }
    __syncthreads();

    // ---- S (log2 units) for rows 4ty+i, keys 4tx+j
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 8
    for (int d = 0; d < HD; ++d) {
      const float4 q4 = *reinterpret_cast<const float4*>(qt + d * kLd + 4 * ty);
      const float4 k4 = *reinterpret_cast<const float4*>(kt + d * kLd + 4 * tx);
      const float qv[4] = {q4.x, q4.y, q4.z, q4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
    }
    const bool full = block_full_f(mk, pos0 + t0, pos0 + tl, kb, kb + kBK - 1, kv_end) && kb + kBK - 1 <= hi;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qpos = pos0 + t0 + 4 * ty + i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kk = kb + 4 * tx + j;
        if (a.alibi) s[i][j] -= slope2 * (float)abs(qpos - kk);
        if (!full && !(kk <= hi && kk < kv_end && allow_f(mk, qpos, kk))) s[i][j] = -INFINITY;
      }
    }
    // ---- online softmax per row (16 threads per row: lanes xor 1, 2, 4, 8)
    float p[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (a.sigmoid) {
#pragma unroll
        for (int j = 0; j < 4; ++j) p[i][j] = s[i][j] == -INFINITY ? 0.f : 1.f / (1.f + ex2f(-s[i][j]));
        continue;
      }
      float mx = fmaxf(fmaxf(s[i][0], s[i][1]), fmaxf(s[i][2], s[i][3]));
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mnew = fmaxf(m[i], mx);
      const float mref = mnew == -INFINITY ? 0.f : mnew;
      const float corr = ex2f(m[i] - mref);  // m = -inf: 0 (nothing accumulated)
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        p[i][j] = ex2f(s[i][j] - mref);
        ps += p[i][j];
      }
      l[i] = l[i] * corr + ps;  // this thread's keys; reduced over the row at the end
#pragma unroll
      for (int j = 0; j < 4 * NH; ++j) o[i][j] *= corr;
      m[i] = mnew;
    }
    // ---- P^T to shared memory, then O += P V
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4*>(pt + (4 * tx + j) * kLd + 4 * ty) = make_float4(p[0][j], p[1][j], p[2][j], p[3][j]);
    __syncthreads();
#pragma unroll 4
    for (int k = 0; k < kBK; ++k) {
      const float4 p4 = *reinterpret_cast<const float4*>(pt + k * kLd + 4 * ty);
      const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
      for (int hh = 0; hh < NH; ++hh) {
        const float4 v4 = *reinterpret_cast<const float4*>(vs + k * HD + 64 * hh + 4 * tx);
        const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) o[i][4 * hh + j] = fmaf(pv[i], vv[j], o[i][4 * hh + j]);
      }
    }
  }
  // ---- row sums over the 16 threads of a row, normalise, write (and TF32 split)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float ls = l[i];
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
    const int t = t0 + 4 * ty + i;
    if (t >= Tq) continue;
    const float inv = a.sigmoid ? 1.f : (ls > 0.f ? 1.f / ls : 0.f);
    const size_t ob = (size_t)(row_base + t) * a.ldo + (size_t)head * HD;
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      const int d = 64 * hh + 4 * tx;
      const float4 v = make_float4(o[i][4 * hh] * inv, o[i][4 * hh + 1] * inv, o[i][4 * hh + 2] * inv,
                                   o[i][4 * hh + 3] * inv);
      *reinterpret_cast<float4*>(static_cast<float*>(a.out) + ob + d) = v;
      if (a.out_hi) {
        const float4 h = make_float4(to_tf32(v.x), to_tf32(v.y), to_tf32(v.z), to_tf32(v.w));
        *reinterpret_cast<float4*>(a.out_hi + ob + d) = h;
        *reinterpret_cast<float4*>(a.out_lo + ob + d) = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
      }
    }
  }
}

}  // namespace

bool attn_f32_supported(const AttnArgs& a) {
  if (a.is_bf16 || !(a.head_dim == 64 || a.head_dim == 128)) return false;
  if (a.num_kv_heads <= 0 || a.num_heads % a.num_kv_heads) return false;
  if (a.stream_mode && a.batch * a.seq > a.max_seq_len) return false;  // ring wrap: generic kernel
  if (a.ldq % 4 || a.ldk % 4 || a.ldo % 4) return false;               // 16-byte rows
  const uintptr_t al = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                       reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.out) |
                       reinterpret_cast<uintptr_t>(a.out_hi) | reinterpret_cast<uintptr_t>(a.out_lo);
  return al % 16 == 0;
}

cudaError_t attn_prefill_f32(const AttnArgs& a, cudaStream_t s) {
  if (!attn_f32_supported(a)) return cudaErrorNotSupported;
  const dim3 grid((a.seq + kBQ - 1) / kBQ, a.num_heads, a.batch);
  const MaskF mk{a.mask, a.window, a.max_seq_len, a.prefix_len, a.window_causal};
  auto go = [&](auto kern, int hd) -> cudaError_t {
    const size_t smem = sizeof(float) * (2 * hd * kLd + kBK * hd + kBK * kLd);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kThreads, smem, s>>>(a, mk);
    return cudaGetLastError();
  };
  return a.head_dim == 64 ? go(attn_f32_kernel<64>, 64) : go(attn_f32_kernel<128>, 128);
}

}  // namespace wv
