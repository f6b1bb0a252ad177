// Attention forward on CUDA cores, covering every variant of op_attention
// (shaders/ops_mha.metal:31-127): masks of attn_allow (:1-12), ALiBi, sigmoid
// scores, GQA, any head_dim up to 256, the reference stream semantics and the
// per-sequence mode. Flash-style: K/V tiles of 32 keys in shared memory, one warp
// per query row at a time, online softmax in FP32; the reference's single-thread
// serial loop (F1 in the survey of the reference) is replaced by
// (query-tile x head x sequence) parallelism.
//
// FP32 inputs with head_dim 64/128 and no ring wrap go to the register-tiled
// kernel of attn_f32.cu instead. Also here: the split-KV decode entry (BF16 shapes
// go to decode_tc.cu, the rest to the CUDA-core decode_kernel below), the split
// combine kernel and the KV append kernel.
#include "common.cuh"
#include "kernels.h"

#include <math.h>

namespace wv {
namespace {

constexpr int kRows = 16;  // query rows per block
constexpr int kKeys = 32;  // keys per smem tile

struct MaskP {
  int mask, window, msl, prefix, window_causal;
};

// attn_allow (ops_mha.metal:1-12) on positions.
__device__ __forceinline__ bool allow(const MaskP& m, int q, int k) {
  if (m.mask == 2) return true;
  if (m.mask == 3) {
    const int w = m.window > 0 ? m.window : m.msl;
    return m.window_causal ? (k <= q && k >= q - w + 1) : (abs(q - k) < w);
  }
  if (m.mask == 4 && q < m.prefix && k < m.prefix) return true;
  return k <= q;
}

// Inclusive key-position range that can be allowed for queries [q0, q1] with
// keys below kv_end: lets a tile skip key blocks that are fully masked.
__device__ __forceinline__ void key_range(const MaskP& m, int q0, int q1, int kv_end, int& lo, int& hi) {
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

template <typename T> __device__ __forceinline__ float ldf(const T* p, size_t i);
template <> __device__ __forceinline__ float ldf<float>(const float* p, size_t i) { return p[i]; }
template <> __device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p, size_t i) {
  return __bfloat162float(p[i]);
}

template <typename T>
__global__ void __launch_bounds__(128) attn_simt_kernel(AttnArgs a, MaskP mp) {
  extern __shared__ float sm[];
  const int hd = a.head_dim, ldk_s = hd + 1;
  float* qs = sm;                      // [kRows][hd]
  float* ks = qs + kRows * hd;         // [kKeys][hd+1]
  float* vs = ks + kKeys * ldk_s;      // [kKeys][hd+1]

  // Sequence b's queries t in [0, T) sit in rows b*T + t. Per-sequence mode: query
  // position t, keys kk in [0, T) at rows b*T + kk. Stream mode (the reference):
  // query position b*T + t, keys kk in [0, (b+1)T), and key index kk reads ring
  // slot kk % MSL, which after sequence b's writes holds the newest position
  // p <= (b+1)T-1 with p == kk (mod MSL) (ops_mha.metal:58-93).
  const int head = blockIdx.y, b = blockIdx.z;
  const int group = a.num_heads / a.num_kv_heads, kh = head / group;
  const int Tq = a.seq;
  const int t0 = blockIdx.x * kRows;
  const int64_t row_base = (int64_t)b * a.seq;
  const int pos0 = a.stream_mode ? b * a.seq : 0;  // position of t = 0
  const int kv_end = a.stream_mode ? (b + 1) * a.seq : a.seq;
  const int msl = a.max_seq_len;
  const int last = kv_end - 1;
  const bool ring = a.stream_mode && kv_end > msl;
  auto key_row = [&](int kk) -> int64_t {
    if (!a.stream_mode) return row_base + kk;
    if (!ring) return kk;
    const int s = kk % msl;
    return (int64_t)s + (int64_t)msl * ((last - s) / msl);
  };
  const T* Q = static_cast<const T*>(a.q);
  const T* K = static_cast<const T*>(a.k);
  const T* V = static_cast<const T*>(a.v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float slope = a.alibi ? exp2f(-(float)(a.head_base + head + 1) * 8.0f / (float)a.total_heads) : 0.f;

  for (int i = threadIdx.x; i < kRows * hd; i += blockDim.x) {
    const int r = i / hd, d = i % hd, t = t0 + r;
    qs[i] = t < Tq ? ldf(Q, (size_t)(row_base + t) * a.ldq + (size_t)head * hd + d) : 0.f;
  }

  // key window for the whole tile (key indices = positions)
  const int tl = min(t0 + kRows, Tq) - 1;
  int lo, hi;
  key_range(mp, pos0 + t0, pos0 + tl, kv_end, lo, hi);

  constexpr int kMaxD = 8;  // hd <= 256
  float o[4][kMaxD];
  float mrow[4], lrow[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    mrow[r] = -INFINITY;
    lrow[r] = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxD; ++j) o[r][j] = 0.f;
  }
  const int nd = (hd + 31) / 32;

  for (int kb = (lo / kKeys) * kKeys; kb <= hi; kb += kKeys) {
    __syncthreads();
    for (int i = threadIdx.x; i < kKeys * hd; i += blockDim.x) {
      const int j = i / hd, d = i % hd, kk = kb + j;
      float kv = 0.f, vv = 0.f;
      if (kk <= hi) {
        const size_t off = (size_t)key_row(kk) * a.ldk + (size_t)kh * hd + d;
        kv = ldf(K, off);
        vv = ldf(V, off);
      }
      ks[j * ldk_s + d] = kv;
      vs[j * ldk_s + d] = vv;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int rr = warp * 4 + r, t = t0 + rr;
      if (t >= Tq) continue;
      const int qpos = pos0 + t;
      const int kk = kb + lane;
      const bool ok = kk <= hi && kk < kv_end && allow(mp, qpos, kk);
      float s = 0.f;
      const float* qr = qs + rr * hd;
      const float* kr = ks + lane * ldk_s;
      for (int d = 0; d < hd; ++d) s = fmaf(qr[d], kr[d], s);
      s *= a.scale;
      if (a.alibi) s -= slope * (float)abs(qpos - kk);
      float p;
      if (a.sigmoid) {
        p = ok ? 1.f / (1.f + expf(-s)) : 0.f;
      } else {
        float mx = ok ? s : -INFINITY;
        for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float mnew = fmaxf(mrow[r], mx);
        if (mnew == -INFINITY) continue;  // nothing allowed yet (warp-uniform)
        const float corr = expf(mrow[r] - mnew);
        p = ok ? expf(s - mnew) : 0.f;
        float ps = p;
        for (int off = 16; off; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        lrow[r] = lrow[r] * corr + ps;
        mrow[r] = mnew;
#pragma unroll
        for (int j = 0; j < kMaxD; ++j) o[r][j] *= corr;
      }
      for (int j2 = 0; j2 < kKeys; ++j2) {
        const float pj = __shfl_sync(0xffffffffu, p, j2);
        if (pj == 0.f) continue;
        const float* vr = vs + j2 * ldk_s;
#pragma unroll
        for (int j = 0; j < kMaxD; ++j)
          if (j < nd && lane + 32 * j < hd) o[r][j] = fmaf(pj, vr[lane + 32 * j], o[r][j]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int t = t0 + warp * 4 + r;
    if (t >= Tq) continue;
    const float inv = a.sigmoid ? 1.f : (lrow[r] > 0.f ? 1.f / lrow[r] : 0.f);
    const size_t ob = (size_t)(row_base + t) * a.ldo + (size_t)head * hd;
#pragma unroll
    for (int j = 0; j < kMaxD; ++j) {
      const int d = lane + 32 * j;
      if (j < nd && d < hd) {
        const float val = o[r][j] * inv;
        if (a.is_bf16)
          static_cast<__nv_bfloat16*>(a.out)[ob + d] = __float2bfloat16_rn(val);
        else
          static_cast<float*>(a.out)[ob + d] = val;
        if (a.out_hi) {
          const float h = to_tf32(val);
          a.out_hi[ob + d] = h;
          a.out_lo[ob + d] = val - h;
        }
      }
    }
  }
}

// ------------------------------------------------------------------ decode
// Split-KV decode. One block per (split, kv head, sequence); the G = NH/NK query
// heads of the group share every K/V row read. A key row of HD elements is read
// by LPK lanes with 16-byte loads; a warp covers 32/LPK keys per step.
template <typename T, int HD, int G>
__global__ void __launch_bounds__(128) decode_kernel(DecodeArgs a, int splits, int chunk) {
  constexpr int VEC = 16 / sizeof(T);   // elements per 16-byte load
  constexpr int LPK = HD / VEC;         // lanes per key row
  constexpr int KPW = 32 / LPK;         // keys per warp step
  constexpr int MAXG = G;
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int NK = a.num_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPK, sl = lane % LPK;  // key slot within the warp step, lane within key
  const int L = a.ctx_len[b];
  const int k0 = split * chunk, k1 = min(L, k0 + chunk);
  

  // Scores in the log2 domain: q is pre-scaled by scale*log2(e), m/l track exp2.
  constexpr int U = 4;  // key groups in flight per warp iteration (memory-level parallelism)
  float q[MAXG][VEC];
  float o[MAXG][VEC];
  float m[MAXG], l[MAXG];
  float slope2[MAXG];
  const T* Q = static_cast<const T*>(a.q);
  const float qs = a.scale * 1.4426950408889634f;
#pragma unroll
  for (int g = 0; g < MAXG; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
    const int h = kh * G + g;
    slope2[g] = a.alibi ? exp2f(-(float)(a.head_base + h + 1) * 8.0f / (float)a.total_heads) * 1.4426950408889634f
                        : 0.f;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      o[g][e] = 0.f;
      q[g][e] = ldf(Q, (size_t)b * a.ldq + (size_t)h * HD + sl * VEC + e) * qs;
    }
  }
  const T* KP = static_cast<const T*>(a.k_pool);
  const T* VP = static_cast<const T*>(a.v_pool);
  const int* bt = a.block_table + (size_t)b * a.max_pages;
  const int wstep = KPW * U;  // keys per warp iteration
  for (int base = k0 + warp * wstep; base < k1; base += 4 * wstep) {
    uint4 kr[U], vr[U];
    bool valid[U];
    int pos[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int p = base + u * KPW + sub;
      pos[u] = p;
      valid[u] = p < k1;
      if (valid[u]) {
        const int page = bt[p / kPageTokens];
        const size_t off = (((size_t)page * NK + kh) * kPageTokens + (p % kPageTokens)) * HD + sl * VEC;
        kr[u] = __ldg(reinterpret_cast<const uint4*>(KP + off));
        vr[u] = __ldg(reinterpret_cast<const uint4*>(VP + off));
      } else {
        kr[u] = vr[u] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int g = 0; g < MAXG; ++g) {
      float s[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const T* kt = reinterpret_cast<const T*>(&kr[u]);
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc = fmaf(q[g][e], ldf(kt, e), acc);
#pragma unroll
        for (int off = LPK / 2; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (a.alibi) acc -= slope2[g] * (float)abs((L - 1) - pos[u]);
        s[u] = acc;
      }
      if (a.sigmoid) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const float pr = valid[u] ? 1.f / (1.f + exp2f(-s[u])) : 0.f;
          const T* vt = reinterpret_cast<const T*>(&vr[u]);
#pragma unroll
          for (int e = 0; e < VEC; ++e) o[g][e] = fmaf(pr, ldf(vt, e), o[g][e]);
        }
        continue;
      }
      float mx = m[g];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (valid[u]) mx = fmaxf(mx, s[u]);
      if (mx == -INFINITY) continue;  // no key of this group is valid
      const float corr = exp2f(m[g] - mx);
      l[g] *= corr;
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[g][e] *= corr;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float pr = valid[u] ? exp2f(s[u] - mx) : 0.f;
        l[g] += pr;
        const T* vt = reinterpret_cast<const T*>(&vr[u]);
#pragma unroll
        for (int e = 0; e < VEC; ++e) o[g][e] = fmaf(pr, ldf(vt, e), o[g][e]);
      }
      m[g] = mx;
    }
  }
  // Combine the KPW key slots of each warp, then the 4 warps, through smem.
  __shared__ float red_m[4 * 8][MAXG], red_l[4 * 8][MAXG];
  __shared__ float red_o[MAXG][HD];
  const int slot = warp * KPW + sub;  // 0 .. 4*KPW-1
  for (int g = 0; g < G; ++g) {
    if (sl == 0) {
      red_m[slot][g] = m[g];
      red_l[slot][g] = l[g];
    }
  }
  __syncthreads();
  float gm[MAXG], scl[MAXG];
  for (int g = 0; g < G; ++g) {
    float mm = -INFINITY;
    for (int s2 = 0; s2 < 4 * KPW; ++s2) mm = fmaxf(mm, red_m[s2][g]);
    gm[g] = mm;
    scl[g] = a.sigmoid ? 1.f : (m[g] == -INFINITY ? 0.f : exp2f(m[g] - mm));
  }
  for (int i = threadIdx.x; i < G * HD; i += blockDim.x) red_o[i / HD][i % HD] = 0.f;
  __syncthreads();
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < VEC; ++e) atomicAdd(&red_o[g][sl * VEC + e], o[g][e] * scl[g]);
  __syncthreads();
  // Partial (m, l, o) of this split per query head.
  for (int i = threadIdx.x; i < G * (HD + 2); i += blockDim.x) {
    const int g = i / (HD + 2), c = i % (HD + 2);
    const int h = kh * G + g;
    float lsum = 0.f;
    if (c == HD + 1) {
      for (int s2 = 0; s2 < 4 * KPW; ++s2) {
        const float ms = red_m[s2][g];
        lsum += a.sigmoid ? red_l[s2][g] : (ms == -INFINITY ? 0.f : red_l[s2][g] * exp2f(ms - gm[g]));
      }
    }
    const float val = c < HD ? red_o[g][c] : (c == HD ? gm[g] : lsum);
    a.partial[(((size_t)b * a.num_heads + h) * splits + split) * (HD + 2) + c] = val;
  }
}

template <typename T>
__global__ void decode_combine_kernel(DecodeArgs a, int splits) {
  pdl_trigger();  // the next kernel (the output projection) may start loading its weights
  pdl_wait();     // launched as a programmatic dependent: the split partials are complete
  const int h = blockIdx.x, b = blockIdx.y, hd = a.head_dim;
  const float* P = a.partial + ((size_t)b * a.num_heads + h) * splits * (hd + 2);
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, P[s * (hd + 2) + hd]);
  float lsum = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float ms = P[s * (hd + 2) + hd];
    const float w = a.sigmoid ? 1.f : (ms == -INFINITY ? 0.f : exp2f(ms - mx));
    lsum += w * P[s * (hd + 2) + hd + 1];
  }
  const float inv = a.sigmoid ? 1.f : (lsum > 0.f ? 1.f / lsum : 0.f);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float ms = P[s * (hd + 2) + hd];
      const float w = a.sigmoid ? 1.f : (ms == -INFINITY ? 0.f : exp2f(ms - mx));
      acc += w * P[s * (hd + 2) + d];
    }
    const float val = acc * inv;
    const size_t off = (size_t)b * a.ldo + (size_t)h * hd + d;
    if (a.is_bf16)
      static_cast<__nv_bfloat16*>(a.out)[off] = __float2bfloat16_rn(val);
    else
      static_cast<float*>(a.out)[off] = val;
  }
}

template <typename T>
__global__ void kv_append_kernel(const T* k, const T* v, int ld, int rows, int kd, int hd, const int* slot,
                                 T* kp, T* vp) {
  const int NK = kd / hd;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)rows * kd;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / kd), c = (int)(i % kd);
    const int s = slot[r];
    if (s < 0) continue;
    const int page = s / kPageTokens, ps = s % kPageTokens, kh = c / hd, d = c % hd;
    const size_t off = (((size_t)page * NK + kh) * kPageTokens + ps) * hd + d;
    kp[off] = k[(size_t)r * ld + c];
    vp[off] = v[(size_t)r * ld + c];
  }
}

} // namespace

cudaError_t attn_prefill_simt(const AttnArgs& a, cudaStream_t s) {
  if (a.head_dim <= 0 || a.head_dim > 256 || a.num_kv_heads <= 0 || a.num_heads % a.num_kv_heads)
    return cudaErrorInvalidValue;
  if (attn_f32_supported(a)) return attn_prefill_f32(a, s);
  dim3 grid((a.seq + kRows - 1) / kRows, a.num_heads, a.batch);
  const size_t smem = sizeof(float) * (kRows * a.head_dim + 2 * kKeys * (a.head_dim + 1));
  MaskP mp{a.mask, a.window, a.max_seq_len, a.prefix_len, a.window_causal};
  if (a.is_bf16) {
    cudaFuncSetAttribute(attn_simt_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attn_simt_kernel<__nv_bfloat16><<<grid, 128, smem, s>>>(a, mp);
  } else {
    cudaFuncSetAttribute(attn_simt_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attn_simt_kernel<float><<<grid, 128, smem, s>>>(a, mp);
  }
  return cudaGetLastError();
}

int decode_splits(const DecodeArgs& a) {
  if (a.splits > 0) return a.splits;
  const int pairs = a.batch * a.num_kv_heads;
  const int max_by_len = std::max(1, (a.max_ctx + 255) / 256);  // >= 256 keys per split
  if (decode_tc_supported(a)) {
    // Tensor-core kernel (about 96 KB of pages in flight per CTA, 2 CTAs per SM):
    // when the (sequence, KV head) pairs leave room, as many equal splits as fill one
    // wave, so every CTA streams its keys with all the others resident; more splits
    // than that would leave a last wave of a few CTAs running the tail of the KV read
    // at a fraction of the HBM bandwidth. More pairs than one wave holds: one split.
    const int slots = decode_tc_ctas_per_sm(a.head_dim) * a.sm_count;
    return std::max(1, std::min(max_by_len, slots / pairs));
  }
  const int target = 4 * a.sm_count;
  const int sp = std::max(1, (target + pairs - 1) / pairs);
  return std::min(sp, max_by_len);
}

size_t decode_scratch_floats(const DecodeArgs& a) {
  return (size_t)a.batch * a.num_heads * decode_splits(a) * (a.head_dim + 2);
}

cudaError_t attn_decode(const DecodeArgs& a, cudaStream_t s) {
  const int G = a.num_kv_heads > 0 ? a.num_heads / a.num_kv_heads : 0;
  if (G <= 0 || G > 8 || a.num_heads % a.num_kv_heads) return cudaErrorInvalidValue;
  const int splits = decode_splits(a);
  if (decode_tc_supported(a)) {
    cudaError_t e = attn_decode_tc(a, splits, s);
    if (e != cudaSuccess) return e;
    if (a.is_bf16)
      return launch_pdl(decode_combine_kernel<__nv_bfloat16>, dim3(a.num_heads, a.batch), dim3(128), 0, s, a,
                        splits);
    return cudaGetLastError();
  }
  const int chunk = (a.max_ctx + splits - 1) / splits;
  dim3 grid(splits, a.num_kv_heads, a.batch);
#define WV_DEC_G(T, HD)                                                                  \
  switch (G) {                                                                            \
  case 1: decode_kernel<T, HD, 1><<<grid, 128, 0, s>>>(a, splits, chunk); break;          \
  case 2: decode_kernel<T, HD, 2><<<grid, 128, 0, s>>>(a, splits, chunk); break;          \
  case 4: decode_kernel<T, HD, 4><<<grid, 128, 0, s>>>(a, splits, chunk); break;          \
  case 8: decode_kernel<T, HD, 8><<<grid, 128, 0, s>>>(a, splits, chunk); break;          \
  default: return cudaErrorInvalidValue;                                                  \
  }
#define WV_DEC(T, HD)                                                                     \
  WV_DEC_G(T, HD)                                                                         \
  decode_combine_kernel<T><<<dim3(a.num_heads, a.batch), 128, 0, s>>>(a, splits);
  if (a.is_bf16) {
    if (a.head_dim == 64) { WV_DEC(__nv_bfloat16, 64) }
    else if (a.head_dim == 128) { WV_DEC(__nv_bfloat16, 128) }
    else if (a.head_dim == 256) { WV_DEC(__nv_bfloat16, 256) }
    else return cudaErrorInvalidValue;
  } else {
    if (a.head_dim == 64) { WV_DEC(float, 64) }
    else if (a.head_dim == 128) { WV_DEC(float, 128) }
    else return cudaErrorInvalidValue;
  }
#undef WV_DEC
#undef WV_DEC_G
  return cudaGetLastError();
}

cudaError_t kv_append(const void* k, const void* v, int ld, int rows, int kd, int hd, int is_bf16,
                         const int* slot, void* k_pool, void* v_pool, cudaStream_t s) {
  const int64_t n = (int64_t)rows * kd;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  if (is_bf16)
    kv_append_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v), ld, rows, kd, hd, slot,
        static_cast<__nv_bfloat16*>(k_pool), static_cast<__nv_bfloat16*>(v_pool));
  else
    kv_append_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(k), static_cast<const float*>(v), ld,
                                                 rows, kd, hd, slot, static_cast<float*>(k_pool),
                                                 static_cast<float*>(v_pool));
  return cudaGetLastError();
}

} // namespace wv
