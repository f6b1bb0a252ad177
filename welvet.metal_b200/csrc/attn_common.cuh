// Pieces shared by the tensor-core flash-attention kernels (attn_tc.cu: BF16,
// attn_tf32.cu: FP32 through 3xTF32): launch parameters, the reference's mask
// predicate attn_allow (shaders/ops_mha.metal:1-12) on positions and the key
// intervals it admits, and packed FP32 arithmetic for the softmax.
#pragma once
#include <cstdint>

namespace wv {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // lazy O rescale: log2 units

struct FParams {
  int batch, seq, num_heads, num_kv_heads, stream_mode;
  int mask, window, msl, prefix, window_causal, head_base, total_heads;
  float scale_log2;  // scale * log2(e)
  void* out;
  int ldo;
  int nqt;
  uint32_t* err;
};

// attn_allow (ops_mha.metal:1-12) on positions.
__device__ __forceinline__ bool allow(const FParams& p, int q, int k) {
  if (p.mask == 2) return true;
  if (p.mask == 3) {
    const int w = p.window > 0 ? p.window : p.msl;
    return p.window_causal ? (k <= q && k >= q - w + 1) : (abs(q - k) < w);
  }
  if (p.mask == 4 && q < p.prefix && k < p.prefix) return true;
  return k <= q;
}

// Inclusive key range allowed to queries [q0, q1] below kv_end.
__device__ __forceinline__ void key_range(const FParams& p, int q0, int q1, int kv_end, int& lo, int& hi) {
  lo = 0;
  hi = kv_end - 1;
  if (p.mask == 2) return;
  if (p.mask == 3) {
    const int w = p.window > 0 ? p.window : p.msl;
    lo = max(0, q0 - w + 1);
    hi = p.window_causal ? min(hi, q1) : min(hi, q1 + w - 1);
    return;
  }
  int h = q1;
  if (p.mask == 4 && q0 < p.prefix) h = max(h, p.prefix - 1);
  hi = min(hi, h);
}

// True when every (query, key) pair of the block is allowed and in range.
__device__ __forceinline__ bool block_full(const FParams& p, int q0, int q1, int k0, int k1, int kv_end) {
  if (k1 >= kv_end) return false;
  if (p.mask == 2) return true;
  if (p.mask == 3) {
    const int w = p.window > 0 ? p.window : p.msl;
    return p.window_causal ? (k1 <= q0 && k0 >= q1 - w + 1) : (q1 - k0 < w && k1 - q0 < w);
  }
  if (p.mask == 4 && q1 < p.prefix && k1 < p.prefix) return true;
  return k1 <= q0;
}


__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed FP32 pairs (sm_100 f32x2 ALU ops) and a three-input max.
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

} // namespace
} // namespace wv
