// FormatNone round trips, decode(encode(w)) of the reference's WeightStore for
// every dtype 0-33, one element at a time. Host and device compile the same code:
// the device kernels (codec.cu) and the CPU checker that compares these functions
// with the C restatement of the reference (tests/formatnone_check.cpp). On the
// host every operation is a single IEEE operation (compile without contraction);
// on the device the _rn intrinsics keep each multiply and add separately rounded.
#pragma once
#include <stdint.h>

#include <cmath>
#include <cstring>

#if defined(__CUDACC__)
#define WV_HD __host__ __device__ __forceinline__
#else
#define WV_HD inline
#endif

namespace wv {

WV_HD uint32_t f2u(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
#endif
}
WV_HD float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  std::memcpy(&f, &u, 4);
  return f;
#endif
}
#ifdef __CUDA_ARCH__
WV_HD float rn_div(float a, float b) { return __fdiv_rn(a, b); }
WV_HD float rn_mul(float a, float b) { return __fmul_rn(a, b); }
WV_HD float rn_add(float a, float b) { return __fadd_rn(a, b); }
WV_HD float rn_sub(float a, float b) { return __fsub_rn(a, b); }
#else
WV_HD float rn_div(float a, float b) { return a / b; }
WV_HD float rn_mul(float a, float b) { return a * b; }
WV_HD float rn_add(float a, float b) { return a + b; }
WV_HD float rn_sub(float a, float b) { return a - b; }
#endif

// kNf4 (src/weights/native_codec.cpp:93-110): the 16 NF4 levels.
WV_HD float nf4_level(int c) {
  switch (c & 15) {
  case 0: return -1.0f;
  case 1: return -0.6961928009986877f;
  case 2: return -0.5250730514526367f;
  case 3: return -0.39491748809814453f;
  case 4: return -0.28444138169288635f;
  case 5: return -0.18477343022823334f;
  case 6: return -0.09105003625154495f;
  case 7: return 0.0f;
  case 8: return 0.07958029955625534f;
  case 9: return 0.16093020141124725f;
  case 10: return 0.24611230194568634f;
  case 11: return 0.33791524171829224f;
  case 12: return 0.44070982933044434f;
  case 13: return 0.5626170039176941f;
  case 14: return 0.7229568362236023f;
  default: return 1.0f;
  }
}

// Nearest-value search over an ascending table t[0..2^LOG2N-1] followed by a
// +inf sentinel t[2^LOG2N]. The reference scans every value and keeps the first
// strict minimum of |r - t[c]| (native_codec.cpp:524-533). The rounded error is
// monotone in t[c] on each side of r, and the table's spacing is far above the
// rounding of |r| <= 1, so that minimum is one of the two values bracketing r;
// on a tie the lower index wins, as in the scan. A NaN r compares false
// everywhere and gives index 0, as in the scan.
template <int LOG2N>
WV_HD int nearest_sorted(float r, const float* t) {
  int c = 0;
#pragma unroll
  for (int step = 1 << (LOG2N - 1); step; step >>= 1) c += (r >= t[c + step]) ? step : 0;
  return (fabsf(rn_sub(r, t[c + 1])) < fabsf(rn_sub(r, t[c]))) ? c + 1 : c;
}

// NF4 code of r = w/absmax (first minimum over the 16 levels); t holds the 16
// levels and +inf (nf4_table).
WV_HD int nf4_nearest(float r, const float* t) { return nearest_sorted<4>(r, t); }
WV_HD void nf4_table(float* t) {
  for (int c = 0; c < 16; ++c) t[c] = nf4_level(c);
  t[16] = u2f(0x7f800000u);
}

// Whether a dtype's round trip reads the per-tensor statistics.
WV_HD bool formatnone_needs_stats(int dtype) {
  switch (dtype) {
  case 0: case 1: case 2: case 3: case 4: case 5: case 16: case 24: case 25: return false;
  default: return dtype >= 0 && dtype <= 33;
  }
}

// Round trips of the float formats written directly on the FP32 bit pattern,
// equal to decode(encode(w)) of the scalar converters for every input (checked
// against the C restatement over all 2^32 patterns by tests/formatnone_check.cpp):
//  E4M3 (float_codecs.cpp:57-117): 0 and NaN give +0; magnitudes below 2^-6
//  (subnormal codes) give signed zero; above 448, or reaching 256 after rounding
//  (exponent field 15), +-448; otherwise 3 mantissa bits, half rounded up.
WV_HD float rt_e4m3(float f) {
  const uint32_t b = f2u(f), u = b & 0x7fffffffu, s = b & 0x80000000u;
  if (u == 0u || u > 0x7f800000u) return 0.f;
  if (u < 0x3c800000u) return u2f(s);
  uint32_t r = (u + 0x80000u) & 0xfff00000u;
  if (u > 0x43e00000u || r >= 0x43800000u) r = 0x43e00000u;
  return u2f(s | r);
}
//  E5M2 (:119-181): NaN gives a positive quiet NaN; below 2^-14 signed zero; from
//  2^16, or after rounding, +-inf; otherwise 2 mantissa bits, half rounded up.
WV_HD float rt_e5m2(float f) {
  const uint32_t b = f2u(f), u = b & 0x7fffffffu, s = b & 0x80000000u;
  if (u > 0x7f800000u) return u2f(0x7fc00000u);
  if (u < 0x38800000u) return u2f(s);
  uint32_t r = (u + 0x100000u) & 0xffe00000u;
  if (u >= 0x47800000u || r >= 0x47800000u) r = 0x7f800000u;
  return u2f(s | r);
}
//  F16 (:23-51): below 2^-14 signed zero, from 2^16 (NaN included) +-inf,
//  otherwise the mantissa truncated to 10 bits.
WV_HD float rt_f16(float f) {
  const uint32_t b = f2u(f), u = b & 0x7fffffffu, s = b & 0x80000000u;
  if (u < 0x38800000u) return u2f(s);
  if (u >= 0x47800000u) return u2f(s | 0x7f800000u);
  return u2f(s | (u & 0xffffe000u));
}

// FP4 round trip (float_codecs.cpp:184, first code of least |w - value| over
// {0, .5, 1, 1.5, 2, 3, 4, 6, -0, -.5, ..., -6}). For w < 0 every positive code
// but 0 has a larger error than code 0 (|w|) and code 8 (-0) ties code 0, so the
// choice is the nearest magnitude of |w| with ties to the smaller one, read as +0
// for magnitude 0 and -value otherwise; for w >= 0 the same with a positive
// result. Up to 6 both errors of the bracketing pair are exact (Sterbenz), so the
// choice is the exact nearest with ties down: below 1 by comparison with the
// midpoints 0.25 and 0.75, from 1 by keeping one mantissa bit, rounding half down.
// Beyond 6 rounded errors of several values can be equal and the scan keeps the
// first, so the scan runs. Errors of FLT_MAX or more never win (the scan starts
// from FLT_MAX), which maps +-FLT_MAX, +-inf and NaN to +0.
WV_HD float fp4_roundtrip(float w) {
  const float m = fabsf(w);
  if (!(m < 3.402823466e38f)) return 0.f;
  float r;
  if (m <= 6.f) {
    r = m >= 1.f ? u2f((f2u(m) + 0x1fffffu) & 0xffc00000u)
                 : (m > 0.75f ? 1.f : (m > 0.25f ? 0.5f : 0.f));
  } else {
    const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    r = 0.f;
    float best = 3.402823466e38f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float e = fabsf(rn_sub(m, mag[c]));
      if (e < best) {
        best = e;
        r = mag[c];
      }
    }
  }
  return (w < 0.f && r > 0.f) ? -r : r;
}

// Per-tensor constants of the FormatNone quantisers (src/weights/native_codec.cpp:189-560):
// absmax for the symmetric formats, the minimum and span (max - min, 1 when 0)
// for the unsigned ones.
struct RtStats {
  float amax, mn, span;
};

// Symmetric n-bit: s = absmax / (2^(n-1) - 1) (1 when 0), q = clamp(round(w / s)).
WV_HD float rt_signed(float w, float amax, int bits) {
  const int max_q = (1 << (bits - 1)) - 1, min_q = -(1 << (bits - 1));
  float s = rn_div(amax, (float)max_q);
  if (s == 0.f) s = 1.f;
  int q = (int)roundf(rn_div(w, s));
  q = q > max_q ? max_q : (q < min_q ? min_q : q);
  return rn_mul((float)q, s);
}

// Affine unsigned: q = clamp(round((w - min) / span * maxq), 0, hi), decoded
// q * (span / maxq) + min. The reference rounds and clamps in double and holds q
// in a 32- or 64-bit integer before converting it back to float; for a float qf
// that equals clamping roundf(qf) to [0, float(hi)] in float (float(2^32 - 1) =
// 2^32 and float(1e15) are the images of the integer limits; -0 gives +0),
// checked against the C restatement for every float in four ranges.
WV_HD float rt_unsigned(float w, const RtStats& st, float maxq, float hi) {
  const float scale = rn_div(st.span, maxq);
  const float x = roundf(rn_mul(rn_div(rn_sub(w, st.mn), st.span), maxq));
  const float fq = x > 0.f ? fminf(x, hi) : 0.f;
  return rn_add(rn_mul(fq, scale), st.mn);
}

// Int16/Int32/Int64: s = absmax (1 when 0), q = round(w / s * mult) in double,
// clamped (Int16) and held in an integer. |w / s| <= 1, so q is an integer of at
// most 2^31 in magnitude and float arithmetic gives the same value: roundf of the
// float product, float clamps, and for Int32 the x86-64 conversion of the
// out-of-range +2^31 (the positive absmax element) to INT32_MIN; a rounded -0
// becomes +0 as the integer would.
WV_HD float rt_wide(float w, float amax, float mult, int kind) {
  const float s = amax == 0.f ? 1.f : amax, scale = rn_div(s, mult);
  float q = roundf(rn_mul(rn_div(w, s), mult));
  if (kind == 16) q = fminf(fmaxf(q, -32768.f), 32767.f);
  if (kind == 32 && q >= 2147483648.f) q = -2147483648.f;
  if (q == 0.f) q = 0.f;  // the integer has no -0
  return rn_mul(q, scale);
}

// decode(encode(w)) for FormatNone dtype DT, element-wise in the reference's
// float/double arithmetic order (pack_native :189-560, weight_at/decode_row_f64
// :561-870), with every multiply and add rounded separately (no contraction).
// `t` is the NF4 level table of nf4_table (shared memory on the device).
template <int DT>
WV_HD float rt_elem(float w, const RtStats& st, const float* t) {
  switch (DT) {
  case 0: case 24: case 25: return (float)(double)w;  // Float64, Complex64/128 real part
  case 1: return w;
  case 2: return rt_f16(w);
  case 3: return u2f(f2u(w) & 0xffff0000u);  // BF16, truncating
  case 4: return rt_e4m3(w);
  case 5: return rt_e5m2(w);
  case 6: case 21: return rt_wide(w, st.amax, 1e6f, 64);  // Int64, Int
  case 7: return rt_wide(w, st.amax, 2147483647.0f, 32);
  case 8: return rt_wide(w, st.amax, 32767.0f, 16);
  case 9: return rt_signed(w, st.amax, 8);
  case 10: case 22: case 23: return rt_unsigned(w, st, 1e15f, 1e15f);  // Uint64, Uint, Uintptr
  case 11: return rt_unsigned(w, st, 4294967296.0f, 4294967296.0f);
  case 12: return rt_unsigned(w, st, 65535.0f, 65535.0f);
  case 13: return rt_unsigned(w, st, 255.0f, 255.0f);
  case 14: return rt_signed(w, st.amax, 4);
  case 15: return rt_unsigned(w, st, 15.0f, 15.0f);
  case 16: return fp4_roundtrip(w);
  case 17: {  // Int2: q in [-2, 1] of w / absmax
    const float s = st.amax == 0.f ? 1.f : st.amax;
    float q = fminf(fmaxf(roundf(rn_div(w, s)), -2.f), 1.f);
    if (q == 0.f) q = 0.f;  // the integer has no -0
    return rn_mul(q, s);
  }
  case 18: {  // Uint2: a = (w - min) / span in float, q = round(a * 3.0 in double)
    // a * 3 is exact in double, so q counts the thresholds 1/6, 1/2, 5/6 that a
    // reaches; 0x1.555556p-3 and 0x1.aaaaacp-1 are the least floats >= 1/6, 5/6.
    const float a = rn_div(rn_sub(w, st.mn), st.span);
    const float q = (float)((a >= 0x1.555556p-3f) + (a >= 0.5f) + (a >= 0x1.aaaaacp-1f));
    return rn_add(rn_mul(q, rn_div(st.span, 3.0f)), st.mn);
  }
  case 19: {  // Ternary: +-absmax beyond half of it, else 0
    const float s = st.amax == 0.f ? 1.f : st.amax, r = rn_div(w, s);
    return r > 0.5f ? s : (r < -0.5f ? -s : 0.f);
  }
  case 20: {  // Binary: sign times absmax
    const float s = st.amax == 0.f ? 1.f : st.amax;
    return w >= 0.f ? s : -s;
  }
  case 26: {
    const float s = st.amax == 0.f ? 1.f : st.amax;
    return rn_mul(t[nf4_nearest(rn_div(w, s), t)], s);
  }
  case 27: case 28: return rt_signed(w, st.amax, 6);  // FP6 (stored as signed 6-bit), Int6
  case 30: return rt_signed(w, st.amax, 5);
  case 32: return rt_signed(w, st.amax, 3);
  case 29: case 31: case 33: {  // Uint6, Uint5, Uint3
    constexpr int bits = DT == 29 ? 6 : (DT == 31 ? 5 : 3), max_q = (1 << bits) - 1;
    return rt_unsigned(w, st, (float)max_q, (float)max_q);
  }
  default: return 0.f;
  }
}

} // namespace wv
