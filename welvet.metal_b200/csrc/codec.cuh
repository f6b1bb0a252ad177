// Scalar weight codecs on the device, bit-exact to the reference converters
// (src/core/float_codecs.cpp, src/weights/native_codec.cpp). Integer work on
// the IEEE bit patterns plus IEEE-rounded float division/compare, so host and
// device produce identical codes.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "formatnone.cuh"

namespace wv {

// Fills t[0..16] with the NF4 levels and the sentinel; callers sync before use.
__device__ __forceinline__ void nf4_table_init(float* t) {
  if (threadIdx.x < 17) t[threadIdx.x] = threadIdx.x < 16 ? nf4_level(threadIdx.x) : __int_as_float(0x7f800000);
}

// float_codecs.cpp:53 (truncating) / :55.
__device__ __forceinline__ uint16_t bf16_encode_trunc(float f) {
  return (uint16_t)(__float_as_uint(f) >> 16);
}
__device__ __forceinline__ float bf16_decode(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

// float_codecs.cpp:23-35 (no subnormals, truncating mantissa).
__device__ __forceinline__ uint16_t f16_encode(float f) {
  const uint32_t b = __float_as_uint(f);
  const uint16_t sign = (uint16_t)((b >> 16) & 0x8000);
  const int expo = (int)((b >> 23) & 0xff) - 127 + 15;
  const uint32_t mant = b & 0x7fffff;
  if (expo <= 0) return sign;
  if (expo >= 31) return (uint16_t)(sign | 0x7c00);
  return (uint16_t)(sign | (expo << 10) | (mant >> 13));
}
// float_codecs.cpp:37-51.
__device__ __forceinline__ float f16_decode(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  const uint32_t expo = (h >> 10) & 0x1f, mant = h & 0x3ff;
  if (expo == 0) {
    if (mant == 0) return __uint_as_float(sign);
    return __uint_as_float(sign | __float_as_uint(__fdiv_rn(__fdiv_rn((float)mant, 1024.0f), 16384.0f)));
  }
  if (expo == 31) return __uint_as_float(sign | 0x7f800000u | (mant << 13));
  return __uint_as_float(sign | ((expo - 15 + 127) << 23) | (mant << 13));
}

// float_codecs.cpp:57-97.
__device__ __forceinline__ uint8_t e4m3_encode(float f) {
  if (f == 0.0f || isnan(f)) return 0;
  uint8_t sign = 0;
  if (f < 0) {
    sign = 0x80;
    f = -f;
  }
  if (f > 448.0f) return (uint8_t)(sign | 0x7e);
  const uint32_t b = __float_as_uint(f);
  const int ex = (int)((b >> 23) & 0xff) - 127;
  uint32_t mant = b & 0x7fffff;
  int e = ex + 7;
  if (e <= 0) {
    if (e < -2) return sign;
    mant |= 0x800000;
    return (uint8_t)(sign | ((mant >> (unsigned)(21 - e)) & 0x7));
  }
  if (e >= 15) return (uint8_t)(sign | 0x7e);
  uint32_t m = (mant >> 20) & 0x7;
  if (mant & 0x80000) {
    if (++m == 8) {
      m = 0;
      if (++e >= 15) return (uint8_t)(sign | 0x7e);
    }
  }
  return (uint8_t)(sign | (e << 3) | m);
}
// float_codecs.cpp:99-117: subnormal codes decode to signed zero (the reference
// multiplies a signed zero), 0x7f/0xff decode to +-448.
__device__ __forceinline__ float e4m3_decode(uint8_t b) {
  const uint32_t sign = (b & 0x80) ? 0x80000000u : 0u;
  const int e = (b >> 3) & 0xf, m = b & 0x7;
  if (e == 0) return __uint_as_float(sign);
  if (e == 15 && m == 7) return __uint_as_float(sign | 0x43e00000u);
  return __uint_as_float(sign | ((uint32_t)(e - 7 + 127) << 23) | ((uint32_t)m << 20));
}

// float_codecs.cpp:119-158.
__device__ __forceinline__ uint8_t e5m2_encode(float f) {
  if (isnan(f)) return 0x7e;
  uint8_t sign = 0;
  if (f < 0 || signbit(f)) {
    sign = 0x80;
    if (f < 0) f = -f;
  }
  if (isinf(f)) return (uint8_t)(sign | 0x7c);
  if (f == 0.0f) return sign;
  const uint32_t b = __float_as_uint(f);
  const int ex = (int)((b >> 23) & 0xff) - 127;
  const uint32_t mant = b & 0x7fffff;
  int e = ex + 15;
  if (e <= 0) return sign;
  if (e >= 31) return (uint8_t)(sign | 0x7c);
  uint32_t m = (mant >> 21) & 0x3;
  if (mant & 0x100000) {
    if (++m == 4) {
      m = 0;
      if (++e >= 31) return (uint8_t)(sign | 0x7c);
    }
  }
  return (uint8_t)(sign | (e << 2) | m);
}
// float_codecs.cpp:160-181 (subnormals decode to signed zero).
__device__ __forceinline__ float e5m2_decode(uint8_t b) {
  const uint32_t sign = (b & 0x80) ? 0x80000000u : 0u;
  const int e = (b >> 2) & 0x1f, m = b & 0x3;
  if (e == 0) return __uint_as_float(sign);
  if (e == 31) return __uint_as_float(sign | (m == 0 ? 0x7f800000u : 0x7fc00000u));
  return __uint_as_float(sign | ((uint32_t)(e - 15 + 127) << 23) | ((uint32_t)m << 21));
}

} // namespace wv
