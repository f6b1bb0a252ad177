// Test infrastructure — NOT part of the product. Restatement of the reference's
// scalar weight codecs for the dtypes on the MHA path, plus the two extension
// formats (per-row FP8 scale, block-64 NF4) built on the same element codes.
// The restatement is pinned bit-for-bit against the reference's own codec source
// compiled into oracle/_ref (tests/test_oracle_pin.py).
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <vector>

namespace {
// FP4 (e2m1) grid of the reference converter, code order (float_codecs.cpp:184).
constexpr float kFp4Grid[16] = {0, 0.5f, 1, 1.5f, 2, 3, 4, 6, -0.0f, -0.5f, -1, -1.5f, -2, -3, -4, -6};

uint32_t bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}
float fbits(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// kNf4 codebook, native_codec.cpp:93-110 (the standard 16-level NF4 table).
const float kNf4Levels[16] = {-1.0f,
                              -0.6961928009986877f,
                              -0.5250730514526367f,
                              -0.39491748809814453f,
                              -0.28444138169288635f,
                              -0.18477343022823334f,
                              -0.09105003625154495f,
                              0.0f,
                              0.07958029955625534f,
                              0.16093020141124725f,
                              0.24611230194568634f,
                              0.33791524171829224f,
                              0.44070982933044434f,
                              0.5626170039176941f,
                              0.7229568362236023f,
                              1.0f};

float absmax(const float* w, int64_t n) {
  float m = 0;
  for (int64_t i = 0; i < n; ++i) {
    const float a = std::fabs(w[i]);
    if (a > m) m = a;
  }
  return m;
}

// Nearest level with the first minimum winning (strict <), native_codec.cpp:524-533.
int nf4_nearest(float r) {
  int best = 0;
  float best_err = std::numeric_limits<float>::max();
  for (int c = 0; c < 16; ++c) {
    const float e = std::fabs(r - kNf4Levels[c]);
    if (e < best_err) {
      best_err = e;
      best = c;
    }
  }
  return best;
}

void put16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xff);
  p[1] = (uint8_t)(v >> 8);
}
uint16_t get16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

} // namespace

extern "C" {

uint16_t oracle_bf16_encode(float f) { return (uint16_t)(bits(f) >> 16); }
float oracle_bf16_decode(uint16_t h) { return fbits((uint32_t)h << 16); }

uint16_t oracle_f16_encode(float f) {
  const uint32_t b = bits(f);
  const uint16_t sign = (uint16_t)((b >> 16) & 0x8000);
  const int expo = (int)((b >> 23) & 0xff) - 127 + 15;
  const uint32_t mant = b & 0x7fffff;
  if (expo <= 0) return sign;           // no subnormals: flush
  if (expo >= 31) return (uint16_t)(sign | 0x7c00);
  return (uint16_t)(sign | (expo << 10) | (mant >> 13)); // truncating
}

float oracle_f16_decode(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  const uint32_t expo = (h >> 10) & 0x1f, mant = h & 0x3ff;
  if (expo == 0) {
    if (mant == 0) return fbits(sign);
    return fbits(sign | bits((float)mant / 1024.0f / 16384.0f));
  }
  if (expo == 31) return fbits(sign | 0x7f800000u | (mant << 13));
  return fbits(sign | ((expo - 15 + 127) << 23) | (mant << 13));
}

// E4M3 encode, float_codecs.cpp:57-97: NaN and 0 -> 0x00; >448 saturates to
// 0x7e; rounding adds one on the first dropped mantissa bit (half away from
// zero); subnormal range truncates; below 2^-9 flushes to signed zero.
uint8_t oracle_e4m3_encode(float f) {
  if (f == 0.0f || std::isnan(f)) return 0;
  uint8_t sign = 0;
  if (f < 0) {
    sign = 0x80;
    f = -f;
  }
  if (f > 448.0f) return (uint8_t)(sign | 0x7e);
  const uint32_t b = bits(f);
  const int exp = (int)((b >> 23) & 0xff) - 127;
  uint32_t mant = b & 0x7fffff;
  int e = exp + 7;
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

// E4M3 decode, float_codecs.cpp:99-117: the subnormal branch multiplies a
// signed ZERO, so every subnormal code decodes to +-0; 0x7f/0xff decode to +-448.
float oracle_e4m3_decode(uint8_t b) {
  const uint32_t sign = (b & 0x80) ? 0x80000000u : 0u;
  const int e = (b >> 3) & 0xf, m = b & 0x7;
  if (e == 0) {
    if (m == 0) return fbits(sign);
    return fbits(sign) * (float)m / 8.0f / 64.0f;
  }
  if (e == 15 && m == 7) return fbits(sign | bits(448.0f));
  return fbits(sign | ((uint32_t)(e - 7 + 127) << 23) | ((uint32_t)m << 20));
}

uint8_t oracle_e5m2_encode(float f) {
  if (std::isnan(f)) return 0x7e;
  uint8_t sign = 0;
  if (f < 0 || std::signbit(f)) {
    sign = 0x80;
    if (f < 0) f = -f;
  }
  if (std::isinf(f)) return (uint8_t)(sign | 0x7c);
  if (f == 0.0f) return sign;
  const uint32_t b = bits(f);
  const int exp = (int)((b >> 23) & 0xff) - 127;
  const uint32_t mant = b & 0x7fffff;
  int e = exp + 15;
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

float oracle_e5m2_decode(uint8_t b) {
  const uint32_t sign = (b & 0x80) ? 0x80000000u : 0u;
  const int e = (b >> 2) & 0x1f, m = b & 0x3;
  if (e == 0) {
    if (m == 0) return fbits(sign);
    return fbits(sign) * (float)m / 4.0f / 16384.0f;
  }
  if (e == 31) return fbits(sign | (m == 0 ? 0x7f800000u : 0x7fc00000u));
  return fbits(sign | ((uint32_t)(e - 15 + 127) << 23) | ((uint32_t)m << 21));
}

float oracle_nf4_level(int32_t code) { return kNf4Levels[code & 0xf]; }

int64_t oracle_encode(int32_t dtype, const float* w, int64_t n, uint8_t* out, float* scale) {
  *scale = 1.0f;
  switch (dtype) {
  case 0: // Float64: IEEE bits of double(w), little-endian (native_codec.cpp:193-198)
    for (int64_t i = 0; i < n; ++i) {
      const double d = (double)w[i];
      std::memcpy(out + i * 8, &d, 8);
    }
    return n * 8;
  case 1: // Float32 keeps the f32 buffer (native_codec.cpp:826-831)
    std::memcpy(out, w, (size_t)n * 4);
    return n * 4;
  case 2:
    for (int64_t i = 0; i < n; ++i) put16(out + i * 2, oracle_f16_encode(w[i]));
    return n * 2;
  case 3:
    for (int64_t i = 0; i < n; ++i) put16(out + i * 2, oracle_bf16_encode(w[i]));
    return n * 2;
  case 4:
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_e4m3_encode(w[i]);
    return n;
  case 5:
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_e5m2_encode(w[i]);
    return n;
  case 26: { // NF4, one absmax for the whole tensor (native_codec.cpp:519-542)
    if (n <= 0) return 0;
    float s = absmax(w, n);
    if (s == 0) s = 1;
    std::memset(out, 0, (size_t)((n + 1) / 2));
    for (int64_t i = 0; i < n; ++i) {
      const int best = nf4_nearest(w[i] / s);
      if (i % 2 == 0)
        out[i / 2] = (uint8_t)(best & 0xf);
      else
        out[i / 2] |= (uint8_t)((best & 0xf) << 4);
    }
    *scale = s;
    return (n + 1) / 2;
  }
  default:
    return -2;
  }
}

int32_t oracle_decode(int32_t dtype, const uint8_t* raw, int64_t n, float scale, float* out) {
  switch (dtype) {
  case 0:
    for (int64_t i = 0; i < n; ++i) {
      double d;
      std::memcpy(&d, raw + i * 8, 8);
      out[i] = (float)d;
    }
    return 0;
  case 1:
    std::memcpy(out, raw, (size_t)n * 4);
    return 0;
  case 2:
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_f16_decode(get16(raw + i * 2));
    return 0;
  case 3:
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_bf16_decode(get16(raw + i * 2));
    return 0;
  case 4:
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_e4m3_decode(raw[i]);
    return 0;
  case 5:
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_e5m2_decode(raw[i]);
    return 0;
  case 26: {
    const float s = scale == 0 ? 1.0f : scale;
    for (int64_t i = 0; i < n; ++i) {
      const int code = (i % 2 == 0) ? (raw[i / 2] & 0xf) : (raw[i / 2] >> 4);
      out[i] = kNf4Levels[code] * s;
    }
    return 0;
  }
  default:
    return -2;
  }
}

// decode(encode(w)) for every FormatNone dtype of the reference
// (pack_native, src/weights/native_codec.cpp:189-560, and weight_at /
// decode_row_f64, :561-870), element by element in float arithmetic without
// contraction. Per-tensor statistics: absmax (signed formats, Ternary, Binary,
// NF4) or min/max (unsigned formats, stored minimum added back on decode).
// Platform choices of the reference as built here (x86-64): Int and Uint are the
// 64-bit forms, and a double at or above 2^31 converted to int32 (Int32's
// positive absmax element, w/s*2147483648.0f) gives INT32_MIN.
int32_t oracle_roundtrip(int32_t dtype, const float* w, int64_t n, float* out) {
  if (n <= 0) return 0;
  float amax = absmax(w, n), mn = w[0], mx = w[0];
  for (int64_t i = 1; i < n; ++i) {
    if (w[i] < mn) mn = w[i];
    if (w[i] > mx) mx = w[i];
  }
  const float span = (mx - mn) == 0 ? 1.0f : (mx - mn);
  auto rnd = [](double v) { return std::round(v); };
  auto clampd = [](double v, double lo, double hi) { return v < lo ? lo : (v > hi ? hi : v); };
  auto signed_nbit = [&](int bits) {
    const int max_q = (1 << (bits - 1)) - 1, min_q = -(1 << (bits - 1));
    float s = amax / (float)max_q;
    if (s == 0) s = 1;
    for (int64_t i = 0; i < n; ++i) {
      int q = (int)std::round(w[i] / s);
      q = q > max_q ? max_q : (q < min_q ? min_q : q);
      out[i] = (float)q * s;
    }
  };
  auto unsigned_q = [&](float maxq_f, double clamp_hi, bool as_u64) {
    const float scale = span / maxq_f;
    for (int64_t i = 0; i < n; ++i) {
      const float qf = (w[i] - mn) / span * maxq_f;
      const double q = clampd(rnd((double)qf), 0.0, clamp_hi);
      const float fq = as_u64 ? (float)(uint64_t)q : (float)(uint32_t)q;
      out[i] = fq * scale + mn;
    }
  };
  switch (dtype) {
  case 0: case 24: case 25:  // Float64, Complex64 / Complex128 (real part)
    for (int64_t i = 0; i < n; ++i) out[i] = (float)(double)w[i];
    return 0;
  case 1:
    std::memcpy(out, w, (size_t)n * 4);
    return 0;
  case 2: case 3: case 4: case 5: case 26: {
    std::vector<uint8_t> raw((size_t)n * 8 + 8);
    float scale = 1.0f;
    if (oracle_encode(dtype, w, n, raw.data(), &scale) < 0) return -2;
    return oracle_decode(dtype, raw.data(), n, scale, out);
  }
  case 6: case 21: {  // Int64, Int (64-bit host): w/s*1e6 rounded
    const float s = amax == 0 ? 1.0f : amax, scale = s / 1e6f;
    for (int64_t i = 0; i < n; ++i) {
      const float qf = w[i] / s * 1e6f;
      out[i] = (float)(int64_t)rnd((double)qf) * scale;
    }
    return 0;
  }
  case 7: {  // Int32
    const float s = amax == 0 ? 1.0f : amax, scale = s / 2147483647.0f;
    for (int64_t i = 0; i < n; ++i) {
      const float qf = w[i] / s * 2147483647.0f;
      const double r = rnd((double)qf);
      const int32_t q = (r >= 2147483648.0 || r < -2147483648.0) ? INT32_MIN : (int32_t)r;
      out[i] = (float)q * scale;
    }
    return 0;
  }
  case 8: {  // Int16
    const float s = amax == 0 ? 1.0f : amax, scale = s / 32767.0f;
    for (int64_t i = 0; i < n; ++i) {
      const float qf = w[i] / s * 32767.0f;
      out[i] = (float)(int)clampd(rnd((double)qf), -32768.0, 32767.0) * scale;
    }
    return 0;
  }
  case 9: {  // Int8
    float s = amax / 127.0f;
    if (s == 0) s = 1;
    for (int64_t i = 0; i < n; ++i) out[i] = (float)(int)clampd(std::round(w[i] / s), -128.0, 127.0) * s;
    return 0;
  }
  case 13: unsigned_q(255.0f, 255.0, false); return 0;                     // Uint8
  case 12: unsigned_q(65535.0f, 65535.0, false); return 0;                 // Uint16
  case 11: unsigned_q((float)4294967295u, 4294967295.0, false); return 0;  // Uint32
  case 10: case 22: case 23: unsigned_q(1e15f, 1e15, true); return 0;      // Uint64, Uint, Uintptr
  case 14: {  // Int4
    float s = amax / 7.0f;
    if (s == 0) s = 1;
    for (int64_t i = 0; i < n; ++i) out[i] = (float)(int)clampd(std::round(w[i] / s), -8.0, 7.0) * s;
    return 0;
  }
  case 15: unsigned_q(15.0f, 15.0, false); return 0;  // Uint4
  case 16:  // FP4: nearest grid value, no scale
    for (int64_t i = 0; i < n; ++i) {
      int best = 0;
      float best_err = std::numeric_limits<float>::max();
      for (int c = 0; c < 16; ++c) {
        const float e = std::fabs(w[i] - kFp4Grid[c]);
        if (e < best_err) {
          best_err = e;
          best = c;
        }
      }
      out[i] = kFp4Grid[best];
    }
    return 0;
  case 17: {  // Int2
    const float s = amax == 0 ? 1.0f : amax;
    for (int64_t i = 0; i < n; ++i) out[i] = (float)(int)clampd(std::round(w[i] / s), -2.0, 1.0) * s;
    return 0;
  }
  case 18: {  // Uint2: ((w-mn)/span) in float, times 3.0 in double
    const float scale = span / 3.0f;
    for (int64_t i = 0; i < n; ++i) {
      const int q = (int)clampd(rnd((double)((w[i] - mn) / span) * 3.0), 0.0, 3.0);
      out[i] = (float)q * scale + mn;
    }
    return 0;
  }
  case 19: {  // Ternary
    const float s = amax == 0 ? 1.0f : amax;
    for (int64_t i = 0; i < n; ++i) {
      const float r = w[i] / s;
      out[i] = r > 0.5f ? s : (r < -0.5f ? -s : 0.0f);
    }
    return 0;
  }
  case 20: {  // Binary
    const float s = amax == 0 ? 1.0f : amax;
    for (int64_t i = 0; i < n; ++i) out[i] = w[i] >= 0 ? s : -s;
    return 0;
  }
  case 27: case 28: signed_nbit(6); return 0;  // FP6 (stored as signed 6-bit), Int6
  case 30: signed_nbit(5); return 0;             // Int5
  case 32: signed_nbit(3); return 0;             // Int3
  case 29: case 31: case 33: {                   // Uint6, Uint5, Uint3
    const int bits = dtype == 29 ? 6 : (dtype == 31 ? 5 : 3);
    const int max_q = (1 << bits) - 1;
    const float scale = span / (float)max_q;
    for (int64_t i = 0; i < n; ++i) {
      const int q = (int)clampd(std::round((w[i] - mn) / span * max_q), 0.0, (double)max_q);
      out[i] = (float)q * scale + mn;
    }
    return 0;
  }
  default:
    return -2;
  }
}

void oracle_fp8_rowscale_encode(const float* w, int64_t rows, int64_t cols, uint8_t* codes,
                                float* scales) {
  for (int64_t r = 0; r < rows; ++r) {
    float s = absmax(w + r * cols, cols) / 448.0f;
    if (s == 0) s = 1;
    scales[r] = s;
    for (int64_t c = 0; c < cols; ++c) codes[r * cols + c] = oracle_e4m3_encode(w[r * cols + c] / s);
  }
}

void oracle_fp8_rowscale_decode(const uint8_t* codes, const float* scales, int64_t rows,
                                int64_t cols, float* out) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c)
      out[r * cols + c] = oracle_e4m3_decode(codes[r * cols + c]) * scales[r];
}

void oracle_nf4_block_encode(const float* w, int64_t n, int32_t block, uint8_t* packed,
                             float* amax) {
  const int64_t nblk = (n + block - 1) / block;
  std::memset(packed, 0, (size_t)((n + 1) / 2));
  for (int64_t j = 0; j < nblk; ++j) {
    const int64_t i0 = j * block, i1 = std::min<int64_t>(n, i0 + block);
    float s = absmax(w + i0, i1 - i0);
    if (s == 0) s = 1;
    amax[j] = s;
    for (int64_t i = i0; i < i1; ++i) {
      const int best = nf4_nearest(w[i] / s);
      if (i % 2 == 0)
        packed[i / 2] = (uint8_t)(best & 0xf);
      else
        packed[i / 2] |= (uint8_t)((best & 0xf) << 4);
    }
  }
}

void oracle_nf4_block_decode(const uint8_t* packed, const float* amax, int64_t n, int32_t block,
                             float* out) {
  for (int64_t i = 0; i < n; ++i) {
    const int code = (i % 2 == 0) ? (packed[i / 2] & 0xf) : (packed[i / 2] >> 4);
    out[i] = kNf4Levels[code] * amax[i / block];
  }
}

} // extern "C"
