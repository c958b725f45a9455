// Host-side IEEE binary16 conversions used for weight packing and host IO.
//
// HalfToFloat is exact. FloatToHalfRNE rounds to nearest-even with gradual underflow
// (subnormal halves), saturating to +/-inf on overflow and keeping NaN a (quiet) NaN:
// the semantics of the reference engine's FloatToHalfBitsRNE
// (src/vapoursynth/hip_engine.cc:1190-1232). FloatToHalfFTZ is the load-time
// converter's variant that flushes every result below the smallest normal half to a
// signed zero and maps NaN to inf (src/vapoursynth/convert_float_to_float16.cpp:165-186).
#pragma once

#include <cstdint>
#include <cstring>

namespace ah {

inline float HalfToFloat(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  const int exp = (h >> 10) & 0x1F;
  uint32_t mant = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (mant << 13);
  } else if (exp != 0) {
    bits = sign | (static_cast<uint32_t>(exp + 112) << 23) | (mant << 13);
  } else if (mant == 0) {
    bits = sign;
  } else {
    // subnormal: value = mant * 2^-24; renormalise
    int e = 113;  // exponent of 2^-14 in fp32 bias terms, decremented while shifting
    while ((mant & 0x400u) == 0) {
      mant <<= 1;
      --e;
    }
    bits = sign | (static_cast<uint32_t>(e) << 23) | ((mant & 0x3FFu) << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline uint16_t FloatToHalfRNE(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint16_t sign = static_cast<uint16_t>((x >> 16) & 0x8000u);
  const uint32_t absx = x & 0x7FFFFFFFu;
  if (absx >= 0x7F800000u) {  // inf or NaN
    return static_cast<uint16_t>(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u : 0u));
  }
  if (absx >= 0x477FF000u) {  // rounds to >= 65520 -> inf
    return static_cast<uint16_t>(sign | 0x7C00u);
  }
  if (absx < 0x38800000u) {  // below the smallest normal half (2^-14): subnormal or zero
    // value / 2^-24 rounded to nearest-even, computed exactly on the integer significand
    const int e = static_cast<int>(absx >> 23);  // biased fp32 exponent
    if (e < 102) return sign;                    // < 2^-25: rounds to zero
    const uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
    const int shift = 126 - e;  // bits to drop so the result is in units of 2^-24
    uint32_t q = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return static_cast<uint16_t>(sign | q);
  }
  // normal range: rebias exponent and round the 13 dropped significand bits
  uint32_t r = absx - 0x38000000u;  // exponent bias 127 -> 15 (shifted into place below)
  const uint32_t low = r & 0x1FFFu;
  r >>= 13;
  if (low > 0x1000u || (low == 0x1000u && (r & 1u))) ++r;  // may carry into the exponent
  return static_cast<uint16_t>(sign | r);
}

inline uint16_t FloatToHalfFTZ(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint16_t sign = static_cast<uint16_t>((x >> 16) & 0x8000u);
  const uint32_t e = x & 0x7F800000u;
  if (e >= 0x47800000u) return static_cast<uint16_t>(sign | 0x7C00u);  // overflow, inf, NaN -> inf
  if (e <= 0x38000000u) return sign;                                  // below 2^-14 -> zero
  uint32_t mant = x & 0x7FFFFFu;
  const uint32_t hexp = (e - 0x38000000u) >> 13;
  // round half to even on the 13 dropped bits; a carry out of the mantissa bumps the exponent
  if ((mant & 0x3FFFu) != 0x1000u) mant += 0x1000u;
  return static_cast<uint16_t>(sign + hexp + (mant >> 13));
}

}  // namespace ah
