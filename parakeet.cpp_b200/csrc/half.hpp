// Host-side f16 / bf16 <-> f32 conversion (IEEE 754 binary16 and bfloat16,
// round to nearest even), used when weights are re-packed at load.
#pragma once
#include <cstdint>
#include <cstring>

namespace pkc {

inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t ex = (h >> 10) & 0x1f;
  uint32_t mant = h & 0x3ff;
  uint32_t bits;
  if (ex == 0) {
    if (mant == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      int e = -1;
      do { mant <<= 1; ++e; } while (!(mant & 0x400));
      mant &= 0x3ff;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
    }
  } else if (ex == 31) {
    bits = sign | 0x7f800000u | (mant << 13);
  } else {
    bits = sign | ((ex + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline uint16_t f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000;
  const uint32_t ex = (x >> 23) & 0xff;
  uint32_t mant = x & 0x7fffff;
  if (ex == 0xff) return (uint16_t)(sign | 0x7c00 | (mant ? 0x200 : 0));
  const int e = (int)ex - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    mant |= 0x800000;
    const int shift = 14 - e;
    uint32_t hm = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1), halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (hm & 1))) ++hm;
    return (uint16_t)(sign | hm);
  }
  uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
  const uint32_t rem = mant & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) ++h;  // carry into the exponent is correct
  return (uint16_t)h;
}

inline float bf16_to_f32(uint16_t h) {
  const uint32_t bits = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline uint16_t f32_to_bf16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  if ((x & 0x7fffffff) > 0x7f800000) return (uint16_t)((x >> 16) | 0x40);  // NaN stays NaN
  x += 0x7fff + ((x >> 16) & 1);
  return (uint16_t)(x >> 16);
}

}  // namespace pkc
