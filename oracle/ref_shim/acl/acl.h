// Stand-in for the two CANN fp16 helpers the reference's CPU position code
// calls (aclFloat16ToFloat / aclFloatToFloat16), so that those reference
// source files compile on a host without CANN.  IEEE 754 binary16 conversion
// with round-to-nearest-even, written here from the format's definition.
// TEST INFRASTRUCTURE ONLY (oracle/_ref).
#pragma once

#include <cstdint>
#include <cstring>

typedef uint16_t aclFloat16;

inline float aclFloat16ToFloat(aclFloat16 h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      exp = 113;  // 127 - 15 + 1
      while (!(man & 0x400u)) {
        man <<= 1;
        --exp;
      }
      bits = sign | (exp << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline aclFloat16 aclFloatToFloat16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t absx = x & 0x7FFFFFFFu;
  if (absx >= 0x7F800000u) return (aclFloat16)(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u : 0u));
  if (absx >= 0x477FF000u) return (aclFloat16)(sign | 0x7C00u);  // rounds past 65504
  if (absx < 0x38800000u) {                                      // subnormal half (or zero)
    if (absx < 0x33000000u) return (aclFloat16)sign;
    const uint32_t e = absx >> 23, m = (absx & 0x7FFFFFu) | 0x800000u;
    const int shift = 126 - (int)e;  // 14 .. 24
    uint32_t r = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (r & 1))) ++r;
    return (aclFloat16)(sign | r);
  }
  uint32_t r = ((absx - 0x38000000u) >> 13);
  const uint32_t rem = absx & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1))) ++r;
  return (aclFloat16)(sign | r);
}
