// IEEE binary16 / bfloat16 <-> binary32 conversions for the CPU oracle.
// Test infrastructure only: the product path never includes this file.
// Round-to-nearest-even, matching GLSL float16_t() and CUDA __float2half_rn.
#pragma once
#include <cstdint>
#include <cmath>
#include <cstring>

namespace oracle {

inline float bits_to_f32(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline uint32_t f32_to_bits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }

inline float h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ffu;
  if (exp == 0) {
    if (man == 0) return bits_to_f32(sign);
    // subnormal: value = man * 2^-24
    float v = (float)man * (1.0f / 16777216.0f);
    return sign ? -v : v;
  }
  if (exp == 31) return bits_to_f32(sign | 0x7f800000u | (man << 13));
  return bits_to_f32(sign | ((exp + 112) << 23) | (man << 13));
}

inline uint16_t f2h(float f) {
  uint32_t x = f32_to_bits(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) {  // inf or nan
    return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  }
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to inf
  if (ax < 0x38800000u) {  // below smallest normal half (2^-14): subnormal or zero
    // value / 2^-24 rounded to nearest even integer
    float v = bits_to_f32(ax) * 16777216.0f;  // exact scaling by 2^24
    // round-half-even of v (v < 1024)
    float r = v + 8388608.0f - 8388608.0f;   // uses FPU RNE (default mode)
    return (uint16_t)(sign | (uint32_t)r);
  }
  uint32_t exp = (ax >> 23) - 112;
  uint32_t man = ax & 0x7fffffu;
  uint32_t h = (exp << 10) | (man >> 13);
  uint32_t rem = man & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;  // carry may bump exponent: correct
  return (uint16_t)(sign | h);
}

inline float bf2f(uint16_t b) { return bits_to_f32((uint32_t)b << 16); }

inline uint16_t f2bf(float f) {
  uint32_t x = f32_to_bits(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
  uint32_t lsb = (x >> 16) & 1u;
  x += 0x7fffu + lsb;
  return (uint16_t)(x >> 16);
}

inline float round_h(float f) { return h2f(f2h(f)); }

}  // namespace oracle

namespace oracle {
// The shaders' exp()/log() have implementation-defined precision (GLSL allows
// several ulps), so the decode-path restatement fixes them to one definition
// a GPU can reproduce exactly: evaluate in double precision and round once to
// float. (The chunk rule keeps std::exp on float: it restates the reference's
// own C++ code, src/runtime/deltanet_chunk.cpp, bit for bit.)
inline float exp_d(float x) { return (float)std::exp((double)x); }
inline float log_d(float x) { return (float)std::log((double)x); }
}  // namespace oracle
