// Narrow-weight encoders shared by the host and the device: one source, so a
// weight quantised on the GPU has exactly the bits the host would give it.
#pragma once

#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define SPARSL_HD __host__ __device__
#else
#define SPARSL_HD
#endif

namespace sparsl {

SPARSL_HD inline uint32_t codec_fbits(float v) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(v);
#else
  uint32_t u;
  memcpy(&u, &v, 4);
  return u;
#endif
}

// IEEE binary16 encoder, round to nearest even; overflow goes to infinity and
// NaN payloads are kept non-zero (the contract of src/half.rs:101-161).  Like
// the reference, magnitudes below 2^-24 (exponent < -24) encode to zero.
SPARSL_HD inline uint16_t encode_f16(float value) {
  const uint32_t x = codec_fbits(value);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t e = (x >> 23) & 0xffu;
  const uint32_t man = x & 0x7fffffu;
  if (e == 0xffu) {
    uint16_t p = (uint16_t)(man >> 13);
    if (man != 0 && p == 0) p = 1;
    return sign | 0x7c00u | p;
  }
  const int ex = (int)e - 127;
  if (ex >= 16) return sign | 0x7c00u;
  if (ex < -24) return sign;
  // Significand with its hidden one; normal and subnormal targets differ only
  // in how many low bits are rounded away.
  const uint32_t sig = man | 0x800000u;
  const uint32_t drop = ex >= -14 ? 13u : 13u + (uint32_t)(-14 - ex);
  uint32_t q = sig >> drop;
  const uint32_t rem = sig & ((1u << drop) - 1u);
  const uint32_t half = 1u << (drop - 1);
  if (rem > half || (rem == half && (q & 1u))) ++q;
  if (ex >= -14) {
    // q carries the hidden one at bit 10, so adding it bumps the exponent
    // field by one; a rounding carry to 0x800 lands on the next binade (or
    // on infinity, 0x7c00) by the same addition.
    const uint32_t h = ((uint32_t)(ex + 14) << 10) + q;
    return sign | (uint16_t)(h >= 0x7c00u ? 0x7c00u : h);
  }
  return sign | (uint16_t)q;  // subnormal; q == 0x400 is the smallest normal
}

// bfloat16 encoder, round to nearest even; NaN keeps its quiet bit
// (src/half.rs:203-214).
SPARSL_HD inline uint16_t encode_bf16(float value) {
  const uint32_t x = codec_fbits(value);
  if (value != value) return (uint16_t)((x >> 16) | 0x40u);
  const uint32_t lsb = (x >> 16) & 1u;
  return (uint16_t)((x + 0x7fffu + lsb) >> 16);
}

}  // namespace sparsl
