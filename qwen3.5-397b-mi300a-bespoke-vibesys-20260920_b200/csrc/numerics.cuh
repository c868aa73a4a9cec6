// Bit-exact numeric helpers shared by the kernels and the native host tests.
//
// Every function here is `__host__ __device__` and free of device-only intrinsics when compiled
// for the host, so `tests/native/host_numerics.cpp` (built with a plain C++ compiler) checks the
// same code the kernels run: the e2m1 code placement of the f16-decode MoE path, the truncating
// e4m3 split of the block-scaled path, and the scale-chunk layout of the block-scaled MMA.
#pragma once

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define QB_HD __host__ __device__ __forceinline__
#else
#define QB_HD inline
#endif

namespace qb {

QB_HD uint32_t f32_bits(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
#endif
}

QB_HD float bits_f32(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

// PRMT: byte i of the result = byte (s >> 4i) & 7 of the 8-byte value {y:x}; selector bit 3 set
// replicates that byte's sign bit instead.
QB_HD uint32_t byte_perm(uint32_t x, uint32_t y, uint32_t s) {
#if defined(__CUDA_ARCH__)
  return __byte_perm(x, y, s);
#else
  const uint64_t v = ((uint64_t)y << 32) | x;
  uint32_t r = 0;
  for (int i = 0; i < 4; ++i) {
    const uint32_t sel = (s >> (4 * i)) & 15;
    uint32_t b = (uint32_t)(v >> (8 * (sel & 7))) & 0xFF;
    if (sel & 8) b = (b & 0x80) ? 0xFF : 0x00;
    r |= b << (8 * i);
  }
  return r;
#endif
}

// Eight e2m1 codes (code j in bits 4j..4j+3) -> four f16x2 words. A code [s e1 e0 m] placed at f16
// bits 15 / 11 / 10 / 9 is exactly its value times 2^-14 (e = 0 lands in the f16 subnormal range,
// e > 0 in the normal range, both scaled by the same 2^-14); the caller multiplies by the power of
// two 2^(14 + block exponent).
QB_HD void e2m1x8_placed(uint32_t w, uint32_t* o) {
  // even codes: e/m bits to byte bits 1..3, sign to bit 7; odd codes likewise from the high nibble
  const uint32_t ev = ((w << 1) & 0x0E0E0E0Eu) | ((w << 4) & 0x80808080u);
  const uint32_t od = ((w >> 3) & 0x0E0E0E0Eu) | (w & 0x80808080u);
  // interleave (even, odd) byte pairs, then spread each pair into the high bytes of two halves
  // (selector 4 = a byte of the zero operand)
  const uint32_t p01 = byte_perm(ev, od, 0x5140), p23 = byte_perm(ev, od, 0x7362);
  o[0] = byte_perm(p01, 0, 0x1404);
  o[1] = byte_perm(p01, 0, 0x3424);
  o[2] = byte_perm(p23, 0, 0x1404);
  o[3] = byte_perm(p23, 0, 0x3424);
}

// |v| (< 256) -> (e4m3 code, its value), truncated toward zero.
QB_HD uint32_t e4m3_trunc(float av, float& val) {
  const uint32_t b = f32_bits(av);
  if (b >= 0x3C800000u) {  // >= 2^-6: normal e4m3, keep 3 mantissa bits
    val = bits_f32(b & 0xFFF00000u);
    return ((((b >> 23) & 0xFF) - 127 + 7) << 3) | ((b >> 20) & 7);
  }
  const uint32_t m = (uint32_t)(av * 512.f);  // subnormal: m x 2^-9, m < 8
  val = (float)m * (1.f / 512.f);
  return m;
}

// Block exponent of a 32-element block whose largest magnitude has bits `amax_bits`:
// amax / 2^E in [128, 256); at least -123 so that the lo term's scale E - 4 stays a valid e8m0.
QB_HD int mx_block_exponent(uint32_t amax_bits) {
  int E = amax_bits ? (int)(amax_bits >> 23) - 127 - 7 : -127;
  return E < -123 ? -123 : E;
}

// Split one value of a block with exponent E into (hi code, lo code) with sign:
// x = 2^E * hi + 2^(E-4) * lo.
QB_HD void mx_split(float v, int E, uint8_t& hi, uint8_t& lo) {
  const float inv = bits_f32((uint32_t)(127 - E) << 23);  // 2^-E, exact
  const float xs = (v < 0.f ? -v : v) * inv;
  float hv, lv;
  const uint32_t ch = e4m3_trunc(xs, hv);
  const uint32_t cl = e4m3_trunc((xs - hv) * 16.f, lv);
  const uint32_t sg = v < 0.f ? 0x80u : 0u;
  hi = (uint8_t)(ch | (ch ? sg : 0u));
  lo = (uint8_t)(cl | (cl ? sg : 0u));
}

// Byte offset inside one 512-byte scale chunk (128 rows x 4 K-blocks) of row r and K-block j:
// line r % 32 (16 bytes) holds the 4 scales of rows r%32, r%32+32, r%32+64, r%32+96.
QB_HD int mx_chunk_offset(int r, int j) { return (r % 32) * 16 + (r / 32) * 4 + j; }

}  // namespace qb
