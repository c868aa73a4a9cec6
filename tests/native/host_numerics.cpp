// Native host checks of the kernels' numeric helpers (csrc/numerics.cuh), compiled with a plain
// C++ compiler: the same functions the sm_100a kernels run, checked here exhaustively or on
// large random samples against independent reference decodings. Exit code 0 = all checks pass.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>

#include "numerics.cuh"

using namespace qb;

static int failures = 0;
#define CHECK(cond, ...)                  \
  do {                                    \
    if (!(cond)) {                        \
      if (failures < 20) {                \
        std::printf("FAIL: " __VA_ARGS__); \
        std::printf("\n");                \
      }                                   \
      ++failures;                         \
    }                                     \
  } while (0)

// f16 bit pattern -> float, from the IEEE binary16 definition (subnormals included).
static float f16_value(uint32_t h) {
  const int s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023;
  float v = e == 0 ? std::ldexp((float)m, -24) : std::ldexp(1.f + m / 1024.f, e - 15);
  return s ? -v : v;
}

// OCP e2m1: 0, 0.5, 1, 1.5, 2, 3, 4, 6 and negatives.
static float e2m1_value(int c) {
  static const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  return (c & 8) ? -mag[c & 7] : mag[c & 7];
}

// OCP e4m3 (bias 7, subnormals m x 2^-9; 0x7F / 0xFF are NaN).
static float e4m3_value(uint8_t c) {
  const int s = c >> 7, e = (c >> 3) & 15, m = c & 7;
  float v = e == 0 ? std::ldexp((float)m, -9) : std::ldexp(1.f + m / 8.f, e - 7);
  return s ? -v : v;
}

static void check_e2m1_placement() {
  // every code in every one of the 8 positions, plus random words
  std::mt19937 rng(1);
  for (int trial = 0; trial < 200000; ++trial) {
    uint32_t w = trial < 128 ? (uint32_t)((trial % 16) << (4 * (trial / 16))) : rng();
    uint32_t o[4];
    e2m1x8_placed(w, o);
    for (int j = 0; j < 8; ++j) {
      const int code = (w >> (4 * j)) & 15;
      const uint32_t half = (o[j / 2] >> (16 * (j % 2))) & 0xFFFF;
      const float got = f16_value(half) * 16384.f;  // placed value = code value * 2^-14
      CHECK(got == e2m1_value(code) || (code == 8 && got == 0.f), "e2m1 word %08x code %d pos %d: %g vs %g", w,
            code, j, got, e2m1_value(code));
    }
  }
}

static float bf16_round(float x) {  // round-to-nearest-even to 8 significant bits
  uint32_t u = f32_bits(x);
  u += 0x7FFF + ((u >> 16) & 1);
  return bits_f32(u & 0xFFFF0000u);
}

static void check_mx_split() {
  std::mt19937 rng(2);
  std::uniform_real_distribution<float> uni(-1.f, 1.f);
  std::uniform_int_distribution<int> ex(-40, 20);
  for (int blk = 0; blk < 200000; ++blk) {
    float x[32];
    const int e0 = ex(rng);
    const int spread = blk % 4 == 0 ? 20 : 10;  // some blocks span more than 2^14
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) {
      x[i] = bf16_round(std::ldexp(uni(rng), e0 - (int)(rng() % spread)));
      if (rng() % 16 == 0) x[i] = 0.f;
      amax = std::fmax(amax, std::fabs(x[i]));
    }
    const int E = mx_block_exponent(f32_bits(amax));
    for (int i = 0; i < 32; ++i) {
      uint8_t hi, lo;
      mx_split(x[i], E, hi, lo);
      CHECK((hi & 0x7F) != 0x7F && (lo & 0x7F) != 0x7F, "NaN code for %g", x[i]);
      const double rec = std::ldexp((double)e4m3_value(hi), E) + std::ldexp((double)e4m3_value(lo), E - 4);
      // exact whenever hi is a normal e4m3 (|x| >= 2^(E-6)), which every |x| >= 2^-13 amax is
      if (std::fabs(x[i]) >= std::ldexp(1.0f, E - 6)) {
        CHECK(rec == (double)x[i], "split not exact: x=%.9g amax=%.9g E=%d rec=%.9g", x[i], amax, E, rec);
      } else {
        CHECK(std::fabs(x[i]) < std::ldexp(amax, -13), "exactness bound: x=%.9g amax=%.9g", x[i], amax);
        CHECK(std::fabs(rec - x[i]) <= std::ldexp((double)amax, -20), "split error too large: x=%.9g amax=%.9g",
              x[i], amax);
      }
    }
  }
}

static void check_chunk_layout() {
  int seen[512] = {0};
  for (int r = 0; r < 128; ++r)
    for (int j = 0; j < 4; ++j) {
      const int o = mx_chunk_offset(r, j);
      CHECK(o >= 0 && o < 512, "offset out of range");
      seen[o]++;
      // line r % 32 holds rows r % 32 + 32 c, c = 0..3, four scales each
      CHECK(o / 16 == r % 32 && (o % 16) / 4 == r / 32 && o % 4 == j, "layout r=%d j=%d -> %d", r, j, o);
    }
  for (int o = 0; o < 512; ++o) CHECK(seen[o] == 1, "offset %d hit %d times", o, seen[o]);
}

static void check_byte_perm() {
  // the zero-operand selector and sign replication behave as the kernels assume
  CHECK(byte_perm(0x44332211u, 0x88776655u, 0x3210) == 0x44332211u, "identity");
  CHECK(byte_perm(0x44332211u, 0x88776655u, 0x7654) == 0x88776655u, "upper");
  CHECK(byte_perm(0x44332211u, 0u, 0x1404) == 0x22001100u, "spread");
  CHECK(byte_perm(0x80u, 0u, 0x0008) == 0x808080FFu, "sign replicate");
}

int main() {
  check_byte_perm();
  check_e2m1_placement();
  check_mx_split();
  check_chunk_layout();
  std::printf("%s (%d failures)\n", failures ? "FAILED" : "ok", failures);
  return failures ? 1 : 0;
}
