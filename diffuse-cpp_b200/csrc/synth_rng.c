/*
 * synth_rng.c — counter-based Gaussian generator for synthetic benchmark weights
 * (libdmoe_synth.so; not part of the libdiffuse_moe drop-in ABI).
 *
 * Element i of stream (seed, stream) is a deterministic function of (seed, stream, i): pair
 * j = i / 2 draws two 64-bit splitmix64 outputs, maps them to u1 in (0, 1] and u2 in [0, 1),
 * and applies the Box-Muller transform (z0, z1) = sqrt(-2 ln u1) (cos 2 pi u2, sin 2 pi u2).
 * The result does not depend on the thread count, so every machine builds the same weights.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static inline uint16_t f32_to_f16_rne(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
  if (ax < 0x38800000u) {
    float a;
    memcpy(&a, &ax, 4);
    return (uint16_t)(sign | (uint16_t)nearbyintf(a * 16777216.0f));
  }
  const uint32_t e = (ax >> 23) - 112, m = ax & 0x7FFFFFu;
  uint32_t h = (e << 10) | (m >> 13);
  const uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;
  return (uint16_t)(sign | h);
}

static inline void normal_pair(uint64_t key, uint64_t j, float* z0, float* z1) {
  const uint64_t r1 = splitmix64(key + 2 * j);
  const uint64_t r2 = splitmix64(key + 2 * j + 1);
  const float u1 = (float)((r1 >> 40) + 1) * (1.0f / 16777216.0f);
  const float u2 = (float)(r2 >> 40) * (1.0f / 16777216.0f);
  const float r = sqrtf(-2.0f * logf(u1));
  const float a = 6.2831853071795864f * u2;
  *z0 = r * cosf(a);
  *z1 = r * sinf(a);
}

/* out[i] = f16(std * z_i), i in [0, n) */
void dmoe_synth_normal_f16(uint64_t seed, uint64_t stream, int64_t n, float std, uint16_t* out) {
  const uint64_t key = splitmix64(splitmix64(seed) ^ (stream * 0xD1B54A32D192ED03ull));
  const int64_t npairs = (n + 1) / 2;
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < npairs; ++j) {
    float z0, z1;
    normal_pair(key, (uint64_t)j, &z0, &z1);
    out[2 * j] = f32_to_f16_rne(std * z0);
    if (2 * j + 1 < n) out[2 * j + 1] = f32_to_f16_rne(std * z1);
  }
}

/* out[i] = std * z_i as float */
void dmoe_synth_normal_f32(uint64_t seed, uint64_t stream, int64_t n, float std, float* out) {
  const uint64_t key = splitmix64(splitmix64(seed) ^ (stream * 0xD1B54A32D192ED03ull));
  const int64_t npairs = (n + 1) / 2;
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < npairs; ++j) {
    float z0, z1;
    normal_pair(key, (uint64_t)j, &z0, &z1);
    out[2 * j] = std * z0;
    if (2 * j + 1 < n) out[2 * j + 1] = std * z1;
  }
}
