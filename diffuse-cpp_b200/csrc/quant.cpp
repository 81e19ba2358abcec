// quant.cpp — host-side GGUF block quantisers (F16, Q8_0, Q4_K) used to build weights.
//
// The reference quantises through ggml (tools/quant_lib.c:16-27 -> ggml_quantize_chunk;
// scheme tools/quantize_streaming.py:112-124 puts MoE experts and the shared expert at Q4_K for
// q4_k_m / q4_k_s and Q8_0 for q8_0). ggml is not available here, so:
//   Q8_0 follows ggml's round-to-nearest rule: d = amax / 127, q = roundf(x / d)
//        (bit-identical to gguf-py's Q8_0.quantize_blocks, checked by the tests);
//   Q4_K is this library's own quantiser of the same super-block format (per sub-block
//        min/max -> 6-bit scale and min against f16 super-block scales), not ggml's search.
// Oracle and kernels consume the same bytes, so the quantiser does not affect parity.
#include <cmath>
#include <cstdint>
#include <cstring>

#include "../../include/diffuse_moe.h"

namespace dmoe {

uint16_t f32_to_f16_bits(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
  if (ax < 0x38800000u) {
    float a;
    std::memcpy(&a, &ax, 4);
    const float r = std::nearbyint(a * 16777216.0f);
    return (uint16_t)(sign | (uint16_t)r);
  }
  const uint32_t e = (ax >> 23) - 112;
  const uint32_t m = ax & 0x7FFFFFu;
  uint32_t h = (e << 10) | (m >> 13);
  const uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;
  return (uint16_t)(sign | h);
}

float f16_bits_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t ex = (h >> 10) & 0x1F;
  const uint32_t man = h & 0x3FF;
  uint32_t bits;
  if (ex == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      const float v = (float)man * (1.0f / 16777216.0f);
      std::memcpy(&bits, &v, 4);
      bits |= sign;
    }
  } else if (ex == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((ex + 112) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

size_t row_size(int32_t type, int64_t k) {
  switch (type) {
    case DMOE_TYPE_F32: return (size_t)k * 4;
    case DMOE_TYPE_F16: return (size_t)k * 2;
    case DMOE_TYPE_Q8_0: return (k % 32) ? 0 : (size_t)(k / 32) * 34;
    case DMOE_TYPE_Q4_K: return (k % 256) ? 0 : (size_t)(k / 256) * 144;
    default: return 0;
  }
}

static void quant_q8_0_row(const float* x, uint8_t* y, int64_t k) {
  for (int64_t b = 0; b < k / 32; ++b) {
    const float* xb = x + b * 32;
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) amax = std::fmax(amax, std::fabs(xb[j]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint8_t* yb = y + b * 34;
    const uint16_t dh = f32_to_f16_bits(d);
    yb[0] = (uint8_t)(dh & 0xFF);
    yb[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < 32; ++j) {
      const float v = xb[j] * id;
      yb[2 + j] = (uint8_t)(int8_t)std::roundf(v);
    }
  }
}

static inline int nearest_int_clamped(float v, int lo, int hi) {
  int q = (int)std::lrintf(v);
  return q < lo ? lo : (q > hi ? hi : q);
}

static void quant_q4_k_row(const float* x, uint8_t* y, int64_t k) {
  for (int64_t b = 0; b < k / 256; ++b) {
    const float* xb = x + b * 256;
    uint8_t* yb = y + b * 144;
    float scale[8], minv[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
      float mn = 0.0f, mx = -INFINITY;
      for (int l = 0; l < 32; ++l) {
        mn = std::fmin(mn, xb[32 * j + l]);
        mx = std::fmax(mx, xb[32 * j + l]);
      }
      if (mx < mn) mx = mn;
      scale[j] = (mx - mn) / 15.0f;
      minv[j] = -mn;  // >= 0: the format subtracts dmin * m
      max_scale = std::fmax(max_scale, scale[j]);
      max_min = std::fmax(max_min, minv[j]);
    }
    const uint16_t dh = f32_to_f16_bits(max_scale / 63.0f);
    const uint16_t mh = f32_to_f16_bits(max_min / 63.0f);
    const float d = f16_bits_to_f32(dh), dmin = f16_bits_to_f32(mh);
    int ls[8], lm[8];
    for (int j = 0; j < 8; ++j) {
      ls[j] = d > 0.0f ? nearest_int_clamped(scale[j] / d, 0, 63) : 0;
      lm[j] = dmin > 0.0f ? nearest_int_clamped(minv[j] / dmin, 0, 63) : 0;
    }
    yb[0] = (uint8_t)(dh & 0xFF);
    yb[1] = (uint8_t)(dh >> 8);
    yb[2] = (uint8_t)(mh & 0xFF);
    yb[3] = (uint8_t)(mh >> 8);
    uint8_t* sc = yb + 4;
    std::memset(sc, 0, 12);
    for (int j = 0; j < 8; ++j) {
      if (j < 4) {
        sc[j] |= (uint8_t)(ls[j] & 63);
        sc[j + 4] |= (uint8_t)(lm[j] & 63);
      } else {
        sc[j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
        sc[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
        sc[j] |= (uint8_t)((lm[j] >> 4) << 6);
      }
    }
    uint8_t q[256];
    for (int j = 0; j < 8; ++j) {
      const float d1 = d * (float)ls[j];
      const float m1 = dmin * (float)lm[j];
      for (int l = 0; l < 32; ++l) {
        const float v = xb[32 * j + l];
        q[32 * j + l] = (uint8_t)(d1 > 0.0f ? nearest_int_clamped((v + m1) / d1, 0, 15) : 0);
      }
    }
    uint8_t* qs = yb + 16;
    for (int g = 0; g < 4; ++g)
      for (int l = 0; l < 32; ++l) qs[32 * g + l] = (uint8_t)(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
  }
}

}  // namespace dmoe

extern "C" size_t dmoe_quantized_size(int32_t type, int64_t nrows, int64_t n_per_row) {
  if (nrows < 0 || n_per_row <= 0) return 0;
  return dmoe::row_size(type, n_per_row) * (size_t)nrows;
}

extern "C" size_t dmoe_quantize(int32_t type, const float* src, void* dst, int64_t nrows, int64_t n_per_row) {
  const size_t rs = dmoe::row_size(type, n_per_row);
  if (!src || !dst || nrows < 0 || rs == 0) return 0;
  uint8_t* out = static_cast<uint8_t*>(dst);
  bool bad = false;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < nrows; ++r) {
    const float* x = src + r * n_per_row;
    uint8_t* y = out + (size_t)r * rs;
    switch (type) {
      case DMOE_TYPE_F32: std::memcpy(y, x, rs); break;
      case DMOE_TYPE_F16:
        for (int64_t i = 0; i < n_per_row; ++i) {
          const uint16_t h = dmoe::f32_to_f16_bits(x[i]);
          y[2 * i] = (uint8_t)(h & 0xFF);
          y[2 * i + 1] = (uint8_t)(h >> 8);
        }
        break;
      case DMOE_TYPE_Q8_0: dmoe::quant_q8_0_row(x, y, n_per_row); break;
      case DMOE_TYPE_Q4_K: dmoe::quant_q4_k_row(x, y, n_per_row); break;
      default: bad = true; break;
    }
  }
  return bad ? 0 : rs * (size_t)nrows;
}
