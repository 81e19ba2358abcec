/*
 * dmoe_oracle_ggml.c — ggml-faithful CPU restatement of the MoE experts of diffuse-cpp
 * (src/diffuse-moe-graph.cpp:264-286). TEST INFRASTRUCTURE ONLY: the checker of what the
 * reference's ggml CPU backend would output, and the timed CPU baseline. Never the product.
 *
 * The reference computes the experts with ggml_mul_mat_id on the quantised expert tensors
 * (:265-269). On the CPU backend ggml then keeps the weights in their GGUF blocks and converts
 * each activation row to the weight type's "vec-dot type" before the dot products:
 *   Q4_K weights -> activations as Q8_K  (256-value blocks: float d, 256 int8, 16 int16 sums)
 *   Q8_0 weights -> activations as Q8_0  (32-value blocks: fp16 d, 32 int8)
 *   F16  weights -> activations as F16
 * and every weight row . activation row product is an integer dot product per block, scaled
 * by the two block scales in float. This file restates that:
 *   x rows rounded to the vec-dot type; g = W_g x, u = W_u x (quantised dots); h = silu(g) u in
 *   f32 (:266-268); h rows rounded to the down matrix's vec-dot type; y = W_d h (:269); y * w
 *   (:270); slot sum in slot order with f32 adds (:273-278); the shared expert on weights cast
 *   to F32 (ensure_f32_moe, :8-12, :280-285), f32 dot products, added last.
 * Rounding rules of the activation formats (ggml, an un-vendored submodule, commit unpinned;
 * restated from its published reference quantisers):
 *   Q8_K: per 256 values, max = the value of largest magnitude, iscale = -127 / max,
 *         q = min(127, round-half-even(iscale x)), d = 1 / iscale, bsums = sums of 16 q's.
 *   Q8_0: per 32 values, d = amax / 127, q = round-half-away(x / d), d stored as fp16.
 *   F16:  round to nearest even.
 * The integer parts of every dot product are exact; only the float combination of the block
 * scales (and the summation order inside the SIMD lanes) may differ from a given ggml build.
 *
 * Speed: the dot products are AVX2 integer kernels (unsigned x signed byte multiply-adds into
 * 16-bit pairs, then 32-bit sums with the sub-block scales folded into the second step), the
 * work split over OpenMP threads by (expert, 16-row chunk); scalar versions of each kernel
 * (dmoe_oracle_ggml_dot) are kept for the unit test that checks the SIMD ones.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "dmoe_oracle.h"
#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__AVX2__) && defined(__FMA__) && defined(__F16C__)
#include <immintrin.h>
#define ORC_SIMD 1
#else
#define ORC_SIMD 0
#endif

#define QK_K 256
#define QK8_0 32

/* Q8_K activation block (ggml block_q8_K layout: float d; int8 qs[256]; int16 bsums[16]) */
typedef struct {
  float d;
  int8_t qs[QK_K];
  int16_t bsums[QK_K / 16];
} q8k_blk;

/* Q8_0 activation block, kept with the scale already widened (fp16 value as float) */
typedef struct {
  float d;
  int8_t qs[QK8_0];
} q80_blk;

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ------------------------------------------------------------------------------------------ */
/* activation rounding                                                                          */
/* ------------------------------------------------------------------------------------------ */
static void quant_row_q8k(const float* x, int64_t k, q8k_blk* y) {
  for (int64_t b = 0; b < k / QK_K; ++b) {
    const float* xb = x + b * QK_K;
    float amax = 0.0f, mx = 0.0f;
    for (int j = 0; j < QK_K; ++j) {
      const float ax = fabsf(xb[j]);
      if (ax > amax) {
        amax = ax;
        mx = xb[j];
      }
    }
    if (amax == 0.0f) {
      memset(&y[b], 0, sizeof(q8k_blk));
      continue;
    }
    const float iscale = -127.0f / mx;
    for (int j = 0; j < QK_K; ++j) {
      const long v = lrintf(iscale * xb[j]); /* round half to even */
      y[b].qs[j] = (int8_t)(v > 127 ? 127 : v);
    }
    for (int j = 0; j < QK_K / 16; ++j) {
      int s = 0;
      for (int i = 0; i < 16; ++i) s += y[b].qs[16 * j + i];
      y[b].bsums[j] = (int16_t)s;
    }
    y[b].d = 1.0f / iscale;
  }
}

static void quant_row_q80(const float* x, int64_t k, q80_blk* y) {
  for (int64_t b = 0; b < k / QK8_0; ++b) {
    const float* xb = x + b * QK8_0;
    float amax = 0.0f;
    for (int j = 0; j < QK8_0; ++j) amax = fmaxf(amax, fabsf(xb[j]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    for (int j = 0; j < QK8_0; ++j) y[b].qs[j] = (int8_t)roundf(xb[j] * id);
    y[b].d = dmoe_oracle_f16_to_f32(dmoe_oracle_f32_to_f16(d));
  }
}

static void quant_row_f16(const float* x, int64_t k, uint16_t* y) {
  for (int64_t j = 0; j < k; ++j) y[j] = dmoe_oracle_f32_to_f16(x[j]);
}

/* bytes of one activation row in the vec-dot type of weight type `t` */
static size_t act_row_bytes(int t, int64_t k) {
  switch (t) {
    case ORC_Q4_K: return (size_t)(k / QK_K) * sizeof(q8k_blk);
    case ORC_Q8_0: return (size_t)(k / QK8_0) * sizeof(q80_blk);
    case ORC_F16: return (size_t)k * 2;
    default: return 0;
  }
}

static void quant_act(int t, const float* x, int64_t k, void* y) {
  if (t == ORC_Q4_K) quant_row_q8k(x, k, (q8k_blk*)y);
  else if (t == ORC_Q8_0) quant_row_q80(x, k, (q80_blk*)y);
  else quant_row_f16(x, k, (uint16_t*)y);
}

/* ------------------------------------------------------------------------------------------ */
/* dot products: weight row (GGUF blocks) . activation row (vec-dot type)                      */
/* ------------------------------------------------------------------------------------------ */
/* Q4_K sub-block scales and mins of one super-block (6-bit packed, format of block_q4_K) */
static inline void q4k_unpack(const uint8_t* q, int16_t* sc, int16_t* m) {
  for (int j = 0; j < 4; ++j) {
    sc[j] = q[j] & 63;
    m[j] = q[j + 4] & 63;
  }
  for (int j = 4; j < 8; ++j) {
    sc[j] = (int16_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
    m[j] = (int16_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

/* per super-block combination shared by both versions: exact integer sums, then
 * sum += d_w d_y isum; sum -= dmin_w d_y msum */
static inline float q4k_combine(float sumf, const uint8_t* blk, const q8k_blk* y, int32_t isum, int32_t msum) {
  const float d = dmoe_oracle_f16_to_f32(rd16(blk)) * y->d;
  const float dmin = dmoe_oracle_f16_to_f32(rd16(blk + 2)) * y->d;
  sumf += d * (float)isum;
  sumf -= dmin * (float)msum;
  return sumf;
}

static float dot_q4k_scalar(const uint8_t* row, const q8k_blk* y, int64_t nsb) {
  float sumf = 0.0f;
  for (int64_t b = 0; b < nsb; ++b) {
    const uint8_t* blk = row + b * 144;
    int16_t sc[8], m[8];
    q4k_unpack(blk + 4, sc, m);
    const uint8_t* qs = blk + 16;
    int32_t isum = 0, msum = 0;
    for (int g = 0; g < 4; ++g) {
      int32_t lo = 0, hi = 0;
      for (int l = 0; l < 32; ++l) {
        lo += (qs[32 * g + l] & 0xF) * y[b].qs[64 * g + l];
        hi += (qs[32 * g + l] >> 4) * y[b].qs[64 * g + 32 + l];
      }
      isum += sc[2 * g] * lo + sc[2 * g + 1] * hi;
    }
    for (int j = 0; j < 8; ++j) msum += m[j] * (y[b].bsums[2 * j] + y[b].bsums[2 * j + 1]);
    sumf = q4k_combine(sumf, blk, &y[b], isum, msum);
  }
  return sumf;
}

static float dot_q80_scalar(const uint8_t* row, const q80_blk* y, int64_t nb) {
  float sumf = 0.0f;
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = row + b * 34;
    int32_t s = 0;
    for (int j = 0; j < QK8_0; ++j) s += (int8_t)blk[2 + j] * y[b].qs[j];
    sumf += (float)s * (dmoe_oracle_f16_to_f32(rd16(blk)) * y[b].d);
  }
  return sumf;
}

static float dot_f16_scalar(const uint8_t* row, const uint16_t* y, int64_t k) {
  float s = 0.0f;
  for (int64_t j = 0; j < k; ++j) s += dmoe_oracle_f16_to_f32(rd16(row + 2 * j)) * dmoe_oracle_f16_to_f32(y[j]);
  return s;
}

#if ORC_SIMD
static inline int32_t hsum_i32(__m256i v) {
  __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
  s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
  s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
  return _mm_cvtsi128_si32(s);
}
static inline float hsum_f32(__m256 v) {
  __m128 s = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  s = _mm_add_ps(s, _mm_movehl_ps(s, s));
  s = _mm_add_ss(s, _mm_movehdup_ps(s));
  return _mm_cvtss_f32(s);
}

/* sc/m: the row's unpacked scales and mins, 8 + 8 per super-block */
static float dot_q4k_simd(const uint8_t* row, const int16_t* scm, const q8k_blk* y, int64_t nsb) {
  const __m256i m4 = _mm256_set1_epi8(0x0F);
  float sumf = 0.0f;
  for (int64_t b = 0; b < nsb; ++b) {
    const uint8_t* blk = row + b * 144;
    const uint8_t* qs = blk + 16;
    const int16_t* sc = scm + 16 * b;
    const int16_t* m = sc + 8;
    __m256i acc = _mm256_setzero_si256();
    for (int g = 0; g < 4; ++g) {
      const __m256i q4 = _mm256_loadu_si256((const __m256i*)(qs + 32 * g));
      const __m256i lo = _mm256_and_si256(q4, m4);
      const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(q4, 4), m4);
      const __m256i yl = _mm256_loadu_si256((const __m256i*)(y[b].qs + 64 * g));
      const __m256i yh = _mm256_loadu_si256((const __m256i*)(y[b].qs + 64 * g + 32));
      const __m256i pl = _mm256_maddubs_epi16(lo, yl); /* <= 2 * 15 * 127: no saturation */
      const __m256i ph = _mm256_maddubs_epi16(hi, yh);
      acc = _mm256_add_epi32(acc, _mm256_madd_epi16(pl, _mm256_set1_epi16(sc[2 * g])));
      acc = _mm256_add_epi32(acc, _mm256_madd_epi16(ph, _mm256_set1_epi16(sc[2 * g + 1])));
    }
    /* mins: sum_j m_j (bsum_2j + bsum_2j+1) */
    const __m128i bs = _mm_hadd_epi16(_mm_loadu_si128((const __m128i*)y[b].bsums),
                                      _mm_loadu_si128((const __m128i*)(y[b].bsums + 8)));
    const __m128i mm = _mm_madd_epi16(bs, _mm_loadu_si128((const __m128i*)m));
    __m128i ms = _mm_add_epi32(mm, _mm_shuffle_epi32(mm, 0x4E));
    ms = _mm_add_epi32(ms, _mm_shuffle_epi32(ms, 0xB1));
    sumf = q4k_combine(sumf, blk, &y[b], hsum_i32(acc), _mm_cvtsi128_si32(ms));
  }
  return sumf;
}

static float dot_q80_simd(const uint8_t* row, const q80_blk* y, int64_t nb) {
  __m256 acc = _mm256_setzero_ps();
  const __m256i ones = _mm256_set1_epi16(1);
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = row + b * 34;
    const __m256i w = _mm256_loadu_si256((const __m256i*)(blk + 2));
    const __m256i x = _mm256_loadu_si256((const __m256i*)y[b].qs);
    const __m256i p = _mm256_maddubs_epi16(_mm256_sign_epi8(w, w), _mm256_sign_epi8(x, w));
    const __m256i s = _mm256_madd_epi16(p, ones);
    const __m256 d = _mm256_set1_ps(dmoe_oracle_f16_to_f32(rd16(blk)) * y[b].d);
    acc = _mm256_fmadd_ps(d, _mm256_cvtepi32_ps(s), acc);
  }
  return hsum_f32(acc);
}

static float dot_f16_simd(const uint8_t* row, const uint16_t* y, int64_t k) {
  __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
  int64_t j = 0;
  for (; j + 16 <= k; j += 16) {
    a0 = _mm256_fmadd_ps(_mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(row + 2 * j))),
                         _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(y + j))), a0);
    a1 = _mm256_fmadd_ps(_mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(row + 2 * j + 16))),
                         _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(y + j + 8))), a1);
  }
  float s = hsum_f32(_mm256_add_ps(a0, a1));
  for (; j < k; ++j) s += dmoe_oracle_f16_to_f32(rd16(row + 2 * j)) * dmoe_oracle_f16_to_f32(y[j]);
  return s;
}

static float dot_f32_simd(const float* a, const float* b, int64_t k) {
  __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps(), a2 = _mm256_setzero_ps(), a3 = _mm256_setzero_ps();
  int64_t j = 0;
  for (; j + 32 <= k; j += 32) {
    a0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + j), _mm256_loadu_ps(b + j), a0);
    a1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + j + 8), _mm256_loadu_ps(b + j + 8), a1);
    a2 = _mm256_fmadd_ps(_mm256_loadu_ps(a + j + 16), _mm256_loadu_ps(b + j + 16), a2);
    a3 = _mm256_fmadd_ps(_mm256_loadu_ps(a + j + 24), _mm256_loadu_ps(b + j + 24), a3);
  }
  float s = hsum_f32(_mm256_add_ps(_mm256_add_ps(a0, a1), _mm256_add_ps(a2, a3)));
  for (; j < k; ++j) s += a[j] * b[j];
  return s;
}
#endif

static float dot_f32(const float* a, const float* b, int64_t k) {
#if ORC_SIMD
  return dot_f32_simd(a, b, k);
#else
  float s = 0.0f;
  for (int64_t j = 0; j < k; ++j) s += a[j] * b[j];
  return s;
#endif
}

/* one weight row . one activation row; scm: unpacked Q4_K scales of the row (or NULL) */
static inline float dot_row(int t, const uint8_t* row, const int16_t* scm, const void* act, int64_t k) {
#if ORC_SIMD
  if (t == ORC_Q4_K) return dot_q4k_simd(row, scm, (const q8k_blk*)act, k / QK_K);
  if (t == ORC_Q8_0) return dot_q80_simd(row, (const q80_blk*)act, k / QK8_0);
  return dot_f16_simd(row, (const uint16_t*)act, k);
#else
  (void)scm;
  if (t == ORC_Q4_K) return dot_q4k_scalar(row, (const q8k_blk*)act, k / QK_K);
  if (t == ORC_Q8_0) return dot_q80_scalar(row, (const q80_blk*)act, k / QK8_0);
  return dot_f16_scalar(row, (const uint16_t*)act, k);
#endif
}

static void unpack_scales(int t, const uint8_t* row, int64_t k, int16_t* scm) {
  if (t != ORC_Q4_K) return;
  for (int64_t b = 0; b < k / QK_K; ++b) q4k_unpack(row + b * 144 + 4, scm + 16 * b, scm + 16 * b + 8);
}

/* Unit-test hook: dot of nrows weight rows with one float activation row (rounded to the
 * vec-dot type here), by the SIMD kernel (simd = 1) or the scalar one (0). Returns 0 on success. */
int dmoe_oracle_ggml_dot(int type, const void* w, int64_t nrows, int64_t k, const float* x, float* out, int simd) {
  const size_t rs = dmoe_oracle_row_size(type, k);
  const size_t ab = act_row_bytes(type, k);
  if (!rs || !ab) return -1;
  void* act = malloc(ab);
  quant_act(type, x, k, act);
  int16_t* scm = (int16_t*)malloc(sizeof(int16_t) * (size_t)(16 * (k / QK_K) + 16));
  for (int64_t r = 0; r < nrows; ++r) {
    const uint8_t* row = (const uint8_t*)w + r * rs;
    if (simd && ORC_SIMD) {
      unpack_scales(type, row, k, scm);
      out[r] = dot_row(type, row, scm, act, k);
    } else if (type == ORC_Q4_K) {
      out[r] = dot_q4k_scalar(row, (const q8k_blk*)act, k / QK_K);
    } else if (type == ORC_Q8_0) {
      out[r] = dot_q80_scalar(row, (const q80_blk*)act, k / QK8_0);
    } else {
      out[r] = dot_f16_scalar(row, (const uint16_t*)act, k);
    }
  }
  free(scm);
  free(act);
  return 0;
}

/* Activation rounding hook for the unit tests: x [k] -> the dequantised vec-dot-type values. */
int dmoe_oracle_ggml_round_act(int type, const float* x, int64_t k, float* out) {
  const size_t ab = act_row_bytes(type, k);
  if (!ab) return -1;
  void* act = malloc(ab);
  quant_act(type, x, k, act);
  if (type == ORC_Q4_K) {
    const q8k_blk* y = (const q8k_blk*)act;
    for (int64_t j = 0; j < k; ++j) out[j] = y[j / QK_K].d * (float)y[j / QK_K].qs[j % QK_K];
  } else if (type == ORC_Q8_0) {
    const q80_blk* y = (const q80_blk*)act;
    for (int64_t j = 0; j < k; ++j) out[j] = y[j / QK8_0].d * (float)y[j / QK8_0].qs[j % QK8_0];
  } else {
    const uint16_t* y = (const uint16_t*)act;
    for (int64_t j = 0; j < k; ++j) out[j] = dmoe_oracle_f16_to_f32(y[j]);
  }
  free(act);
  return 0;
}

static inline float silu_f(float g) { return g / (1.0f + expf(-g)); }

#define ORC_RB 16 /* weight rows per work item */

int dmoe_oracle_experts_ggml(const orc_layer* L, const float* x, int64_t n, const int32_t* idx, const float* w,
                             float* out, int nthreads) {
  const int64_t H = L->H, I = L->I, E = L->E, K = L->top_k, Is = L->Is;
  const int et = L->expert_type;
  const size_t rs_h = dmoe_oracle_row_size(et, H), rs_i = dmoe_oracle_row_size(et, I);
  const size_t ab_h = act_row_bytes(et, H), ab_i = act_row_bytes(et, I);
  if (!rs_h || !rs_i || !ab_h || !ab_i || n < 0 || I % ORC_RB || H % ORC_RB) return -1;
  for (int64_t i = 0; i < n * K; ++i)
    if (idx[i] < 0 || idx[i] >= E) return -2;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
  /* expert-sorted (token, slot) pairs */
  int64_t* cnt = (int64_t*)calloc((size_t)E + 1, sizeof(int64_t));
  for (int64_t i = 0; i < n * K; ++i) cnt[idx[i]]++;
  int64_t* off = (int64_t*)malloc(sizeof(int64_t) * (size_t)(E + 1));
  off[0] = 0;
  for (int64_t e = 0; e < E; ++e) off[e + 1] = off[e] + cnt[e];
  int64_t* fill = (int64_t*)calloc((size_t)E + 1, sizeof(int64_t));
  const int64_t np = n * K;
  int64_t* pair_tok = (int64_t*)malloc(sizeof(int64_t) * (size_t)(np + 1));
  int64_t* pair_slot = (int64_t*)malloc(sizeof(int64_t) * (size_t)(np + 1));
  for (int64_t t = 0; t < n; ++t)
    for (int64_t s = 0; s < K; ++s) {
      const int32_t e = idx[t * K + s];
      const int64_t p = off[e] + fill[e]++;
      pair_tok[p] = t;
      pair_slot[p] = t * K + s;
    }
  /* x rows in the vec-dot type (each token once; mul_mat_id converts src1 rows once) */
  uint8_t* xq = (uint8_t*)malloc(ab_h * (size_t)(n + 1));
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int64_t t = 0; t < n; ++t) quant_act(et, x + t * H, H, xq + (size_t)t * ab_h);
  /* gate/up work items: (expert, 16-row chunk) */
  int64_t* items = (int64_t*)malloc(sizeof(int64_t) * (size_t)(E * (H / ORC_RB) + 1));
  int64_t nit = 0;
  for (int64_t e = 0; e < E; ++e)
    if (cnt[e])
      for (int64_t r = 0; r < I / ORC_RB; ++r) items[nit++] = e * (I / ORC_RB) + r;
  float* hbuf = (float*)malloc(sizeof(float) * (size_t)(np * I + 1)); /* [pair][I] expert-sorted */
#ifdef _OPENMP
#pragma omp parallel
#endif
  {
    int16_t* scg = (int16_t*)malloc(sizeof(int16_t) * (size_t)(ORC_RB * 16 * (H / QK_K) + 16));
    int16_t* scu = (int16_t*)malloc(sizeof(int16_t) * (size_t)(ORC_RB * 16 * (H / QK_K) + 16));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
    for (int64_t it = 0; it < nit; ++it) {
      const int64_t e = items[it] / (I / ORC_RB), r0 = (items[it] % (I / ORC_RB)) * ORC_RB;
      const uint8_t* Wg = (const uint8_t*)L->w_gate + ((size_t)e * I + r0) * rs_h;
      const uint8_t* Wu = (const uint8_t*)L->w_up + ((size_t)e * I + r0) * rs_h;
      for (int rr = 0; rr < ORC_RB; ++rr) {
        unpack_scales(et, Wg + rr * rs_h, H, scg + rr * 16 * (H / QK_K));
        unpack_scales(et, Wu + rr * rs_h, H, scu + rr * 16 * (H / QK_K));
      }
      for (int64_t j = off[e]; j < off[e + 1]; ++j) {
        const uint8_t* act = xq + (size_t)pair_tok[j] * ab_h;
        for (int rr = 0; rr < ORC_RB; ++rr) {
          const float g = dot_row(et, Wg + rr * rs_h, scg + rr * 16 * (H / QK_K), act, H);
          const float u = dot_row(et, Wu + rr * rs_h, scu + rr * 16 * (H / QK_K), act, H);
          hbuf[j * I + r0 + rr] = silu_f(g) * u; /* ggml_silu then ggml_mul, f32 (:266-268) */
        }
      }
    }
    free(scg);
    free(scu);
  }
  /* h rows in the down matrix's vec-dot type */
  uint8_t* hq = (uint8_t*)malloc(ab_i * (size_t)(np + 1));
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int64_t j = 0; j < np; ++j) quant_act(et, hbuf + j * I, I, hq + (size_t)j * ab_i);
  free(hbuf);
  /* down work items: (expert, 16-row chunk of the H rows); y[slot][H] = (W_d h) * w (:269-270) */
  float* y = (float*)malloc(sizeof(float) * (size_t)(np * H + 1));
  nit = 0;
  for (int64_t e = 0; e < E; ++e)
    if (cnt[e])
      for (int64_t r = 0; r < H / ORC_RB; ++r) items[nit++] = e * (H / ORC_RB) + r;
#ifdef _OPENMP
#pragma omp parallel
#endif
  {
    int16_t* scd = (int16_t*)malloc(sizeof(int16_t) * (size_t)(ORC_RB * 16 * (I / QK_K) + 16));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
    for (int64_t it = 0; it < nit; ++it) {
      const int64_t e = items[it] / (H / ORC_RB), r0 = (items[it] % (H / ORC_RB)) * ORC_RB;
      const uint8_t* Wd = (const uint8_t*)L->w_down + ((size_t)e * H + r0) * rs_i;
      for (int rr = 0; rr < ORC_RB; ++rr) unpack_scales(et, Wd + rr * rs_i, I, scd + rr * 16 * (I / QK_K));
      for (int64_t j = off[e]; j < off[e + 1]; ++j) {
        const uint8_t* act = hq + (size_t)j * ab_i;
        const int64_t sl = pair_slot[j];
        const float wj = w[sl];
        for (int rr = 0; rr < ORC_RB; ++rr)
          y[sl * H + r0 + rr] = dot_row(et, Wd + rr * rs_i, scd + rr * 16 * (I / QK_K), act, I) * wj;
      }
    }
    free(scd);
  }
  free(hq);
  /* shared expert: weights cast to F32 (:282-284, every forward), f32 products */
  float* sd = NULL;
  if (L->sw_gate && Is > 0) {
    const int st = L->shared_type;
    float* Wg = (float*)malloc(sizeof(float) * (size_t)(Is * H));
    float* Wu = (float*)malloc(sizeof(float) * (size_t)(Is * H));
    float* Wd = (float*)malloc(sizeof(float) * (size_t)(H * Is));
    if (dmoe_oracle_dequant(st, L->sw_gate, Is, H, Wg) || dmoe_oracle_dequant(st, L->sw_up, Is, H, Wu) ||
        dmoe_oracle_dequant(st, L->sw_down, H, Is, Wd))
      return -1;
    float* sh = (float*)malloc(sizeof(float) * (size_t)(n * Is + 1));
    sd = (float*)malloc(sizeof(float) * (size_t)(n * H + 1));
    const int64_t TB = 8;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
#endif
    for (int64_t t0 = 0; t0 < n; t0 += TB)
      for (int64_t r0 = 0; r0 < Is; r0 += ORC_RB)
        for (int64_t t = t0; t < t0 + TB && t < n; ++t)
          for (int64_t r = r0; r < r0 + ORC_RB && r < Is; ++r) {
            const float g = dot_f32(Wg + r * H, x + t * H, H);
            const float u = dot_f32(Wu + r * H, x + t * H, H);
            sh[t * Is + r] = silu_f(g) * u;
          }
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
#endif
    for (int64_t t0 = 0; t0 < n; t0 += TB)
      for (int64_t r0 = 0; r0 < H; r0 += ORC_RB)
        for (int64_t t = t0; t < t0 + TB && t < n; ++t)
          for (int64_t r = r0; r < r0 + ORC_RB && r < H; ++r) sd[t * H + r] = dot_f32(Wd + r * Is, sh + t * Is, Is);
    free(sh);
    free(Wg);
    free(Wu);
    free(Wd);
  }
  /* slot sum in slot order (:273-278), then the shared expert (:285) */
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int64_t t = 0; t < n; ++t)
    for (int64_t o = 0; o < H; ++o) {
      float acc = y[(t * K) * H + o];
      for (int64_t s = 1; s < K; ++s) acc += y[(t * K + s) * H + o];
      if (sd) acc += sd[t * H + o];
      out[t * H + o] = acc;
    }
  free(sd);
  free(y);
  free(items);
  free(xq);
  free(cnt);
  free(off);
  free(fill);
  free(pair_tok);
  free(pair_slot);
  return 0;
}
