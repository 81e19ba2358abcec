/*
 * dmoe_oracle.c — CPU restatement of diffuse-cpp's block-routed MoE FFN layer.
 * TEST INFRASTRUCTURE ONLY (the checker, never the product). Header: dmoe_oracle.h.
 *
 * Build: see oracle/Makefile. Compiled with -ffp-contract=off so that the only fused
 * multiply-adds are the explicit fmaf()/fma() calls of the canonical order.
 */
#include "dmoe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK8_0 32
#define QK_K 256
#define ROUTER_SEG 256

/* ------------------------------------------------------------------------------------------ */
/* IEEE binary16 <-> binary32, round to nearest even (GGML_FP32_TO_FP16 semantics)            */
/* ------------------------------------------------------------------------------------------ */
float dmoe_oracle_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t exp = (h >> 10) & 0x1F;
  const uint32_t man = h & 0x3FF;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal half -> normal float */
      float v = (float)man * (1.0f / 16777216.0f); /* man * 2^-24, exact */
      memcpy(&bits, &v, 4);
      bits |= sign;
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t dmoe_oracle_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) { /* inf / nan */
    return (uint16_t)(sign | 0x7C00 | (ax > 0x7F800000u ? 0x200 : 0));
  }
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00); /* rounds to >= 65520 -> inf */
  if (ax < 0x38800000u) {                                   /* below min normal half: subnormal */
    /* value * 2^24 rounded to nearest even integer = half subnormal mantissa */
    float a;
    memcpy(&a, &ax, 4);
    float s = a * 16777216.0f; /* exact scaling by power of two */
    float r = nearbyintf(s);   /* ties to even in default rounding mode */
    return (uint16_t)(sign | (uint16_t)r);
  }
  /* normal: round mantissa from 23 to 10 bits, ties to even */
  uint32_t e = (ax >> 23) - 112;
  uint32_t m = ax & 0x7FFFFFu;
  uint32_t h = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1; /* carry may bump exponent: fine */
  return (uint16_t)(sign | h);
}

/* ------------------------------------------------------------------------------------------ */
/* GGUF block formats                                                                          */
/* ------------------------------------------------------------------------------------------ */
size_t dmoe_oracle_row_size(int type, int64_t k) {
  switch (type) {
    case ORC_F32: return (size_t)k * 4;
    case ORC_F16: return (size_t)k * 2;
    case ORC_Q8_0: return (size_t)(k / QK8_0) * 34;
    case ORC_Q4_K: return (size_t)(k / QK_K) * 144;
    default: return 0;
  }
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Q4_K 6-bit scale/min unpack: sub-block j of a super-block (format of ggml's block_q4_K). */
static inline void q4k_scale_min(int j, const uint8_t* q, uint8_t* sc, uint8_t* m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
    *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

static void dequant_row(int type, const uint8_t* src, int64_t k, float* dst) {
  if (type == ORC_F32) {
    memcpy(dst, src, (size_t)k * 4);
  } else if (type == ORC_F16) {
    for (int64_t i = 0; i < k; ++i) dst[i] = dmoe_oracle_f16_to_f32(rd16(src + 2 * i));
  } else if (type == ORC_Q8_0) {
    for (int64_t b = 0; b < k / QK8_0; ++b) {
      const uint8_t* blk = src + b * 34;
      const float d = dmoe_oracle_f16_to_f32(rd16(blk));
      for (int j = 0; j < QK8_0; ++j) dst[b * QK8_0 + j] = (float)(int8_t)blk[2 + j] * d;
    }
  } else if (type == ORC_Q4_K) {
    for (int64_t b = 0; b < k / QK_K; ++b) {
      const uint8_t* blk = src + b * 144;
      const float d = dmoe_oracle_f16_to_f32(rd16(blk));
      const float dmin = dmoe_oracle_f16_to_f32(rd16(blk + 2));
      const uint8_t* scales = blk + 4;
      const uint8_t* qs = blk + 16;
      float* y = dst + b * QK_K;
      for (int g = 0; g < 4; ++g) { /* 64 weights per group: 32 low nibbles, then 32 high */
        uint8_t sc, m;
        q4k_scale_min(2 * g, scales, &sc, &m);
        const float d1 = d * (float)sc, m1 = dmin * (float)m;
        q4k_scale_min(2 * g + 1, scales, &sc, &m);
        const float d2 = d * (float)sc, m2 = dmin * (float)m;
        for (int l = 0; l < 32; ++l) y[64 * g + l] = d1 * (float)(qs[32 * g + l] & 0xF) - m1;
        for (int l = 0; l < 32; ++l) y[64 * g + 32 + l] = d2 * (float)(qs[32 * g + l] >> 4) - m2;
      }
    }
  }
}

int dmoe_oracle_dequant(int type, const void* src, int64_t nrows, int64_t k, float* dst) {
  const size_t rs = dmoe_oracle_row_size(type, k);
  if (rs == 0) return -1;
  if ((type == ORC_Q8_0 && k % QK8_0) || (type == ORC_Q4_K && k % QK_K)) return -1;
  for (int64_t r = 0; r < nrows; ++r) dequant_row(type, (const uint8_t*)src + r * rs, k, dst + r * k);
  return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* Router: canonical logits, sigmoid                                                            */
/* ------------------------------------------------------------------------------------------ */

/* exp(-l) rounded to float. Cody-Waite reduction x = k ln2 + r, |r| <= ln2/2, then the degree-12
 * Taylor polynomial of e^r by Horner with fma, then scaling by 2^k. All double arithmetic is
 * IEEE (fma, mul, rint), so the CUDA router computes the same bits. */
float dmoe_oracle_exp_neg(float l) {
  const double x = -(double)l;
  if (x > 104.0) return INFINITY;
  if (x < -110.0) return 0.0f;
  const double kd = rint(x * 1.4426950408889634);
  double r = fma(-kd, 0x1.62e42fefa39efp-1, x);
  r = fma(-kd, 2.3190468138462996e-17, r);
  double p = 2.08767569878681e-09;
  p = fma(p, r, 2.505210838544172e-08);
  p = fma(p, r, 2.755731922398589e-07);
  p = fma(p, r, 2.7557319223985893e-06);
  p = fma(p, r, 2.48015873015873e-05);
  p = fma(p, r, 0.0001984126984126984);
  p = fma(p, r, 0.001388888888888889);
  p = fma(p, r, 0.008333333333333333);
  p = fma(p, r, 0.041666666666666664);
  p = fma(p, r, 0.16666666666666666);
  p = fma(p, r, 0.5);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  const int64_t k = (int64_t)kd;
  uint64_t sbits = (uint64_t)(k + 1023) << 52;
  double s;
  memcpy(&s, &sbits, 8);
  return (float)(p * s);
}

float dmoe_oracle_sigmoid(float l) {
  const float e = dmoe_oracle_exp_neg(l);
  const float den = 1.0f + e;
  return 1.0f / den;
}

void dmoe_oracle_logits(const float* x, int64_t n, int64_t h, const float* wr, int64_t e, float* logits, int nthreads) {
  /* W transposed to [h][e] so the inner loop runs over experts (independent fma chains) */
  float* wt = (float*)malloc(sizeof(float) * (size_t)(h * e));
  for (int64_t i = 0; i < e; ++i)
    for (int64_t k = 0; k < h; ++k) wt[k * e + i] = wr[i * h + k];
  const int64_t nseg = (h + ROUTER_SEG - 1) / ROUTER_SEG;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel
#endif
  {
    float* acc = (float*)malloc(sizeof(float) * (size_t)e);
    float* tot = (float*)malloc(sizeof(float) * (size_t)e);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
    for (int64_t t = 0; t < n; ++t) {
      const float* xr = x + t * h;
      for (int64_t s = 0; s < nseg; ++s) {
        for (int64_t i = 0; i < e; ++i) acc[i] = 0.0f;
        const int64_t k1 = (s + 1) * ROUTER_SEG < h ? (s + 1) * ROUTER_SEG : h;
        for (int64_t k = s * ROUTER_SEG; k < k1; ++k) {
          const float xv = xr[k];
          const float* wk = wt + k * e;
          for (int64_t i = 0; i < e; ++i) acc[i] = fmaf(xv, wk[i], acc[i]);
        }
        if (s == 0)
          for (int64_t i = 0; i < e; ++i) tot[i] = acc[i];
        else
          for (int64_t i = 0; i < e; ++i) tot[i] = tot[i] + acc[i];
      }
      memcpy(logits + t * e, tot, sizeof(float) * (size_t)e);
    }
    free(acc);
    free(tot);
  }
  free(wt);
}

/* ------------------------------------------------------------------------------------------ */
/* Router: block capacity + per-token top-k  (src/diffuse-moe-graph.cpp:204-262)              */
/* ------------------------------------------------------------------------------------------ */
static inline int better(float va, int ia, float vb, int ib) { return va > vb || (va == vb && ia < ib); }

int dmoe_oracle_route(const float* logits, int64_t n, int64_t e, const float* bias, int top_k, int cap, int blk,
                      int norm_topk, float scale, int32_t* idx, float* w, float* probs, uint8_t* allowed) {
  float* p = (float*)malloc(sizeof(float) * (size_t)(n * e));
  float* sel = (float*)malloc(sizeof(float) * (size_t)(n * e));
  /* :203-210 sigmoid probs, bias for selection only */
  for (int64_t i = 0; i < n * e; ++i) {
    p[i] = dmoe_oracle_sigmoid(logits[i]);
    sel[i] = bias ? p[i] + bias[i % e] : p[i];
  }
  /* :215-216 block routing switch */
  const int use_block = blk > 1 && cap > 0 && cap < e && (n % blk) == 0;
  if (use_block) {
    const int64_t nb = n / blk;
    float* bmax = (float*)malloc(sizeof(float) * (size_t)e);
    float* srt = (float*)malloc(sizeof(float) * (size_t)e);
    for (int64_t b = 0; b < nb; ++b) {
      const float* s0 = sel + b * blk * e;
      /* :223-229 fold max(a,b) = b + relu(a - b), t = 1..blk-1 in order */
      for (int64_t i = 0; i < e; ++i) bmax[i] = s0[i];
      for (int t = 1; t < blk; ++t) {
        const float* st = s0 + (int64_t)t * e;
        for (int64_t i = 0; i < e; ++i) {
          const float d = bmax[i] - st[i];
          const float rl = d > 0.0f ? d : 0.0f;
          bmax[i] = st[i] + rl;
        }
      }
      /* :231-236 thr = cap-th largest (descending order, index cap-1) */
      for (int64_t i = 0; i < e; ++i) {
        /* rank = number of strictly greater; the value at sorted position cap-1 is the one
         * whose [rank, rank + #equal) interval contains cap-1 */
        srt[i] = bmax[i];
      }
      float thr = 0.0f;
      for (int64_t i = 0; i < e; ++i) {
        int64_t gt = 0, eq = 0;
        for (int64_t j = 0; j < e; ++j) {
          gt += srt[j] > srt[i];
          eq += srt[j] == srt[i];
        }
        if (gt <= cap - 1 && cap - 1 < gt + eq) {
          thr = srt[i];
          break;
        }
      }
      /* :241-248 keep = step(bmax - (thr - 1e-6)); masked scores += -1e30 */
      const float thr_m = thr * 1.0f + (-1e-6f);
      for (int64_t i = 0; i < e; ++i) {
        const float dlt = bmax[i] - thr_m;
        const int keep = dlt > 0.0f;
        if (allowed) allowed[b * e + i] = (uint8_t)keep;
        const float add = keep ? 0.0f : -1e30f;
        for (int t = 0; t < blk; ++t) {
          float* st = sel + (b * blk + t) * e;
          st[i] = st[i] + add;
        }
      }
    }
    free(bmax);
    free(srt);
  }
  /* :252-262 per-token top-k, unbiased weights, renormalise, scale */
  for (int64_t t = 0; t < n; ++t) {
    const float* st = sel + t * e;
    int32_t* it = idx + t * top_k;
    for (int s = 0; s < top_k; ++s) {
      int best = -1;
      for (int64_t i = 0; i < e; ++i) {
        int taken = 0;
        for (int q = 0; q < s; ++q) taken |= it[q] == (int32_t)i;
        if (taken) continue;
        if (best < 0 || better(st[i], (int)i, st[best], best)) best = (int)i;
      }
      it[s] = best;
    }
    float* wt = w + t * top_k;
    for (int s = 0; s < top_k; ++s) wt[s] = p[t * e + it[s]];
    if (norm_topk) {
      double sum = 0.0;
      for (int s = 0; s < top_k; ++s) sum += (double)wt[s];
      const float fs = (float)sum;
      for (int s = 0; s < top_k; ++s) wt[s] = wt[s] / fs;
    }
    if (scale != 1.0f)
      for (int s = 0; s < top_k; ++s) wt[s] = wt[s] * scale;
  }
  if (probs) memcpy(probs, p, sizeof(float) * (size_t)(n * e));
  free(p);
  free(sel);
  return use_block;
}

