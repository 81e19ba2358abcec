/*
 * dmoe_oracle_ffn.c — CPU restatement of the routed + shared SwiGLU experts of diffuse-cpp's
 * MoE layer (src/diffuse-moe-graph.cpp:264-286). TEST INFRASTRUCTURE ONLY (the checker and the
 * timed CPU baseline; never the product).
 *
 * Given the routing (idx, w), for every token t:
 *   out[t] = sum_{s=0..K-1} w[t][s] * Wd_e (silu(Wg_e x_t) * (Wu_e x_t)),  e = idx[t][s]
 *            (+ Ws_d (silu(Ws_g x_t) * (Ws_u x_t)) when the layer has a shared expert)
 * with the weights dequantised to fp32 exactly as their GGUF bytes encode them.
 *
 * mode 0 accumulates in double (the reference answer the CUDA path is compared with);
 * mode 1 accumulates in float (a plain fp32 CPU implementation, used as the CPU baseline).
 * This file is compiled with reassociation allowed so the dot products vectorise; the
 * routing, whose bits must match the GPU, lives in dmoe_oracle.c under strict IEEE flags.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "dmoe_oracle.h"
#ifdef _OPENMP
#include <omp.h>
#endif

static inline double dot_d(const float* a, const float* b, int64_t n) {
  double s = 0.0;
  for (int64_t k = 0; k < n; ++k) s += (double)a[k] * (double)b[k];
  return s;
}
static inline double dot_dd(const float* a, const double* b, int64_t n) {
  double s = 0.0;
  for (int64_t k = 0; k < n; ++k) s += (double)a[k] * b[k];
  return s;
}
static inline float dot_f(const float* a, const float* b, int64_t n) {
  float s = 0.0f;
  for (int64_t k = 0; k < n; ++k) s += a[k] * b[k];
  return s;
}

/* SwiGLU of one expert (dequantised weights Wg/Wu [I][H], Wd [H][I]) over `cnt` token rows;
 * row j's result times wt[j] is added into acc row j (double for mode 0, float for mode 1). */
static void swiglu(const float* Wg, const float* Wu, const float* Wd, int64_t H, int64_t I, const float* x,
                   const int64_t* tok, const float* wt, int64_t cnt, double* accd, float* accf, int mode) {
  if (mode == 0) {
    double* hb = (double*)malloc(sizeof(double) * (size_t)I);
    for (int64_t j = 0; j < cnt; ++j) {
      const float* xr = x + tok[j] * H;
      for (int64_t i = 0; i < I; ++i) {
        const double g = dot_d(Wg + i * H, xr, H);
        const double u = dot_d(Wu + i * H, xr, H);
        hb[i] = g / (1.0 + exp(-g)) * u;
      }
      double* ar = accd + j * H;
      const double wj = (double)wt[j];
      for (int64_t o = 0; o < H; ++o) ar[o] += dot_dd(Wd + o * I, hb, I) * wj;
    }
    free(hb);
  } else {
    float* hb = (float*)malloc(sizeof(float) * (size_t)I);
    for (int64_t j = 0; j < cnt; ++j) {
      const float* xr = x + tok[j] * H;
      for (int64_t i = 0; i < I; ++i) {
        const float g = dot_f(Wg + i * H, xr, H);
        const float u = dot_f(Wu + i * H, xr, H);
        hb[i] = g / (1.0f + expf(-g)) * u;
      }
      float* ar = accf + j * H;
      for (int64_t o = 0; o < H; ++o) ar[o] += dot_f(Wd + o * I, hb, I) * wt[j];
    }
    free(hb);
  }
}

int dmoe_oracle_experts(const orc_layer* L, const float* x, int64_t n, const int32_t* idx, const float* w, float* out,
                        int mode, int nthreads) {
  if (mode == 2) return dmoe_oracle_experts_ggml(L, x, n, idx, w, out, nthreads);
  const int64_t H = L->H, I = L->I, E = L->E, K = L->top_k, Is = L->Is;
  const size_t rs_h = dmoe_oracle_row_size(L->expert_type, H);
  const size_t rs_i = dmoe_oracle_row_size(L->expert_type, I);
  if (!rs_h || !rs_i || n < 0) return -1;
  for (int64_t i = 0; i < n * K; ++i)
    if (idx[i] < 0 || idx[i] >= E) return -2;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
  /* expert-sorted (token, slot) pairs, token order inside each expert */
  int64_t* cnt = (int64_t*)calloc((size_t)E + 1, sizeof(int64_t));
  for (int64_t i = 0; i < n * K; ++i) cnt[idx[i]]++;
  int64_t* off = (int64_t*)malloc(sizeof(int64_t) * (size_t)(E + 1));
  off[0] = 0;
  for (int64_t e = 0; e < E; ++e) off[e + 1] = off[e] + cnt[e];
  int64_t* fill = (int64_t*)calloc((size_t)E + 1, sizeof(int64_t));
  const int64_t np = n * K;
  int64_t* pair_tok = (int64_t*)malloc(sizeof(int64_t) * (size_t)(np + 1));
  int64_t* pair_slot = (int64_t*)malloc(sizeof(int64_t) * (size_t)(np + 1));
  float* pair_w = (float*)malloc(sizeof(float) * (size_t)(np + 1));
  for (int64_t t = 0; t < n; ++t)
    for (int64_t s = 0; s < K; ++s) {
      const int32_t e = idx[t * K + s];
      const int64_t p = off[e] + fill[e]++;
      pair_tok[p] = t;
      pair_slot[p] = t * K + s;
      pair_w[p] = w[t * K + s];
    }
  /* per-slot outputs y[t][s][H], summed in slot order at the end (:273-278) */
  double* yd = mode == 0 ? (double*)calloc((size_t)(np * H), sizeof(double)) : NULL;
  float* yf = mode != 0 ? (float*)calloc((size_t)(np * H), sizeof(float)) : NULL;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1)
#endif
  for (int64_t e = 0; e < E; ++e) {
    const int64_t c = cnt[e];
    if (c == 0) continue;
    float* Wg = (float*)malloc(sizeof(float) * (size_t)(I * H));
    float* Wu = (float*)malloc(sizeof(float) * (size_t)(I * H));
    float* Wd = (float*)malloc(sizeof(float) * (size_t)(H * I));
    dmoe_oracle_dequant(L->expert_type, (const uint8_t*)L->w_gate + (size_t)e * I * rs_h, I, H, Wg);
    dmoe_oracle_dequant(L->expert_type, (const uint8_t*)L->w_up + (size_t)e * I * rs_h, I, H, Wu);
    dmoe_oracle_dequant(L->expert_type, (const uint8_t*)L->w_down + (size_t)e * H * rs_i, H, I, Wd);
    double* td = mode == 0 ? (double*)calloc((size_t)(c * H), sizeof(double)) : NULL;
    float* tf = mode != 0 ? (float*)calloc((size_t)(c * H), sizeof(float)) : NULL;
    swiglu(Wg, Wu, Wd, H, I, x, pair_tok + off[e], pair_w + off[e], c, td, tf, mode);
    for (int64_t j = 0; j < c; ++j) {
      const int64_t sl = pair_slot[off[e] + j];
      if (mode == 0)
        memcpy(yd + sl * H, td + j * H, sizeof(double) * (size_t)H);
      else
        memcpy(yf + sl * H, tf + j * H, sizeof(float) * (size_t)H);
    }
    free(td);
    free(tf);
    free(Wg);
    free(Wu);
    free(Wd);
  }
  /* shared expert on the MoE input with weight 1 (:280-286); its weights are cast to F32 */
  double* shd = NULL;
  float* shf = NULL;
  if (L->sw_gate) {
    const size_t rs_sh = dmoe_oracle_row_size(L->shared_type, H);
    const size_t rs_si = dmoe_oracle_row_size(L->shared_type, Is);
    if (!rs_sh || !rs_si) return -1;
    float* Wg = (float*)malloc(sizeof(float) * (size_t)(Is * H));
    float* Wu = (float*)malloc(sizeof(float) * (size_t)(Is * H));
    float* Wd = (float*)malloc(sizeof(float) * (size_t)(H * Is));
    dmoe_oracle_dequant(L->shared_type, L->sw_gate, Is, H, Wg);
    dmoe_oracle_dequant(L->shared_type, L->sw_up, Is, H, Wu);
    dmoe_oracle_dequant(L->shared_type, L->sw_down, H, Is, Wd);
    int64_t* alltok = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n + 1));
    float* ones = (float*)malloc(sizeof(float) * (size_t)(n + 1));
    for (int64_t t = 0; t < n; ++t) {
      alltok[t] = t;
      ones[t] = 1.0f;
    }
    if (mode == 0)
      shd = (double*)calloc((size_t)(n * H) + 1, sizeof(double));
    else
      shf = (float*)calloc((size_t)(n * H) + 1, sizeof(float));
    const int64_t chunk = 8;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int64_t t0 = 0; t0 < n; t0 += chunk) {
      const int64_t c = (n - t0) < chunk ? (n - t0) : chunk;
      swiglu(Wg, Wu, Wd, H, Is, x, alltok + t0, ones + t0, c, shd ? shd + t0 * H : NULL, shf ? shf + t0 * H : NULL,
             mode);
    }
    free(alltok);
    free(ones);
    free(Wg);
    free(Wu);
    free(Wd);
  }
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int64_t t = 0; t < n; ++t)
    for (int64_t o = 0; o < H; ++o) {
      if (mode == 0) {
        double acc = 0.0;
        for (int64_t s = 0; s < K; ++s) acc += yd[(t * K + s) * H + o];
        if (shd) acc += shd[t * H + o];
        out[t * H + o] = (float)acc;
      } else {
        float acc = 0.0f;
        for (int64_t s = 0; s < K; ++s) acc += yf[(t * K + s) * H + o];
        if (shf) acc += shf[t * H + o];
        out[t * H + o] = acc;
      }
    }
  free(yd);
  free(yf);
  free(shd);
  free(shf);
  free(cnt);
  free(off);
  free(fill);
  free(pair_tok);
  free(pair_slot);
  free(pair_w);
  return 0;
}
