/*
 * dmoe_oracle_sampler.c — CPU restatement of one greedy denoising step of diffuse-cpp's block
 * sampler. TEST INFRASTRUCTURE ONLY (see dmoe_oracle.h): the checker of dmoe_sample_step.
 *
 * Reference (Akicou/diffuse-cpp):
 *   src/diffuse-sampler.cpp:29-49    sample_token, temperature 0: argmax by a strict `>` scan
 *                                     from v = 0; sum = expf(l_v - max) added in float, v
 *                                     ascending; prob = 1.0f / sum
 *   src/diffuse-sampler.cpp:183-206  candidates: the masked positions of the block, in position
 *                                     order, confidence = prob (low-confidence remasking)
 *   src/diffuse-sampler.cpp:212-237  sort by confidence, highest first; commit while fewer than
 *                                     n_transfer are committed or confidence >= threshold; at
 *                                     least one
 * The reference sorts with std::sort, which leaves candidates of equal confidence in an
 * unspecified order; here (and in the CUDA kernel) they keep position order (a stable sort).
 * The reference has no tests of its sampler and cannot be built here (ggml is absent), so this
 * restatement is unpinned against the reference itself.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#include "dmoe_oracle.h"

void dmoe_oracle_sample_row(const float* logits, int64_t n_vocab, int32_t* token, float* prob) {
  int64_t best = 0;
  float best_val = logits[0];
  for (int64_t v = 1; v < n_vocab; v++)
    if (logits[v] > best_val) {
      best_val = logits[v];
      best = v;
    }
  float sum = 0.0f;
  for (int64_t v = 0; v < n_vocab; v++) sum += expf(logits[v] - best_val);
  *token = (int32_t)best;
  *prob = 1.0f / sum;
}

int32_t dmoe_oracle_sample_step(const float* logits, int64_t n_pos, int64_t n_vocab, int32_t* seq, int32_t mask_id,
                                int32_t n_transfer, float threshold, int32_t* token, float* prob) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t r = 0; r < n_pos; r++) {
    if (seq && seq[r] != mask_id) {
      token[r] = -1;
      prob[r] = 0.0f;
      continue;
    }
    dmoe_oracle_sample_row(logits + r * n_vocab, n_vocab, &token[r], &prob[r]);
  }
  if (!seq) return 0;
  /* candidates in position order, then a stable insertion sort by confidence, highest first */
  int64_t* c = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n_pos > 0 ? n_pos : 1));
  int64_t nc = 0;
  for (int64_t r = 0; r < n_pos; r++)
    if (token[r] >= 0) c[nc++] = r;
  for (int64_t a = 1; a < nc; a++) {
    const int64_t x = c[a];
    int64_t b = a;
    while (b > 0 && prob[c[b - 1]] < prob[x]) {
      c[b] = c[b - 1];
      b--;
    }
    c[b] = x;
  }
  int32_t transferred = 0;
  for (int64_t k = 0; k < nc; k++) {
    if (transferred >= n_transfer && prob[c[k]] < threshold) break;
    seq[c[k]] = token[c[k]];
    transferred++;
  }
  if (transferred == 0 && nc > 0) {
    seq[c[0]] = token[c[0]];
    transferred = 1;
  }
  free(c);
  return transferred;
}
