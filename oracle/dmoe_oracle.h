/*
 * dmoe_oracle.h — CPU restatement of diffuse-cpp's block-routed MoE FFN layer.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg load this library, and only as the checker. The product (libdiffuse_moe) never links
 * or calls it.
 *
 * What it restates (reference = Akicou/diffuse-cpp):
 *   src/diffuse-moe-graph.cpp:195-287   router, block capacity mask, top-k, gate weights,
 *                                        routed SwiGLU experts, slot sum, shared expert
 *   src/diffuse-common.h:59-86,103-118   layer tensors and MoE hyper-parameters
 *   src/diffuse-model.cpp:141-158        hparam defaults (capacity 48, block 32, norm_topk 1)
 *   GGUF block formats F16 / Q8_0 / Q4_K (ggml, an un-vendored submodule, commit unpinned);
 *   the dequantisers are pinned bit-for-bit against gguf-py 0.19.0 (tests/golden).
 *
 * Parity status: the quant codecs are pinned against gguf-py golden vectors. The layer maths
 * cannot be pinned against the reference itself, because ggml is absent (empty submodule, no
 * network), and the reference's own tests hold no MoE vectors. For the layer maths, parity is
 * unpinned; this file is the restatement that the CUDA path is checked against.
 *
 * Canonical arithmetic (shared by definition with the CUDA router so routing is bit-exact):
 *   logit[n][e] = P_0 + P_1 + ... + P_{S-1}  (float adds, left to right), where segment
 *   s covers h in [256 s, 256 s + 256) and P_s = fmaf chain acc = fmaf(x[n][h], W[e][h], acc)
 *   over h in order, starting from acc = 0.
 *   sigmoid(l) = 1.0f / (1.0f + (float)exp_d(-(double)l)), exp_d a Cody-Waite reduced
 *   degree-12 Taylor polynomial in double with fma (see dmoe_oracle_exp_neg).
 */
#ifndef DMOE_ORACLE_H
#define DMOE_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (ggml.h enum ggml_type) for the formats on this path */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q8_0 = 8, ORC_Q4_K = 12 };

typedef struct {
  int64_t H, I, Is, E, top_k;
  int expert_type, shared_type;
  const void *w_gate, *w_up, *w_down;    /* [E][I][H], [E][I][H], [E][H][I] in GGUF row blocks */
  const void *sw_gate, *sw_up, *sw_down; /* [Is][H], [Is][H], [H][Is]; NULL = no shared expert */
} orc_layer;

size_t dmoe_oracle_row_size(int type, int64_t k);
uint16_t dmoe_oracle_f32_to_f16(float f);
float dmoe_oracle_f16_to_f32(uint16_t h);
int dmoe_oracle_dequant(int type, const void* src, int64_t nrows, int64_t k, float* dst);

float dmoe_oracle_exp_neg(float l);
float dmoe_oracle_sigmoid(float l);

/* logits [n][e] in the canonical order; wr is [e][h] row-major (ggml ne=[H,E]) */
void dmoe_oracle_logits(const float* x, int64_t n, int64_t h, const float* wr, int64_t e, float* logits, int nthreads);

/* routing from logits. Returns 1 if block routing was used, 0 for plain per-token top-k.
 * probs [n][e] and allowed [n/blk][e] are optional outputs. */
int dmoe_oracle_route(const float* logits, int64_t n, int64_t e, const float* bias, int top_k, int cap, int blk,
                      int norm_topk, float scale, int32_t* idx, float* w, float* probs, uint8_t* allowed);

/* expert FFN + slot sum + shared expert. mode 0: double accumulation on the dequantised weights
 * (reference answer); mode 1: float accumulation on the dequantised weights; mode 2: ggml-faithful
 * (dmoe_oracle_ggml.c: weights stay in their blocks, activations rounded to the weight type's
 * vec-dot type, integer block dot products; the timed CPU baseline). Returns 0 on success. */
int dmoe_oracle_experts(const orc_layer* L, const float* x, int64_t n, const int32_t* idx, const float* w, float* out,
                        int mode, int nthreads);
int dmoe_oracle_experts_ggml(const orc_layer* L, const float* x, int64_t n, const int32_t* idx, const float* w,
                             float* out, int nthreads);
/* unit-test hooks of the ggml-faithful mode: nrows weight rows . x rounded to the vec-dot type
 * (SIMD or scalar kernel), and x rounded to the vec-dot type and widened back to float */
int dmoe_oracle_ggml_dot(int type, const void* w, int64_t nrows, int64_t k, const float* x, float* out, int simd);
int dmoe_oracle_ggml_round_act(int type, const float* x, int64_t k, float* out);

/* Greedy sampler step, src/diffuse-sampler.cpp:29-49,183-237 (dmoe_oracle_sampler.c):
 * per masked position the argmax (strict `>` scan) and 1 / sum_v expf(l_v - max) summed in float
 * in index order; the commit of the candidates sorted by probability (stable: equal
 * probabilities in position order). seq may be NULL (every row a candidate, no commit).
 * Returns the number committed. */
void dmoe_oracle_sample_row(const float* logits, int64_t n_vocab, int32_t* token, float* prob);
int32_t dmoe_oracle_sample_step(const float* logits, int64_t n_pos, int64_t n_vocab, int32_t* seq, int32_t mask_id,
                                int32_t n_transfer, float threshold, int32_t* token, float* prob);

#ifdef __cplusplus
}
#endif
#endif
