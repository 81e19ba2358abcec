/*
 * diffuse_moe.h — C ABI of libdiffuse_moe, a B200 (sm_100a) implementation of diffuse-cpp's
 * block-routed MoE FFN layer (LLaDA2-style: sigmoid router, expert-bias selection, per-block
 * expert capacity, per-token top-k, renormalised x routed_scaling gates, SwiGLU experts and an
 * always-on shared expert).
 *
 * The library is a drop-in for the MoE subgraph the reference graph builder emits
 * (Akicou/diffuse-cpp src/diffuse-moe-graph.cpp:195-287): same weight tensors in their GGUF
 * layouts and quant types (F16, Q8_0, Q4_K), same router semantics, same output
 * (moe_out, routed + shared, without the residual that :292 adds).
 *
 * Plain C types only. Every entry point returns a status; none exits the process and none
 * falls back to the CPU: without a usable CUDA device dmoe_create returns DMOE_ERR_NO_DEVICE.
 */
#ifndef DIFFUSE_MOE_H
#define DIFFUSE_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DMOE_ABI_VERSION 5

/* Replaces the reference's bool returns + DIFFUSE_DIE/exit(1) (src/diffuse-common.h:22-27,
 * src/diffuse-moe-graph.cpp:325-329). */
typedef enum dmoe_status {
  DMOE_OK = 0,
  DMOE_ERR_INVALID_ARG = 1,  /* bad shape, null pointer, unsupported hyper-parameter */
  DMOE_ERR_UNSUPPORTED = 2,  /* quant type / shape this build does not handle */
  DMOE_ERR_NO_DEVICE = 3,    /* no CUDA device (there is no CPU fallback) */
  DMOE_ERR_CUDA = 4,         /* CUDA runtime / driver error; see dmoe_last_error */
  DMOE_ERR_NCCL = 5,         /* expert-parallel communication error */
  DMOE_ERR_TIMEOUT = 6,      /* a bounded wait expired: a device-side wait (the kernel gave up) or a
                                collective past dmoe_dist_cfg.timeout_ms (communicator aborted) */
  DMOE_ERR_OOM = 7           /* device allocation failed */
} dmoe_status;

/* ggml_type ids (ggml.h enum ggml_type) of the weight formats on this path. The GGUF block
 * layouts are unchanged: F16 rows; Q8_0 = 32-weight blocks {f16 d; int8 q[32]};
 * Q4_K = 256-weight super-blocks {f16 d; f16 dmin; u8 scales[12]; u8 qs[128]}. */
enum {
  DMOE_TYPE_F32 = 0,
  DMOE_TYPE_F16 = 1,
  DMOE_TYPE_Q8_0 = 8,
  DMOE_TYPE_Q4_K = 12
};

/* One MoE layer: the tensors of struct diffuse_moe_layer (src/diffuse-common.h:72-82) and the
 * MoE hyper-parameters of struct diffuse_model (src/diffuse-common.h:103-116) as loaded by
 * diffuse_model_load_impl (src/diffuse-model.cpp:141-158, 187-196). All pointers are HOST
 * memory in GGUF layout (ggml ne order, fastest dimension first):
 *   w_gate, w_up   ne = [n_embd, n_ff_exp, n_expert]   ("blk.N.moe_experts_{gate,up}.weight")
 *   w_down         ne = [n_ff_exp, n_embd, n_expert]   ("blk.N.moe_experts_down.weight")
 *   sw_gate, sw_up ne = [n_embd, n_ff_shexp]           ("blk.N.moe_shared_{gate,up}.weight")
 *   sw_down        ne = [n_ff_shexp, n_embd]           ("blk.N.moe_shared_down.weight")
 *   w_router       ne = [n_embd, n_expert], F32        ("blk.N.moe_gate.weight")
 *   b_router       ne = [n_expert], F32, or NULL        ("blk.N.moe_gate_bias.weight")
 * The data is copied to the device by dmoe_create; the caller may free it afterwards. */
typedef struct dmoe_layer_desc {
  int64_t n_embd;          /* H */
  int64_t n_ff_exp;        /* I   expert_feed_forward_length */
  int64_t n_ff_shexp;      /* I_s shared expert width; 0 = no shared expert (:281) */
  int64_t n_expert;        /* E   expert_count */
  int64_t n_expert_used;   /* top-k  expert_used_count (<= 16) */
  int64_t expert_capacity; /* experts allowed per routing block (default 48) */
  int64_t moe_block_size;  /* tokens per routing block (default 32) */
  float routed_scaling;    /* routed_scaling_factor (default 1) */
  int32_t norm_topk_prob;  /* renormalise the top-k gates (default 1) */
  int32_t expert_type;     /* DMOE_TYPE_* of w_gate / w_up / w_down */
  int32_t shared_type;     /* DMOE_TYPE_* of sw_gate / sw_up / sw_down */
  const void* w_gate;
  const void* w_up;
  const void* w_down;
  const void* sw_gate;
  const void* sw_up;
  const void* sw_down;
  const float* w_router;
  const float* b_router;
} dmoe_layer_desc;

/* Expert parallelism: one process per GPU; every rank calls dmoe_create and dmoe_forward
 * collectively with its own token shard (whole routing blocks). NULL (or world_size 1) = single
 * GPU. Rank r owns experts [r E / W, (r + 1) E / W) (E % W == 0, W <= 32); router, bias and shared
 * expert are replicated. Each forward routes locally, sends one fp16 row per (token, owning
 * rank) with its slot list, computes the local experts' weighted partial rows, returns them to
 * the token's rank and adds them to the shared expert's rows there (NCCL send / recv, loaded at
 * run time from libnccl.so.2). Every collective wait has the host deadline timeout_ms; when it
 * passes the call returns DMOE_ERR_TIMEOUT, the communicator is aborted and the layer refuses
 * further forwards (destroy and re-create it on every rank). dmoe_create itself waits at most
 * timeout_ms for all ranks to join. */
typedef struct dmoe_dist_cfg {
  int32_t rank;
  int32_t world_size;
  int32_t device;          /* CUDA device ordinal for this rank */
  int32_t timeout_ms;      /* host deadline for a collective; 0 = 60000 */
  const void* nccl_id;     /* 128-byte ncclUniqueId, identical on all ranks */
} dmoe_dist_cfg;

/* Optional routing outputs (for parity checks and statistics). Any field may be NULL. */
typedef struct dmoe_route_out {
  int32_t* idx;            /* [n_tokens][n_expert_used] selected experts, slot order */
  float* weights;          /* [n_tokens][n_expert_used] applied gates */
  uint8_t* allowed;        /* [n_tokens / moe_block_size][n_expert] capacity mask (block routing) */
} dmoe_route_out;

/* Statistics of the last dmoe_forward, valid after dmoe_sync. */
typedef struct dmoe_stats {
  int32_t n_active;        /* distinct routed experts selected */
  int32_t n_routed_tiles;  /* routed token tiles fed to the expert GEMMs */
  int32_t token_tile;      /* token tile width of the expert GEMMs */
  int32_t ksplit_gateup;   /* split-K factors used */
  int32_t ksplit_down;
  int32_t router_parts;    /* router segment partials (1 = fused running sum) */
  int32_t kernels;         /* kernels enqueued by the last forward */
  int32_t used_block_routing;
  float ms_router;         /* per-stage device times, with DMOE_F_PROFILE */
  float ms_dispatch;
  float ms_gateup;
  float ms_down;
  float ms_total;
  int64_t ep_rows_sent;     /* expert parallelism: (token, rank) rows sent / received */
  int64_t ep_rows_received;
  int32_t fused_gemm;       /* 1: gate/up and down ran as one launch (ms_down holds both, ms_gateup ~ 0) */
} dmoe_stats;

#define DMOE_F_HOST_PTRS 1u   /* x, out and route_out are host memory: the call copies them and
                                 returns after the result is on the host */
#define DMOE_F_ROUTE_ONLY 2u  /* run the router only (out is not touched) */
#define DMOE_F_PROFILE 4u     /* record CUDA events around each stage (dmoe_get_stats) */
#define DMOE_F_DETERMINISTIC 8u /* bitwise-reproducible output: every (token, slot) row of the down
                                   projection is stored and summed per token in slot order, then
                                   the shared expert added (the order of diffuse-moe-graph.cpp:
                                   273-286); without it rows are reduced with fp32 atomics, which
                                   is faster but leaves the summation order to the hardware */

/* Binds one layer: validates the shapes, uploads router, bias and expert weights to the device
 * once (library-owned), prepares the TMA descriptors. Replaces the per-forward weight binding
 * and F32 casts of src/diffuse-moe-graph.cpp:8-12,203,282-284 (weights are never re-staged). */
dmoe_status dmoe_create(const dmoe_layer_desc* desc, const dmoe_dist_cfg* dist, struct dmoe_layer** out);

/* Writes a fresh 128-byte NCCL unique id for dmoe_dist_cfg.nccl_id (create it on one rank and
 * share it with the others). No counterpart in the reference, which runs on one device. */
dmoe_status dmoe_nccl_unique_id(void* id128);

/* dmoe_create for a further expert-parallel layer of the same ranks: its communicator is split
 * from `parent`'s (ncclCommSplit) instead of initialised from dist->nccl_id (which may be NULL),
 * so one unique id serves all layers of a model. Collective over the parent's ranks; dist gives
 * this rank's rank / world_size / device / timeout_ms, which must match the parent's. */
dmoe_status dmoe_create_split(const dmoe_layer_desc* desc, const dmoe_dist_cfg* dist,
                              const struct dmoe_layer* parent, struct dmoe_layer** out);

/* ---- Whole-model upload from GGUF (replaces diffuse_model_load_impl,
 * src/diffuse-model.cpp:67-224, for the MoE layers, and the weight offload that
 * src/diffuse-backend.h:104-118 leaves undone). dmoe_model_load maps the file, reads the
 * hyper-parameters as the reference does (keys "<prefix>.<name>" with prefix "diffuse", "qwen2"
 * or "llama": block_count, embedding_length, expert_count, expert_used_count,
 * expert_shared_count, expert_feed_forward_length, first_k_dense_replace, routed_scaling_factor
 * (default 1), norm_topk_prob (1), expert_capacity (48), moe_block_size (block_length, else 32)),
 * and binds every MoE layer il >= first_k_dense_replace from its tensors blk.<il>.moe_gate.weight,
 * moe_gate_bias.weight (optional), moe_experts_{gate,up,down}.weight and, with shared experts,
 * moe_shared_{gate,up,down}.weight: each is copied to the device once and the file is unmapped
 * before the call returns. The model must be "llada2_moe" (diffuse.model_type; the reference's
 * default without that key unless the architecture is qwen2 or llama). dist: as for dmoe_create
 * (collective); the first MoE layer's communicator comes from dist->nccl_id and the others are
 * split from it. */
typedef struct dmoe_model_info {
  int32_t n_layer;          /* block_count */
  int32_t first_k_dense;    /* layers [0, first_k_dense) are dense: no MoE layer */
  int32_t n_moe_layers;     /* n_layer - first_k_dense */
  int32_t expert_type;      /* DMOE_TYPE_* of the expert stacks, and of the shared expert */
  int32_t shared_type;
  int32_t norm_topk_prob;
  float routed_scaling;
  int64_t n_embd;
  int64_t n_ff_exp;
  int64_t n_ff_shexp;       /* 0 without shared experts */
  int64_t n_expert;
  int64_t n_expert_used;
  int64_t expert_capacity;
  int64_t moe_block_size;
  int64_t moe_bytes;        /* bytes of MoE tensors read from the file, over all layers */
} dmoe_model_info;

struct dmoe_model;
dmoe_status dmoe_model_load(const char* path, const dmoe_dist_cfg* dist, struct dmoe_model** out);
/* The checks of dmoe_model_load without a device: reads the file's hyper-parameters and every MoE
 * tensor's name, shape and type into info; nothing is copied. */
dmoe_status dmoe_model_inspect(const char* path, dmoe_model_info* info);
dmoe_status dmoe_model_get_info(const struct dmoe_model* model, dmoe_model_info* info);
/* The bound layer of block il, or NULL for a dense block or il out of range; owned by the model. */
struct dmoe_layer* dmoe_model_layer(struct dmoe_model* model, int32_t il);
void dmoe_model_free(struct dmoe_model* model);

/* Hot-expert replication for skewed expert-parallel loads. No counterpart in the reference,
 * which runs on one device. Collective: every rank calls it with the same arguments, between
 * forwards. Afterwards every rank holds the weights of n_hot experts besides its own (each copied
 * once from its owner, NCCL broadcast; the host tensors are not needed), and a (token, slot)
 * that selects one of them is computed on the token's own rank, with no exchange; results are
 * unchanged. ids: the experts to replicate, distinct, in [0, n_expert), identical on every
 * rank; NULL: the n_hot experts with the most (token, slot) pairs in the layer's last forward,
 * summed over the ranks (ties to the lower id). n_hot = 0 drops the replicas. Requires
 * n_hot <= DMOE_MAX_HOT and n_hot <= n_expert - n_expert / world_size. Each replica costs one
 * expert's weights of device memory per rank. On one GPU it returns DMOE_OK and does nothing. */
#define DMOE_MAX_HOT 64
dmoe_status dmoe_replicate_experts(struct dmoe_layer* layer, const int32_t* ids, int32_t n_hot);

/* moe_out = MoE(x). Replaces src/diffuse-moe-graph.cpp:195-287 (router :203-262, experts
 * :264-278, shared expert :280-286). x and out are [n_tokens][n_embd] f32, row-major (ggml
 * ne = [n_embd, n_tokens]). Without DMOE_F_HOST_PTRS they are device pointers and the work is
 * enqueued on `stream` (a cudaStream_t, NULL = the CUDA default stream); call dmoe_sync (or
 * synchronise the stream) before reading results. With DMOE_F_HOST_PTRS a NULL stream selects
 * the layer's own stream and the call returns when the results are on the host. Block routing is used iff moe_block_size > 1, 0 < expert_capacity <
 * n_expert and n_tokens % moe_block_size == 0 (:215-216); otherwise plain per-token top-k.
 * Calls on one layer handle are not reentrant. */
dmoe_status dmoe_forward(struct dmoe_layer* layer, const float* x, int64_t n_tokens, float* out,
                         const dmoe_route_out* route, void* stream, uint32_t flags);

/* Waits for the layer's work, reports device-side timeouts (DMOE_ERR_TIMEOUT) and token tiles that
 * the device built out of bounds (DMOE_ERR_CUDA; such a tile is skipped), refreshes the statistics. */
dmoe_status dmoe_sync(struct dmoe_layer* layer);

dmoe_status dmoe_get_stats(const struct dmoe_layer* layer, dmoe_stats* stats);

void dmoe_destroy(struct dmoe_layer* layer);

/* Message of the last error on this thread; returns its full length. */
size_t dmoe_last_error(char* buf, size_t len);

int32_t dmoe_abi_version(void);

/* Host-side GGUF quantiser for building weights. Replaces tools/quant_lib.c:16-27
 * (quantize_to_type -> ggml_quantize_chunk): Q8_0 follows ggml's round-to-nearest scheme
 * (amax / 127, roundf); Q4_K uses this library's own scale/min search over the same block
 * format. F16 is round-to-nearest-even, F32 a copy. Returns the bytes written, 0 on error. */
size_t dmoe_quantize(int32_t type, const float* src, void* dst, int64_t nrows, int64_t n_per_row);

/* Bytes of nrows rows of n_per_row values. Replaces tools/quant_lib.c:30-33. */
size_t dmoe_quantized_size(int32_t type, int64_t nrows, int64_t n_per_row);

/* Routing without any device allocation. No counterpart in the reference: it exists for callers
 * that cannot call cudaMalloc, such as a process whose device memory is owned by another
 * allocator (a serving stack that reserves its whole budget at start-up, or a host framework
 * that hands out every buffer itself). It computes exactly what dmoe_forward with
 * DMOE_F_ROUTE_ONLY computes (same kernels, same canonical bits), but takes every tensor as a
 * DEVICE pointer from the caller and needs no dmoe_create:
 *   x         [n_tokens][n_embd] f32          w_router [n_expert][n_embd] f32 (GGUF layout)
 *   b_router  [n_expert] f32 or NULL          idx / weights [n_tokens][n_expert_used] (outputs)
 * The work is enqueued on `stream` (NULL = the CUDA default stream) of the current device.
 * Its scratch is one fixed array of DMOE_STATIC_SCRATCH_BYTES inside the library, held by every
 * GPU that loads the library until the process exits. The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture. All calls share the array: calls that overlap on the GPU (other
 * streams or threads) race on it. Sizes above n_tokens <= DMOE_STATIC_MAX_TOKENS,
 * n_expert <= DMOE_STATIC_MAX_EXPERTS, n_embd <= DMOE_STATIC_MAX_EMBD are rejected with
 * DMOE_ERR_UNSUPPORTED; n_embd must be a multiple of 256, n_expert of 4. x and b_router must be
 * 16-byte aligned and w_router, idx, weights 4-byte aligned (contiguous row-major tensors);
 * other pointers are refused with DMOE_ERR_INVALID_ARG before any device work. */
#define DMOE_STATIC_MAX_TOKENS 4096
#define DMOE_STATIC_MAX_EXPERTS 256
#define DMOE_STATIC_MAX_EMBD 8192
#define DMOE_STATIC_SCRATCH_BYTES                                                                  \
  (4ull * (1ull * DMOE_STATIC_MAX_TOKENS * DMOE_STATIC_MAX_EXPERTS +                                \
           (unsigned long long)DMOE_STATIC_MAX_EMBD * DMOE_STATIC_MAX_EXPERTS + DMOE_STATIC_MAX_EXPERTS))
dmoe_status dmoe_route_static(const float* x, int64_t n_tokens, int64_t n_embd, const float* w_router,
                              const float* b_router, int64_t n_expert, int64_t n_expert_used,
                              int64_t expert_capacity, int64_t moe_block_size, float routed_scaling,
                              int32_t norm_topk_prob, int32_t* idx, float* weights, void* stream);

/* One denoising step of the block sampler, greedy (temperature 0, low-confidence remasking: the
 * reference's defaults, include/diffuse.h:42-46), on the GPU. Replaces sample_token's argmax
 * branch (src/diffuse-sampler.cpp:29-49) for every masked position and the step's commit
 * (:183-237), so the logits never leave the device (the reference copies all of them to the host,
 * src/diffuse-moe-graph.cpp:331-332). All pointers are DEVICE memory:
 *   logits  [n_pos][n_vocab] f32: the rows of the block's positions
 *   seq     [n_pos] int32: the block's tokens; position r is a candidate iff seq[r] == mask_id.
 *           Committed positions receive their token. NULL: every row is a candidate, nothing is
 *           committed (argmax and probability only).
 *   token, prob [n_pos]: per candidate its argmax (the lowest index among equal maxima) and
 *           1 / sum_v exp(l_v - max); -1 and 0 for other positions
 *   n_committed (optional) : how many positions were committed
 * Commit rule: candidates by probability, highest first (equal probabilities in position order;
 * the reference's std::sort leaves that order unspecified); the first n_transfer are committed,
 * then every further one with probability >= threshold; at least one. Enqueued on `stream`
 * (NULL = the CUDA default stream); n_pos <= DMOE_SAMPLE_MAX_POS. */
#define DMOE_SAMPLE_MAX_POS 1024
dmoe_status dmoe_sample_step(const float* logits, int64_t n_pos, int64_t n_vocab, int32_t* seq, int32_t mask_id,
                             int32_t n_transfer, float threshold, int32_t* token, float* prob,
                             int32_t* n_committed, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DIFFUSE_MOE_H */
