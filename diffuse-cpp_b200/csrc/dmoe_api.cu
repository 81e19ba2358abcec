// dmoe_api.cu — host side of libdiffuse_moe: the C ABI of include/diffuse_moe.h.
//
// dmoe_create   validates the layer (src/diffuse-common.h:59-86,103-118 semantics), uploads the
//               weights once (library-owned device memory; Q8_0 repacked losslessly into an
//               int8 quant plane + fp32 scale plane so TMA can 128B-swizzle the quants), builds
//               the TMA descriptors of every weight tensor.
// dmoe_forward  enqueues the layer on one stream:
//               router logits -> routing -> scan / token tiles -> gather -> gate/up GEMM ->
//               down GEMM (src/diffuse-moe-graph.cpp:195-287).
// No CPU fallback: a missing device or a failed launch is reported, never worked around.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <memory>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <chrono>
#include <mutex>
#include <thread>
#include <string>
#include <vector>

#include "../../include/diffuse_moe.h"
#include "dmoe_internal.h"
#include "sm100.cuh"
#include "nccl_dyn.h"

using namespace dmoe;

namespace {

thread_local std::string g_last_error;

dmoe_status fail(dmoe_status st, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return st;
}

#define DMOE_CUDA(call)                                                                              \
  do {                                                                                               \
    cudaError_t e_ = (call);                                                                         \
    if (e_ != cudaSuccess) return fail(DMOE_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled get_encode_tiled() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  return fn;
}

// 2-D row-major tensor [outer][inner] of `dt` elements, row pitch `pitch_bytes`.
dmoe_status make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  PFN_encodeTiled enc = get_encode_tiled();
  if (!enc) return fail(DMOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {pitch_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): inner=%llu outer=%llu pitch=%llu box=%u,%u",
                (int)r, (unsigned long long)inner, (unsigned long long)outer, (unsigned long long)pitch_bytes,
                box_inner, box_outer);
  return DMOE_OK;
}

bool type_supported(int32_t t) { return t == DMOE_TYPE_F16 || t == DMOE_TYPE_Q8_0 || t == DMOE_TYPE_Q4_K; }

// A weight matrix family on the device: `nmat` matrices of rows x k, in the kernel layout.
struct DevWeight {
  int32_t type = -1;
  int64_t rows = 0;  // total rows (all experts)
  int64_t k = 0;
  void* q = nullptr;      // F16 / Q4_K bytes as in GGUF; Q8_0 int8 quant plane [rows][k]
  float* s = nullptr;     // Q8_0 fp32 scale plane [rows][k / 32]
  CUtensorMap tm_q;
  CUtensorMap tm_s;
};

dmoe_status upload_weight(DevWeight& w, int32_t type, const void* host, int64_t rows, int64_t k) {
  w.type = type;
  w.rows = rows;
  w.k = k;
  const size_t rs = row_size(type, k);
  if (rs == 0) return fail(DMOE_ERR_UNSUPPORTED, "row of %lld values is not a whole number of type-%d blocks",
                           (long long)k, type);
  if (type == DMOE_TYPE_Q8_0) {
    if (cudaMalloc(&w.q, (size_t)rows * k) != cudaSuccess) return fail(DMOE_ERR_OOM, "cudaMalloc q8_0 quants");
    if (cudaMalloc(&w.s, (size_t)rows * (k / 32) * 4) != cudaSuccess) return fail(DMOE_ERR_OOM, "cudaMalloc scales");
    // repack in chunks of rows: {f16 d; int8 q[32]} -> quant plane + fp32 scale plane (lossless)
    const int64_t chunk = std::max<int64_t>(1, (64ll << 20) / (int64_t)rs);
    std::vector<int8_t> qb;
    std::vector<float> sb;
    for (int64_t r0 = 0; r0 < rows; r0 += chunk) {
      const int64_t nr = std::min(chunk, rows - r0);
      qb.resize((size_t)nr * k);
      sb.resize((size_t)nr * (k / 32));
      const uint8_t* src = static_cast<const uint8_t*>(host) + (size_t)r0 * rs;
      for (int64_t r = 0; r < nr; ++r)
        for (int64_t b = 0; b < k / 32; ++b) {
          const uint8_t* blk = src + (size_t)r * rs + b * 34;
          sb[(size_t)r * (k / 32) + b] = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
          std::memcpy(&qb[(size_t)r * k + b * 32], blk + 2, 32);
        }
      DMOE_CUDA(cudaMemcpy(static_cast<int8_t*>(w.q) + (size_t)r0 * k, qb.data(), (size_t)nr * k,
                           cudaMemcpyHostToDevice));
      DMOE_CUDA(cudaMemcpy(w.s + (size_t)r0 * (k / 32), sb.data(), (size_t)nr * (k / 32) * 4, cudaMemcpyHostToDevice));
    }
    dmoe_status st = make_map(&w.tm_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.q, (uint64_t)k, (uint64_t)rows, (uint64_t)k,
                              128, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DMOE_OK) return st;
    return make_map(&w.tm_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.s, (uint64_t)(k / 32), (uint64_t)rows,
                    (uint64_t)(k / 32) * 4, 4, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (cudaMalloc(&w.q, (size_t)rows * rs) != cudaSuccess) return fail(DMOE_ERR_OOM, "cudaMalloc weights");
  DMOE_CUDA(cudaMemcpy(w.q, host, (size_t)rows * rs, cudaMemcpyHostToDevice));
  if (type == DMOE_TYPE_Q4_K)
    return make_map(&w.tm_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.q, (uint64_t)rs, (uint64_t)rows, (uint64_t)rs, 144, 128,
                    CU_TENSOR_MAP_SWIZZLE_NONE);
  return make_map(&w.tm_q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w.q, (uint64_t)k, (uint64_t)rows, (uint64_t)k * 2, 64,
                  128, CU_TENSOR_MAP_SWIZZLE_128B);
}

// TMA descriptors of a weight family already in device memory (the layouts upload_weight makes).
dmoe_status map_weight(DevWeight& w) {
  const size_t rs = row_size(w.type, w.k);
  if (w.type == DMOE_TYPE_Q8_0) {
    dmoe_status st = make_map(&w.tm_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.q, (uint64_t)w.k, (uint64_t)w.rows,
                              (uint64_t)w.k, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DMOE_OK) return st;
    return make_map(&w.tm_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.s, (uint64_t)(w.k / 32), (uint64_t)w.rows,
                    (uint64_t)(w.k / 32) * 4, 4, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (w.type == DMOE_TYPE_Q4_K)
    return make_map(&w.tm_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.q, (uint64_t)rs, (uint64_t)w.rows, (uint64_t)rs, 144, 128,
                    CU_TENSOR_MAP_SWIZZLE_NONE);
  return make_map(&w.tm_q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w.q, (uint64_t)w.k, (uint64_t)w.rows, (uint64_t)w.k * 2,
                  64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Bytes per row of the device layout: one plane (F16 / Q4_K GGUF rows, Q8_0 int8 quants) plus,
// for Q8_0, the fp32 scale plane.
size_t dev_row_bytes(const DevWeight& w) { return w.type == DMOE_TYPE_Q8_0 ? (size_t)w.k : row_size(w.type, w.k); }

void free_weight(DevWeight& w) {
  if (w.q) cudaFree(w.q);
  if (w.s) cudaFree(w.s);
  w.q = nullptr;
  w.s = nullptr;
}

template <class T>
dmoe_status grow(T*& p, size_t& cap, size_t need) {
  if (need <= cap && p) return DMOE_OK;
  if (p) cudaFree(p);
  p = nullptr;
  cap = 0;
  const size_t n = std::max<size_t>(need, 1);
  if (cudaMalloc(reinterpret_cast<void**>(&p), n * sizeof(T)) != cudaSuccess)
    return fail(DMOE_ERR_OOM, "cudaMalloc workspace (%zu bytes)", n * sizeof(T));
  cap = n;
  return DMOE_OK;
}

}  // namespace

void dmoe::set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }

namespace {
thread_local bool g_pdl_call = false;
}

void dmoe::set_pdl_for_call(bool on) {
  static const bool allowed = [] {
    const char* v = getenv("DMOE_PDL");
    return !(v && v[0] == '0');
  }();
  g_pdl_call = allowed && on;
}

bool dmoe::pdl_enabled() { return g_pdl_call; }

struct dmoe_layer {
  // shapes / hyper-parameters
  int64_t H = 0, I = 0, Is = 0, E = 0, K = 0, cap = 0, blk = 0;
  float scale = 1.0f;
  int32_t norm_topk = 1;
  int32_t etype = 0, stype = 0;
  bool has_shared = false, has_bias = false;
  int device = 0, sms = 148;
  cudaStream_t own_stream = nullptr;
  // host-buffer calls of many tokens: chunk copies overlap the compute (two copy streams, so the
  // two PCIe directions run at once), kMaxChunks events per direction
  static constexpr int kMaxChunks = 8;
  cudaStream_t h2d_stream = nullptr, d2h_stream = nullptr;
  cudaEvent_t ev_in[kMaxChunks] = {}, ev_done[kMaxChunks] = {}, ev_start = nullptr;
  // weights
  float* wr = nullptr;  // router weight transposed, [H][E]
  float* br = nullptr;
  DevWeight gate, up, down, sgate, sup, sdown;
  // workspace (grown, never shrunk)
  float* parts = nullptr; size_t parts_cap = 0;    // router logits, or their segment partials (split path)
  int32_t* arrivals = nullptr; size_t arrivals_cap = 0;  // split router: per-tile arrival counters
  int32_t* idx = nullptr; size_t idx_cap = 0;
  float* wts = nullptr; size_t wts_cap = 0;
  uint8_t* allowed = nullptr; size_t allowed_cap = 0;
  int32_t* ints = nullptr; size_t ints_cap = 0;  // counts[E] fill[E] off[E] n_tiles n_active
  TokTile* tiles = nullptr; size_t tiles_cap = 0;
  __half* xg = nullptr; size_t xg_cap = 0;
  __half* hbuf = nullptr; size_t hbuf_cap = 0;
  float* gu = nullptr; size_t gu_cap = 0;
  int32_t* pair_tok = nullptr; size_t pair_tok_cap = 0;
  float* pair_w = nullptr; size_t pair_w_cap = 0;
  int32_t* pair_row = nullptr; size_t pair_row_cap = 0;
  float* ybuf = nullptr; size_t ybuf_cap = 0;
  int32_t* tt_done = nullptr; size_t tt_done_cap = 0;  // fused GEMM: per token tile completion counters
  float* xdev = nullptr; size_t xdev_cap = 0;
  float* odev = nullptr; size_t odev_cap = 0;
  uint32_t* err = nullptr;
  // expert parallelism: this rank owns experts [rank * e_local, (rank + 1) * e_local)
  int world = 1, rank = 0;
  int64_t e_local = 0;
  int timeout_ms = 60000;
  ncclComm_t comm = nullptr;
  bool broken = false;  // a collective failed or timed out; the communicator was aborted
  uint32_t* ep_mask = nullptr; size_t ep_mask_cap = 0;
  int32_t* ep_pos = nullptr; size_t ep_pos_cap = 0;
  int32_t* ep_cnt = nullptr; size_t ep_cnt_cap = 0;  // [send counts W][recv counts W]
  __half* ep_xs = nullptr; size_t ep_xs_cap = 0;     // rows sent, [S][H]
  int32_t* ep_ms = nullptr; size_t ep_ms_cap = 0;    // slot lists sent, [S][2 top_k]
  __half* ep_xr = nullptr; size_t ep_xr_cap = 0;     // rows received, [R][H]
  int32_t* ep_mr = nullptr; size_t ep_mr_cap = 0;    // slot lists received
  float* ep_part = nullptr; size_t ep_part_cap = 0;  // partial rows computed here for others, [R][H]
  float* ep_back = nullptr; size_t ep_back_cap = 0;  // partial rows returned to this rank, [S][H]
  int32_t* ep_host = nullptr;                        // pinned: the 2 W ep_chunks counts
  // chunked exchange: ep_chunks pipeline chunks per forward (DMOE_EP_CHUNKS, 1..kMaxChunks, the
  // same on every rank), NCCL groups on comm_stream, gemm_sm_reserve SMs left to NCCL's kernels
  int ep_chunks = 1;
  int gemm_sm_reserve = 0;
  // hot-expert replicas (dmoe_replicate_experts): n_hot experts held by every rank after its own
  // e_local (local expert e_local + j = global expert hot_ids[j]); hot_slot [E] maps a global
  // expert to j or -1; ep_load [E] is the last forward's (token, slot) count per expert here
  int n_hot = 0;
  std::vector<int32_t> hot_ids;
  int32_t* hot_slot = nullptr;
  int32_t* ep_load = nullptr;
  int32_t* ep_load_sum = nullptr;
  cudaStream_t comm_stream = nullptr;
  cudaEvent_t ev_pack[kMaxChunks] = {}, ev_disp[kMaxChunks] = {}, ev_exp[kMaxChunks] = {}, ev_comb[kMaxChunks] = {};
  // statistics
  dmoe_stats stats{};
  int32_t* host_counters = nullptr;  // pinned: n_tiles, n_active
  cudaEvent_t ev[6] = {};
  bool profiled = false;
  cudaStream_t last_stream = nullptr;  // stream of the last forward (NULL = default stream)
};

namespace {

dmoe_status validate(const dmoe_layer_desc* d) {
  if (!d) return fail(DMOE_ERR_INVALID_ARG, "null layer descriptor");
  if (d->n_embd <= 0 || d->n_ff_exp <= 0 || d->n_expert <= 0 || d->n_expert_used <= 0 || d->n_ff_shexp < 0)
    return fail(DMOE_ERR_INVALID_ARG, "non-positive layer dimension");
  if (d->n_expert_used > 16 || d->n_expert_used > d->n_expert)
    return fail(DMOE_ERR_INVALID_ARG, "n_expert_used must be <= min(16, n_expert)");
  if (d->n_expert > 1024 || d->n_expert % 4) return fail(DMOE_ERR_UNSUPPORTED, "n_expert must be a multiple of 4, <= 1024");
  if (d->expert_capacity < 0 || d->moe_block_size < 0) return fail(DMOE_ERR_INVALID_ARG, "negative capacity/block");
  const int64_t tpb = d->moe_block_size > 1 ? std::max<int64_t>(d->moe_block_size, 32) : 32;
  if (route_smem_bytes(tpb, d->n_expert) > kRouteSmemMax)
    return fail(DMOE_ERR_UNSUPPORTED, "moe_block_size x n_expert too large for the routing kernel");
  if (!type_supported(d->expert_type)) return fail(DMOE_ERR_UNSUPPORTED, "expert weight type %d", d->expert_type);
  if (d->n_ff_shexp > 0 && !type_supported(d->shared_type))
    return fail(DMOE_ERR_UNSUPPORTED, "shared weight type %d", d->shared_type);
  if (!d->w_gate || !d->w_up || !d->w_down || !d->w_router) return fail(DMOE_ERR_INVALID_ARG, "null weight pointer");
  if (d->n_ff_shexp > 0 && (!d->sw_gate || !d->sw_up || !d->sw_down))
    return fail(DMOE_ERR_INVALID_ARG, "null shared-expert weight pointer");
  auto kmul = [](int32_t t) { return t == DMOE_TYPE_Q4_K ? 256 : 128; };
  const int64_t H = d->n_embd, I = d->n_ff_exp, Is = d->n_ff_shexp;
  if (H % kRouterSeg) return fail(DMOE_ERR_UNSUPPORTED, "n_embd must be a multiple of %d (router segments)", kRouterSeg);
  if (H % 128 || H % kmul(d->expert_type) || I % kmul(d->expert_type))
    return fail(DMOE_ERR_UNSUPPORTED, "n_embd / n_ff_exp must be multiples of %d for type %d", kmul(d->expert_type),
                d->expert_type);
  if (Is > 0 && (H % kmul(d->shared_type) || Is % kmul(d->shared_type)))
    return fail(DMOE_ERR_UNSUPPORTED, "n_ff_shexp must be a multiple of %d", kmul(d->shared_type));
  return DMOE_OK;
}

// Tuning overrides (DMOE_NT = 32 / 64 / 128, DMOE_KSPLIT_GU / DMOE_KSPLIT_DN = 1 / 2 / 4 / 8,
// DMOE_ROUTER_SPLIT = 0 whole-K / 1 split 32-token tiles / 2 split 128-token tiles / 3 whole-K
// 112-token tiles,
// DMOE_COMBINE_MIN = tokens); unset or invalid values keep the
// automatic choice.
int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  if (!v || !*v) return dflt;
  return atoi(v);
}

int pick_nt(const dmoe_layer* L, int64_t n) {
  const int forced = env_int("DMOE_NT", 0);
  if (forced == 32 || forced == 64 || forced == 128) return forced;
  const bool use_block = L->blk > 1 && L->cap > 0 && L->cap < L->E && n % L->blk == 0;
  // pairs computed here: n * top_k on one GPU, and the same on average per rank with expert
  // parallelism (every rank sends n * top_k (token, slot) pairs, spread over the ranks)
  const int64_t pairs = n * L->K;
  int64_t active = std::min<int64_t>(L->world > 1 ? L->e_local : L->E, pairs);
  if (use_block && L->world == 1) active = std::min<int64_t>(active, L->cap * (n / L->blk));
  // weights are streamed once per token tile: size the tile for the busiest expert, whose
  // count is at most the number of tokens that can reach it and is estimated as 3x the mean + 8
  const double avg = active > 0 ? (double)pairs / (double)active : 0.0;
  const double busiest = std::min((double)n * L->world, 3.0 * avg + 8.0);
  // measured on B200 (c3): N = 64 tiles run at the full tensor rate (32 cycles per MMA) and keep
  // double-buffered accumulators, so 128 only pays once the average expert has > 128 tokens
  if (busiest <= 32.0) return 32;
  if (avg <= 128.0) return 64;
  return 128;
}

// Split-K factor of an expert GEMM. Measured on B200: the per-tile epilogue and pipeline refill
// cost more than the wave quantisation they remove, at every block count, so split-K runs only
// when forced (DMOE_KSPLIT_GU / DMOE_KSPLIT_DN).
int pick_ksplit(int64_t tiles_est, int sms, std::initializer_list<int> kstages) {
  (void)tiles_est;
  (void)sms;
  (void)kstages;
  return 1;
}

// CTA-pair GEMM tiles (256 output rows per tile, each activation tile loaded half by each CTA of
// a two-SM cluster): quantised weights at NT = 128, every expert matrix a multiple of 256 rows.
// Measured on B200 (c3, 8192 tokens): gate/up 1434 -> 1218 us with pairs, down 997 -> 1077 us
// (its single-matrix tiles already double-buffer the accumulators), so gate/up only by default.
// DMOE_PAIR = 0: off; 1: gate/up; 2: gate/up and down.
bool use_pair(const dmoe_layer* L, int nt, int mode) {
  const int v = env_int("DMOE_PAIR", 1);
  if (v <= 0 || (mode == MODE_DOWN && v < 2)) return false;
  const bool quant = L->etype != DMOE_TYPE_F16 && (!L->has_shared || L->stype != DMOE_TYPE_F16);
  const bool rows256 = L->I % 256 == 0 && L->H % 256 == 0 && (!L->has_shared || L->Is % 256 == 0);
  return quant && rows256 && gemm_pair_ok(L->etype, mode, nt);
}

// n_out_rows / rows_per_tile output tiles per expert (gate/up tiles cover 128 rows of each of the
// two matrices, down tiles 256 rows of the one)
void fill_group(GemmGroup& g, const DevWeight& w, int32_t type, int64_t rows_per_exp, int64_t n_out_rows,
                int64_t rows_per_tile = kMTile) {
  g.n_mt = (int32_t)(n_out_rows / rows_per_tile);
  g.k_stages = (int32_t)(w.k / gemm_stage_k(type));
  g.rows_per_exp = (int32_t)rows_per_exp;
  g.present = 1;
}


// ------------------------------------------------------------------------------------------
// expert stage: gate/up GEMM (+ SwiGLU) and down GEMM over the gathered layout (rows [0, n_sh)
// shared expert, then routed pairs), src/diffuse-moe-graph.cpp:264-286
// ------------------------------------------------------------------------------------------
// out_sh: shared rows' output [n_sh][H]; out_rt: routed rows' reduction target (pair_tok[r]
// indexes it), rt_rows of it zeroed here when it is not out_sh. combine = deterministic path
// (single GPU only): routed rows stored to ybuf, then summed per token in slot order.
dmoe_status run_experts(dmoe_layer* L, cudaStream_t st, int64_t n_sh, int64_t rows, int nt, int32_t* n_tiles,
                        float* out_sh, float* out_rt, int64_t rt_rows, bool combine, bool out_sh_zeroed, bool prof,
                        int& kernels, int groups = 3) {
  // groups: bit 0 the shared expert (rows [0, n_sh)), bit 1 the routed experts (the tile list)
  const bool sh = L->has_shared && (groups & 1);
  const bool rt = (groups & 2) != 0;
  const int64_t H = L->H, K = L->K;
  const int64_t Imax = std::max(L->I, L->Is);
  const int64_t E_here = L->world > 1 ? L->e_local + L->n_hot : L->E;  // owned experts, then replicas
  dmoe_status s;
  const bool pair_gu = use_pair(L, nt, MODE_GATEUP), pair_dn = use_pair(L, nt, MODE_DOWN);
  // activation tiles: NT token rows, or each pair CTA's half of them
  CUtensorMap tm_x, tm_h;
  if ((s = make_map(&tm_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, L->xg, (uint64_t)H, (uint64_t)rows, (uint64_t)H * 2, 64,
                    (uint32_t)(pair_gu ? nt / 2 : nt), CU_TENSOR_MAP_SWIZZLE_128B)) != DMOE_OK)
    return s;
  if ((s = make_map(&tm_h, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, L->hbuf, (uint64_t)Imax, (uint64_t)rows,
                    (uint64_t)Imax * 2, 64, (uint32_t)(pair_dn ? nt / 2 : nt), CU_TENSOR_MAP_SWIZZLE_128B)) != DMOE_OK)
    return s;
  const int64_t pairs = rows - n_sh;
  const int64_t tt_est = std::min<int64_t>(E_here, pairs) + pairs / nt;
  const int64_t sh_tt = sh ? (n_sh + nt - 1) / nt : 0;
  const bool same_type = !sh || L->stype == L->etype;
  const int gu_stage_r = gemm_stage_k(L->etype), gu_stage_s = gemm_stage_k(L->stype);
  const int64_t gu_tiles = tt_est * (L->I / kMTile) + sh_tt * (L->Is / kMTile);
  int ks_gu = pick_ksplit(gu_tiles, L->sms,
                          {(int)(H / gu_stage_r), sh ? (int)(H / gu_stage_s) : (int)(H / gu_stage_r)});
  if ((size_t)rows * 2 * Imax * 4 > (256ull << 20)) ks_gu = 1;
  const int64_t dn_tiles = (tt_est + sh_tt) * (H / kMTile);
  int ks_dn = pick_ksplit(dn_tiles, L->sms,
                          {(int)(L->I / gu_stage_r), sh ? (int)(L->Is / gu_stage_s) : (int)(L->I / gu_stage_r)});
  {
    const int f_gu = env_int("DMOE_KSPLIT_GU", 0), f_dn = env_int("DMOE_KSPLIT_DN", 0);
    auto divides = [&](int ks, int64_t k_r, int64_t k_s) {
      return ks >= 1 && ks <= 8 && (ks & (ks - 1)) == 0 && k_r % ks == 0 && k_s % ks == 0;
    };
    const int64_t gr = H / gu_stage_r, gs = sh ? H / gu_stage_s : gr;
    const int64_t dr = L->I / gu_stage_r, ds = sh ? L->Is / gu_stage_s : dr;
    if (divides(f_gu, gr, gs) && (size_t)rows * 2 * Imax * 4 <= (256ull << 20)) ks_gu = f_gu;
    if (divides(f_dn, dr, ds)) ks_dn = f_dn;
  }
  if (ks_gu > 1) {
    if ((s = grow(L->gu, L->gu_cap, (size_t)rows * 2 * Imax)) != DMOE_OK) return s;
    DMOE_CUDA(cudaMemsetAsync(L->gu, 0, (size_t)rows * 2 * Imax * 4, st));
  }
  GemmParams gp;
  std::memset(&gp, 0, sizeof(gp));
  gp.tm_b = tm_x;
  gp.tiles = L->tiles;
  gp.n_tiles = n_tiles;
  gp.n_shared_tt = (int32_t)sh_tt;
  gp.ksplit = ks_gu;
  gp.n_tokens = n_sh;
  gp.hbuf = L->hbuf;
  gp.h_ld = Imax;
  gp.h_quad_swap = (L->stype == DMOE_TYPE_Q4_K ? 1 : 0) | (L->etype == DMOE_TYPE_Q4_K ? 2 : 0);
  gp.gu_acc = ks_gu > 1 ? L->gu : nullptr;
  gp.gu_half = Imax;
  gp.err = L->err;
  gp.rows_total = rows;
  gp.n_experts = (int32_t)E_here;
  // routed tiles index L->tiles and tt_done[sh_tt + tile]
  gp.tiles_cap = (int32_t)std::min<int64_t>((int64_t)L->tiles_cap, (int64_t)L->tt_done_cap - sh_tt);
  if (sh) {
    gp.tm_w[0][0] = L->sgate.tm_q;
    gp.tm_w[0][1] = L->sup.tm_q;
    gp.tm_s[0][0] = L->sgate.tm_s;
    gp.tm_s[0][1] = L->sup.tm_s;
    fill_group(gp.grp[0], L->sgate, L->stype, L->Is, L->Is, gemm_out_rows(MODE_GATEUP, nt, pair_gu));
  }
  gp.tm_w[1][0] = L->gate.tm_q;
  gp.tm_w[1][1] = L->up.tm_q;
  gp.tm_s[1][0] = L->gate.tm_s;
  gp.tm_s[1][1] = L->up.tm_s;
  fill_group(gp.grp[1], L->gate, L->etype, L->I, L->I, gemm_out_rows(MODE_GATEUP, nt, pair_gu));
  gp.grp[1].present = rt ? 1 : 0;
  // persistent grid; with the chunked expert-parallel exchange a few SMs stay free for NCCL
  const int grid = L->sms - L->gemm_sm_reserve;
  // dequant warpgroups per CTA: 4 (or the most the TMEM ring allows) on 32-64 token tiles,
  // measured 2-3 % faster than 2 at 1-8 blocks; 2 on 128-token tiles, where each warpgroup then
  // alternates between two A-ring slots instead of waiting on one (B200, c3 at 8192 tokens:
  // gate/up 1371 -> 1287 us, down 1068 -> 1027 us, against 4)
  const int ndq = env_int("DMOE_NDQ", nt >= 128 ? 2 : 4);
  // One launch for both GEMMs at small N (the persistent kernel runs all gate/up tiles, then the
  // down tiles, each as soon as its token tile's h rows are written): saves a launch, its ramp
  // and its tail imbalance. Measured on B200 (c3): 1 block 107 -> 95 us for the two GEMMs, even
  // at 8 blocks, 70 us slower at 64 blocks; so only up to 128 tokens (DMOE_FUSED=0/1 overrides).
  const int f_env = env_int("DMOE_FUSED", -1);
  const bool fused = same_type && ks_gu == 1 && ks_dn == 1 && nt <= 64 &&
                     (f_env == 1 || (f_env != 0 && n_sh <= 128));
  gp.tt_done = L->tt_done;
  // experts average more than one token tile: their weight tiles are re-read, keep them in L2
  {
    const int wk = env_int("DMOE_WKEEP", -1);
    gp.w_keep = wk >= 0 ? (wk != 0) : (pairs >= (int64_t)nt * std::min<int64_t>(E_here, pairs) ? 1 : 0);
  }
  if (fused) {
    // launched below, once the down operands are set
  } else if (same_type) {
    DMOE_CUDA(launch_moe_gemm(L->etype, MODE_GATEUP, nt, ndq, pair_gu, gp, grid, st));
    ++kernels;
  } else {
    GemmParams g0 = gp, g1 = gp;
    g0.grp[1].present = 0;
    g1.grp[0].present = 0;
    DMOE_CUDA(launch_moe_gemm(L->stype, MODE_GATEUP, nt, ndq, pair_gu, g0, grid, st));
    DMOE_CUDA(launch_moe_gemm(L->etype, MODE_GATEUP, nt, ndq, pair_gu, g1, grid, st));
    kernels += 2;
  }
  if (ks_gu > 1) {
    DMOE_CUDA(launch_swiglu_finish(L->gu, Imax, rows, n_sh, (int)L->Is, (int)L->I, L->hbuf, Imax,
                                   L->stype == DMOE_TYPE_Q4_K, L->etype == DMOE_TYPE_Q4_K, st));
    ++kernels;
  }
  if (prof) DMOE_CUDA(cudaEventRecord(L->ev[3], st));

  // ---- down GEMM (+ gate weights, slot sum, shared expert)
  // Deterministic path: routed rows are stored to y and summed per token in slot order by
  // combine_kernel, the shared rows stored straight into out. Otherwise the epilogue reduces
  // every row into zeroed outputs with fp32 atomics (measured faster at every size: the y
  // round trip costs more than the reductions).
  combine = combine && ks_dn == 1 && out_rt == out_sh;
  if (combine) {
    if ((s = grow(L->ybuf, L->ybuf_cap, (size_t)pairs * H)) != DMOE_OK) return s;
  }
  if ((!combine || !sh) && !out_sh_zeroed) DMOE_CUDA(cudaMemsetAsync(out_sh, 0, (size_t)n_sh * H * 4, st));
  if (out_rt != out_sh && rt_rows > 0) DMOE_CUDA(cudaMemsetAsync(out_rt, 0, (size_t)rt_rows * H * 4, st));
  GemmParams dp = gp;
  dp.tm_b = tm_h;
  dp.ksplit = ks_dn;
  dp.gu_acc = nullptr;
  dp.out = out_sh;
  dp.out_ld = H;
  dp.out_routed = out_rt;
  dp.y = combine ? L->ybuf : nullptr;
  dp.y_ld = H;
  dp.pair_tok = L->pair_tok;
  dp.pair_w = L->pair_w;
  std::memset(&dp.grp, 0, sizeof(dp.grp));
  if (sh) {
    dp.tm_w[0][0] = L->sdown.tm_q;
    dp.tm_s[0][0] = L->sdown.tm_s;
    fill_group(dp.grp[0], L->sdown, L->stype, L->H, L->H, gemm_out_rows(MODE_DOWN, nt, pair_dn));
  }
  dp.tm_w[1][0] = L->down.tm_q;
  dp.tm_s[1][0] = L->down.tm_s;
  fill_group(dp.grp[1], L->down, L->etype, L->H, L->H, gemm_out_rows(MODE_DOWN, nt, pair_dn));
  dp.grp[1].present = rt ? 1 : 0;
  // Down GEMM with resident activation tiles (BRES, off by default): each CTA holds 64 token rows
  // of h (all of K <= 1024, 128 KB) in shared memory and runs every 256-row m-tile of the down
  // matrix against them, instead of re-reading the activation tile from L2 for each m-tile.
  // DMOE_BRES = 1: at NT = 128 as CTA pairs (each CTA keeps its 64-row half; one 128-row block per
  // CTA leaves room for five 18 KB weight stages); 2: also single CTAs on 64-token tiles (128-row
  // list tiles as two halves, two weight stages). Measured on B200 (c3, ncu at 4096 tokens): the
  // L2-to-SM reads fall from 4.40 to 1.18 GB per launch, but the launch takes 706 against 566 us
  // (8192 tokens: 1.26 against ~1.0 ms; 2048 tokens single-CTA: 0.43 against 0.32 ms): the down
  // GEMM is bound by its dequant issue rate (issue 55-57 % active, tensor pipe 34-38 %), not by
  // L2, and the unit boundaries drain the pipeline.
  const bool quant_dn = L->etype != DMOE_TYPE_F16;
  const int bres_env = env_int("DMOE_BRES", 0);
  const bool bres_ok = !fused && same_type && quant_dn && ks_dn == 1 &&
                       std::max(L->I, sh ? L->Is : 0) <= kBresK;
  const bool bres_pair = bres_ok && bres_env >= 1 && nt == 2 * kBresNT && use_pair(L, nt, MODE_GATEUP);
  const bool bres = bres_pair || (bres_ok && bres_env >= 2 && (nt == kBresNT || nt == 2 * kBresNT));
  if (bres) {
    CUtensorMap tm_h64;
    if ((s = make_map(&tm_h64, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, L->hbuf, (uint64_t)Imax, (uint64_t)rows,
                      (uint64_t)Imax * 2, 64, (uint32_t)kBresNT, CU_TENSOR_MAP_SWIZZLE_128B)) != DMOE_OK)
      return s;
    GemmParams bp = dp;
    bp.tm_b = tm_h64;
    const int bnt = bres_pair ? 2 * kBresNT : kBresNT;  // token rows per tile of the launch
    bp.tile_div = nt / bnt;
    bp.n_shared_tt = sh ? (int32_t)((n_sh + bnt - 1) / bnt) : 0;
    fill_group(bp.grp[1], L->down, L->etype, L->H, L->H, gemm_out_rows(MODE_DOWN, bnt, bres_pair));
    bp.grp[1].present = rt ? 1 : 0;
    if (sh) fill_group(bp.grp[0], L->sdown, L->stype, L->H, L->H, gemm_out_rows(MODE_DOWN, bnt, bres_pair));
    // m-chunks per token tile: whole token tiles while they give every SM (pair) about three units
    const int n_mt = bp.grp[1].n_mt;
    const int64_t units = bp.n_shared_tt + tt_est * bp.tile_div;
    const int64_t workers = bres_pair ? L->sms / 2 : L->sms;
    int chunks = 1;
    while (chunks < 4 && n_mt % (2 * chunks) == 0 && units * chunks < 3 * workers) chunks *= 2;
    if (const int fc = env_int("DMOE_BRES_CHUNKS", 0); fc == 1 || fc == 2 || fc == 4 || fc == 8)
      if (n_mt % fc == 0) chunks = fc;
    bp.bres_chunks = chunks;
    DMOE_CUDA(launch_moe_gemm_bres(L->etype, bres_pair, ndq, bp, grid, st));
    ++kernels;
  } else if (fused) {
    GemmParams fp = gp;  // gate/up operands and tiles ...
    fp.tm_b_dn = dp.tm_b;  // ... then the down phase's
    fp.tm_w_dn[0] = dp.tm_w[0][0];
    fp.tm_w_dn[1] = dp.tm_w[1][0];
    fp.tm_s_dn[0] = dp.tm_s[0][0];
    fp.tm_s_dn[1] = dp.tm_s[1][0];
    fp.grp_dn[0] = dp.grp[0];
    fp.grp_dn[1] = dp.grp[1];
    fp.out = dp.out;
    fp.out_ld = dp.out_ld;
    fp.out_routed = dp.out_routed;
    fp.y = dp.y;
    fp.y_ld = dp.y_ld;
    fp.pair_tok = dp.pair_tok;
    fp.pair_w = dp.pair_w;
    DMOE_CUDA(launch_moe_gemm(L->etype, MODE_FUSED, nt, ndq, false, fp, grid, st));
    ++kernels;
  } else if (same_type) {
    DMOE_CUDA(launch_moe_gemm(L->etype, MODE_DOWN, nt, ndq, pair_dn, dp, grid, st));
    ++kernels;
  } else {
    GemmParams d0 = dp, d1 = dp;
    d0.grp[1].present = 0;
    d1.grp[0].present = 0;
    DMOE_CUDA(launch_moe_gemm(L->stype, MODE_DOWN, nt, ndq, pair_dn, d0, grid, st));
    DMOE_CUDA(launch_moe_gemm(L->etype, MODE_DOWN, nt, ndq, pair_dn, d1, grid, st));
    kernels += 2;
  }
  if (combine) {
    DMOE_CUDA(launch_combine(L->ybuf, H, n_sh, L->pair_row, (int)K, out_sh, H, sh ? 1 : 0, st));
    ++kernels;
  }
  L->stats.token_tile = nt;
  L->stats.ksplit_gateup = ks_gu;
  L->stats.ksplit_down = ks_dn;
  L->stats.fused_gemm = fused ? 1 : 0;
  return DMOE_OK;
}

dmoe_status single_gpu_experts(dmoe_layer* L, cudaStream_t st, const float* xd, int64_t n, const int32_t* idx,
                               const float* w, const int32_t* counts, float* od, uint32_t flags, int& kernels) {
  const int64_t H = L->H, E = L->E, K = L->K;
  const int64_t rows = n * (1 + K);  // shared segment [0, n) + routed pairs
  const int64_t Imax = std::max(L->I, L->Is);
  const bool prof = flags & DMOE_F_PROFILE;
  const int nt = pick_nt(L, n);
  int32_t* fill = L->ints + E;
  int32_t* off = L->ints + 2 * E;
  int32_t* n_tiles = L->ints + 3 * E;
  int32_t* n_active = n_tiles + 1;
  dmoe_status s;
  // ---- dispatch: offsets, token tiles, gathered fp16 rows
  if ((s = grow(L->tiles, L->tiles_cap, (size_t)(n * K / 32 + E + 2))) != DMOE_OK) return s;
  if ((s = grow(L->xg, L->xg_cap, (size_t)rows * H)) != DMOE_OK) return s;
  if ((s = grow(L->hbuf, L->hbuf_cap, (size_t)rows * Imax)) != DMOE_OK) return s;
  if ((s = grow(L->pair_tok, L->pair_tok_cap, (size_t)rows)) != DMOE_OK) return s;
  if ((s = grow(L->pair_w, L->pair_w_cap, (size_t)rows)) != DMOE_OK) return s;
  if ((s = grow(L->pair_row, L->pair_row_cap, (size_t)n * K)) != DMOE_OK) return s;
  if ((s = grow(L->tt_done, L->tt_done_cap, (size_t)(n * K / 32 + E + 2 + (n + 31) / 32))) != DMOE_OK) return s;
  DMOE_CUDA(launch_scan_tiles(counts, (int)E, n, nt, off, fill, L->tiles, n_tiles, n_active, L->tt_done,
                              L->has_shared ? (int)((n + nt - 1) / nt) : 0, st));
  const bool det = (flags & DMOE_F_DETERMINISTIC) || n >= env_int("DMOE_COMBINE_MIN", 1 << 30);
  // the atomic path's output is zeroed by the gather kernel, row by row (no memset in the chain)
  DMOE_CUDA(launch_gather(xd, n, (int)H, (int)K, idx, w, off, fill, L->xg, L->pair_tok, L->pair_w, L->pair_row,
                          L->stype == DMOE_TYPE_Q4_K, L->etype == DMOE_TYPE_Q4_K, L->has_shared ? 1 : 0,
                          det ? nullptr : od, st));
  kernels += 2;
  if (prof) DMOE_CUDA(cudaEventRecord(L->ev[2], st));
  if ((s = run_experts(L, st, n, rows, nt, n_tiles, od, od, 0, det, !det, prof, kernels)) != DMOE_OK) return s;
  if (prof) DMOE_CUDA(cudaEventRecord(L->ev[4], st));
  DMOE_CUDA(cudaMemcpyAsync(L->host_counters, n_tiles, 8, cudaMemcpyDeviceToHost, st));
  return DMOE_OK;
}

// ---------------------------------------------------------------------------------------------
// expert parallelism (NCCL over NVLink; one process per GPU)
// ---------------------------------------------------------------------------------------------
const char* nccl_err(ncclResult_t r) { return nccl().GetErrorString ? nccl().GetErrorString(r) : "?"; }

void ep_abort(dmoe_layer* L) {
  if (L->comm) nccl().CommAbort(L->comm);
  L->comm = nullptr;
  L->broken = true;
}

// Settles a call on the non-blocking communicator: polls its state until the call completed,
// failed, or the layer's deadline passed (then the communicator is aborted).
dmoe_status nccl_settle(dmoe_layer* L, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return DMOE_OK;
  if (r != ncclInProgress) {
    ep_abort(L);
    return fail(DMOE_ERR_NCCL, "%s: %s", what, nccl_err(r));
  }
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    ncclResult_t a = ncclInProgress;
    nccl().CommGetAsyncError(L->comm, &a);
    if (a == ncclSuccess) return DMOE_OK;
    if (a != ncclInProgress) {
      ep_abort(L);
      return fail(DMOE_ERR_NCCL, "%s: %s", what, nccl_err(a));
    }
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(L->timeout_ms)) {
      ep_abort(L);
      return fail(DMOE_ERR_TIMEOUT, "%s did not complete within %d ms; communicator aborted", what, L->timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

// Waits for `st` to drain while watching the communicator; the deadline aborts it.
dmoe_status ep_wait(dmoe_layer* L, cudaStream_t st, const char* what) {
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    const cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) return DMOE_OK;
    if (q != cudaErrorNotReady) return fail(DMOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(q));
    if (L->comm) {
      ncclResult_t a = ncclSuccess;
      nccl().CommGetAsyncError(L->comm, &a);
      if (a != ncclSuccess && a != ncclInProgress) {
        ep_abort(L);
        return fail(DMOE_ERR_NCCL, "%s: %s", what, nccl_err(a));
      }
    }
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(L->timeout_ms)) {
      ep_abort(L);
      return fail(DMOE_ERR_TIMEOUT, "%s did not complete within %d ms; communicator aborted", what, L->timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

#define DMOE_NCCL(call, what)                                               \
  do {                                                                      \
    dmoe_status s_ = nccl_settle(L, (call), what);                          \
    if (s_ != DMOE_OK) return s_;                                           \
  } while (0)

// Expert-parallel experts of one forward, pipelined over `ep_chunks` chunks of this rank's
// tokens (src/diffuse-moe-graph.cpp:264-286 across ranks). Routing is already done for every
// token, so chunk boundaries need not be routing blocks.
//   1. per chunk: plan (per-token destination mask, row positions, counts per destination);
//   2. one count exchange for all chunks (grouped send / recv of `chunks` ints per peer), read
//      on the host: the forward's only host synchronisation (it sizes the transfers);
//   3. per chunk c, ordered by events:
//        compute stream  pack(c) ............ gather + GEMMs(c) ............... final(c) (at the end)
//        comm stream              dispatch(c) ..................... combine(c)
//      dispatch(c + 1) and combine(c - 1) run on the comm stream while the GEMMs of chunk c run
//      on the compute stream; the GEMM grid leaves gemm_sm_reserve SMs to NCCL's kernels.
// Every rank takes the same NCCL steps in the same order: all dispatch groups, then the combine
// groups in chunk order.
dmoe_status ep_experts(dmoe_layer* L, cudaStream_t st, const float* xd, int64_t n, const int32_t* idx,
                       const float* w, float* od, uint32_t flags, int& kernels) {
  const NcclApi& api = nccl();
  const int W = L->world;
  const int C = L->ep_chunks;
  const int64_t H = L->H, K = L->K, El = L->e_local;
  const int64_t Eh = El + L->n_hot;  // local experts: owned, then replicas
  const int32_t* hot = L->n_hot ? L->hot_slot : nullptr;
  const int64_t Imax = std::max(L->I, L->Is);
  const bool prof = flags & DMOE_F_PROFILE;
  if (flags & DMOE_F_DETERMINISTIC)
    return fail(DMOE_ERR_UNSUPPORTED, "DMOE_F_DETERMINISTIC is single-GPU only");
  dmoe_status s;
  cudaStream_t cs = L->comm_stream;
  // chunk c covers tokens [t0[c], t0[c] + nc[c]); near-equal, possibly empty
  int64_t t0[dmoe_layer::kMaxChunks], nc[dmoe_layer::kMaxChunks];
  for (int c = 0; c < C; ++c) {
    t0[c] = n * c / C;
    nc[c] = n * (c + 1) / C - t0[c];
  }
  if ((s = grow(L->ep_mask, L->ep_mask_cap, (size_t)std::max<int64_t>(n, 1))) != DMOE_OK) return s;
  if ((s = grow(L->ep_pos, L->ep_pos_cap, (size_t)std::max<int64_t>(W * n, 1))) != DMOE_OK) return s;
  if ((s = grow(L->ep_cnt, L->ep_cnt_cap, (size_t)2 * W * C)) != DMOE_OK) return s;
  int32_t* cnt_send = L->ep_cnt;          // [W][C]: rows for destination p from chunk c at p * C + c
  int32_t* cnt_recv = L->ep_cnt + W * C;  // [W][C]: rows source p sends from its chunk c
  // ---- 1. plans; chunk c's positions are pos + W * t0[c], laid out [W][nc[c]]
  for (int c = 0; c < C; ++c) {
    DMOE_CUDA(launch_ep_plan(idx + t0[c] * K, nc[c], (int)K, (int)El, hot, L->rank, W, L->ep_mask + t0[c],
                             L->ep_pos + W * t0[c], cnt_send + c, C, st));
    kernels += nc[c] > 0 ? 2 : 1;
  }
  // ---- 2. count exchange, one host read
  DMOE_NCCL(api.GroupStart(), "ncclGroupStart");
  for (int p = 0; p < W; ++p) {
    DMOE_NCCL(api.Send(cnt_send + p * C, (size_t)C, ncclInt32, p, L->comm, st), "ncclSend(counts)");
    DMOE_NCCL(api.Recv(cnt_recv + p * C, (size_t)C, ncclInt32, p, L->comm, st), "ncclRecv(counts)");
  }
  DMOE_NCCL(api.GroupEnd(), "count exchange");
  DMOE_CUDA(cudaMemcpyAsync(L->ep_host, L->ep_cnt, sizeof(int32_t) * 2 * W * C, cudaMemcpyDeviceToHost, st));
  if ((s = ep_wait(L, st, "count exchange")) != DMOE_OK) return s;
  // send / receive layouts: chunk-major, then peer
  RankOffsets soff[dmoe_layer::kMaxChunks], roff[dmoe_layer::kMaxChunks];
  int64_t Rc[dmoe_layer::kMaxChunks];
  int64_t S = 0, R = 0, Rmax = 0;
  for (int c = 0; c < C; ++c) {
    const int64_t r0 = R;
    for (int p = 0; p < W; ++p) {
      soff[c].v[p] = (int32_t)S;
      roff[c].v[p] = (int32_t)R;
      S += L->ep_host[p * C + c];
      R += L->ep_host[W * C + p * C + c];
    }
    Rc[c] = R - r0;
    Rmax = std::max(Rmax, Rc[c]);
  }
  const int64_t nmax = (n + C - 1) / C + 1;
  const int64_t Pmax = Rmax * K;         // upper bound of a chunk's local (row, expert) pairs
  const int64_t rows_max = nmax + Pmax;  // gathered layout of a chunk: shared rows, then pairs
  if ((s = grow(L->ep_xs, L->ep_xs_cap, (size_t)std::max<int64_t>(S, 1) * H)) != DMOE_OK) return s;
  if ((s = grow(L->ep_ms, L->ep_ms_cap, (size_t)std::max<int64_t>(S, 1) * 2 * K)) != DMOE_OK) return s;
  if ((s = grow(L->ep_xr, L->ep_xr_cap, (size_t)std::max<int64_t>(R, 1) * H)) != DMOE_OK) return s;
  if ((s = grow(L->ep_mr, L->ep_mr_cap, (size_t)std::max<int64_t>(R, 1) * 2 * K)) != DMOE_OK) return s;
  if ((s = grow(L->ep_part, L->ep_part_cap, (size_t)std::max<int64_t>(R, 1) * H)) != DMOE_OK) return s;
  if ((s = grow(L->ep_back, L->ep_back_cap, (size_t)std::max<int64_t>(S, 1) * H)) != DMOE_OK) return s;
  if ((s = grow(L->tiles, L->tiles_cap, (size_t)(Pmax / 32 + Eh + 2))) != DMOE_OK) return s;
  if ((s = grow(L->xg, L->xg_cap, (size_t)rows_max * H)) != DMOE_OK) return s;
  if ((s = grow(L->hbuf, L->hbuf_cap, (size_t)rows_max * Imax)) != DMOE_OK) return s;
  if ((s = grow(L->pair_tok, L->pair_tok_cap, (size_t)rows_max)) != DMOE_OK) return s;
  if ((s = grow(L->pair_w, L->pair_w_cap, (size_t)rows_max)) != DMOE_OK) return s;
  if ((s = grow(L->tt_done, L->tt_done_cap, (size_t)(Pmax / 32 + Eh + 2 + (nmax + 31) / 32))) != DMOE_OK) return s;
  // ---- 3a. pack every chunk, each chunk's dispatch on the comm stream once its rows are packed
  for (int c = 0; c < C; ++c) {
    DMOE_CUDA(launch_ep_pack(xd + t0[c] * H, nc[c], (int)H, (int)K, idx + t0[c] * K, w + t0[c] * K, (int)El, hot,
                             L->rank, L->ep_mask + t0[c], L->ep_pos + W * t0[c], soff[c], L->etype == DMOE_TYPE_Q4_K,
                             L->ep_xs, L->ep_ms, st));
    kernels += nc[c] > 0 ? 1 : 0;
    DMOE_CUDA(cudaEventRecord(L->ev_pack[c], st));
  }
  for (int c = 0; c < C; ++c) {
    DMOE_CUDA(cudaStreamWaitEvent(cs, L->ev_pack[c], 0));
    DMOE_NCCL(api.GroupStart(), "ncclGroupStart");
    for (int p = 0; p < W; ++p) {
      const int64_t ns = L->ep_host[p * C + c], nr = L->ep_host[W * C + p * C + c];
      if (ns) {
        DMOE_NCCL(api.Send(L->ep_xs + (int64_t)soff[c].v[p] * H, (size_t)(ns * H), ncclFloat16, p, L->comm, cs),
                  "ncclSend(rows)");
        DMOE_NCCL(api.Send(L->ep_ms + (int64_t)soff[c].v[p] * 2 * K, (size_t)(ns * 2 * K), ncclInt32, p, L->comm, cs),
                  "ncclSend(slots)");
      }
      if (nr) {
        DMOE_NCCL(api.Recv(L->ep_xr + (int64_t)roff[c].v[p] * H, (size_t)(nr * H), ncclFloat16, p, L->comm, cs),
                  "ncclRecv(rows)");
        DMOE_NCCL(api.Recv(L->ep_mr + (int64_t)roff[c].v[p] * 2 * K, (size_t)(nr * 2 * K), ncclInt32, p, L->comm, cs),
                  "ncclRecv(slots)");
      }
    }
    DMOE_NCCL(api.GroupEnd(), "dispatch exchange");
    DMOE_CUDA(cudaEventRecord(L->ev_disp[c], cs));
  }
  if (prof) DMOE_CUDA(cudaEventRecord(L->ev[2], st));
  // ---- 3b. the shared expert over all of this rank's tokens: it needs no exchange, so it runs
  // while the dispatches are in flight (rows [0, n) of the gathered layout, straight into od)
  int32_t* n_tiles = L->ints + 3 * L->E;
  if (L->has_shared && n > 0) {
    const int nt_sh = pick_nt(L, n);
    DMOE_CUDA(launch_gather_shared(xd, n, (int)H, L->stype == DMOE_TYPE_Q4_K, L->xg, st));
    DMOE_CUDA(cudaMemsetAsync(L->tt_done, 0, sizeof(int32_t) * (size_t)((n + nt_sh - 1) / nt_sh), st));
    ++kernels;
    if ((s = run_experts(L, st, n, n, nt_sh, n_tiles, od, od, 0, false, false, false, kernels, /*groups=*/1)) !=
        DMOE_OK)
      return s;
  } else if (n > 0) {
    DMOE_CUDA(cudaMemsetAsync(od, 0, sizeof(float) * (size_t)(n * H), st));
  }
  // ---- 3c. per chunk: the routed experts over the received rows (pairs from row 0 of the
  // gathered layout), then the chunk's combine on the comm stream
  const int nt = pick_nt(L, std::max<int64_t>(1, n / C));
  int32_t* counts = L->ints;  // [e_local] (the router's global counts are not needed any more)
  int32_t* fill = L->ints + L->E;
  int32_t* off = L->ints + 2 * L->E;
  int32_t* n_active = n_tiles + 1;
  for (int c = 0; c < C; ++c) {
    const int64_t rbase = roff[c].v[0];
    DMOE_CUDA(cudaStreamWaitEvent(st, L->ev_disp[c], 0));
    if (Rc[c] > 0) {
      const int64_t rows = Rc[c] * K;
      DMOE_CUDA(cudaMemsetAsync(counts, 0, sizeof(int32_t) * (size_t)Eh, st));
      DMOE_CUDA(launch_ep_count(L->ep_mr + rbase * 2 * K, Rc[c], (int)K, counts, st));
      DMOE_CUDA(launch_scan_tiles(counts, (int)Eh, 0, nt, off, fill, L->tiles, n_tiles, n_active, L->tt_done, 0, st));
      DMOE_CUDA(launch_gather_rows(L->ep_xr + rbase * H, Rc[c], (int)H, (int)K, L->ep_mr + rbase * 2 * K, off, fill,
                                   L->xg, L->pair_tok, L->pair_w, st));
      kernels += 4;
      if ((s = run_experts(L, st, 0, rows, nt, n_tiles, od, L->ep_part + rbase * H, Rc[c], false, true,
                           prof && c == C - 1, kernels, /*groups=*/2)) != DMOE_OK)
        return s;
    }
    DMOE_CUDA(cudaEventRecord(L->ev_exp[c], st));
    DMOE_CUDA(cudaStreamWaitEvent(cs, L->ev_exp[c], 0));
    DMOE_NCCL(api.GroupStart(), "ncclGroupStart");
    for (int p = 0; p < W; ++p) {
      const int64_t ns = L->ep_host[p * C + c], nr = L->ep_host[W * C + p * C + c];
      if (nr)
        DMOE_NCCL(api.Send(L->ep_part + (int64_t)roff[c].v[p] * H, (size_t)(nr * H), ncclFloat32, p, L->comm, cs),
                  "ncclSend(partials)");
      if (ns)
        DMOE_NCCL(api.Recv(L->ep_back + (int64_t)soff[c].v[p] * H, (size_t)(ns * H), ncclFloat32, p, L->comm, cs),
                  "ncclRecv(partials)");
    }
    DMOE_NCCL(api.GroupEnd(), "combine exchange");
    DMOE_CUDA(cudaEventRecord(L->ev_comb[c], cs));
  }
  // ---- 3c. each chunk's owner sum, once its partials are back
  for (int c = 0; c < C; ++c) {
    DMOE_CUDA(cudaStreamWaitEvent(st, L->ev_comb[c], 0));
    DMOE_CUDA(launch_ep_final(od + t0[c] * H, L->ep_back, nc[c], (int)H, L->ep_mask + t0[c], L->ep_pos + W * t0[c],
                              soff[c], st));
    kernels += nc[c] > 0 ? 1 : 0;
  }
  if (prof) DMOE_CUDA(cudaEventRecord(L->ev[4], st));
  DMOE_CUDA(cudaMemcpyAsync(L->host_counters, n_tiles, 8, cudaMemcpyDeviceToHost, st));
  L->stats.ep_rows_sent = S;
  L->stats.ep_rows_received = R;
  return DMOE_OK;
}

// Chunk size for a pipelined host-buffer call, or 0 to run it whole. Only on one GPU, without
// routing outputs or profiling (their per-call buffers would be shared between chunks), for at
// least 4096 tokens, and only where chunking cannot change the routing: chunks are whole routing
// blocks when the call uses block routing, and a call that does not (n % block != 0) is not
// chunked if a chunk of whole blocks would switch block routing on.
// Chunk plan of a host-buffer call (0 chunks: one unchunked call). The copies share PCIe (about
// 51 GB/s one way, 77 GB/s both ways at once, measured on B200) and a chunk's compute costs more
// per token the smaller it is, so the plan starts small (its upload is exposed), grows while
// earlier chunks compute, and ends small (its download is exposed): five chunks in proportions
// 2:4:6:3:1 up to 8192 tokens, six in 1:2:4:4:2:1 above, each a multiple of 8 routing blocks.
// Modelled from the measured per-size layer times, this takes 256 x 32 tokens from 5.6 to 5.2 ms
// against four equal chunks. DMOE_HOST_CHUNK = t forces equal chunks of t tokens (0: never chunk).
int host_chunk_plan(const dmoe_layer* L, int64_t n, bool host, const dmoe_route_out* route, uint32_t flags,
                    int64_t (&sizes)[dmoe_layer::kMaxChunks]) {
  if (!host || route || (flags & (DMOE_F_ROUTE_ONLY | DMOE_F_PROFILE)) || L->world > 1) return 0;
  const int forced = env_int("DMOE_HOST_CHUNK", -1);
  const int64_t threshold = forced > 0 ? 2 * (int64_t)forced : 4096;
  if (forced == 0 || n < threshold) return 0;
  const bool block_possible = L->blk > 1 && L->cap > 0 && L->cap < L->E;
  if (block_possible && n % L->blk) return 0;
  const int64_t unit = block_possible ? L->blk : 32;  // chunks hold whole routing blocks
  int nc = 0;
  if (forced > 0) {
    int64_t chunk = std::max<int64_t>(unit, forced / unit * unit);
    if ((n + chunk - 1) / chunk > dmoe_layer::kMaxChunks)
      chunk = ((n + dmoe_layer::kMaxChunks - 1) / dmoe_layer::kMaxChunks + unit - 1) / unit * unit;
    for (int64_t t0 = 0; t0 < n; t0 += chunk) sizes[nc++] = std::min(chunk, n - t0);
    return nc;
  }
  static constexpr int kW5[] = {2, 4, 6, 3, 1}, kW6[] = {1, 2, 4, 4, 2, 1};
  const bool small = n <= 8192;
  const int* w = small ? kW5 : kW6;
  const int nw = small ? 5 : 6, wsum = 16, biggest = 2;
  const int64_t g = 8 * unit;
  int64_t rest = n;
  for (int i = 0; i < nw; ++i) {
    sizes[i] = std::max<int64_t>(g, (n * w[i] / wsum + g / 2) / g * g);
    rest -= sizes[i];
  }
  sizes[biggest] += rest;  // the remainder (a multiple of the unit) goes to the largest chunk
  if (sizes[biggest] < 0) return 0;
  for (int i = 0; i < nw; ++i)
    if (sizes[i] > 0) sizes[nc++] = sizes[i];
  return nc;
}

}  // namespace

extern "C" {
dmoe_status dmoe_forward(dmoe_layer* L, const float* x, int64_t n, float* out, const dmoe_route_out* route,
                         void* stream, uint32_t flags);
}

namespace {

// Host-buffer call in chunks: H2D of every chunk on h2d_stream, each chunk's layer on the layer's
// stream once its input has landed, the D2H of its output on d2h_stream once it is computed.
// The statistics describe the last chunk.
dmoe_status forward_chunked(dmoe_layer* L, const float* x, int64_t n, float* out, const int64_t* sizes, int nc,
                            uint32_t flags) {
  const int64_t H = L->H;
  dmoe_status s;
  if ((s = grow(L->xdev, L->xdev_cap, (size_t)n * H)) != DMOE_OK) return s;
  if ((s = grow(L->odev, L->odev_cap, (size_t)n * H)) != DMOE_OK) return s;
  cudaStream_t ks = L->own_stream;
  // the copies reuse xdev / odev: order them after earlier work on the layer's stream
  DMOE_CUDA(cudaEventRecord(L->ev_start, ks));
  DMOE_CUDA(cudaStreamWaitEvent(L->h2d_stream, L->ev_start, 0));
  DMOE_CUDA(cudaStreamWaitEvent(L->d2h_stream, L->ev_start, 0));
  int64_t starts[dmoe_layer::kMaxChunks];
  for (int64_t c = 0, t0 = 0; c < nc; t0 += sizes[c], ++c) starts[c] = t0;
  if (starts[nc - 1] + sizes[nc - 1] != n) return fail(DMOE_ERR_INVALID_ARG, "chunk plan does not cover the call");
  for (int c = 0; c < nc; ++c) {
    const int64_t t0 = starts[c], cn = sizes[c];
    DMOE_CUDA(cudaMemcpyAsync(L->xdev + t0 * H, x + t0 * H, (size_t)cn * H * 4, cudaMemcpyHostToDevice, L->h2d_stream));
    DMOE_CUDA(cudaEventRecord(L->ev_in[c], L->h2d_stream));
  }
  int kernels = 0;
  for (int c = 0; c < nc; ++c) {
    const int64_t t0 = starts[c], cn = sizes[c];
    const NvtxRange nvtx_chunk("dmoe host chunk");
    DMOE_CUDA(cudaStreamWaitEvent(ks, L->ev_in[c], 0));
    if ((s = dmoe_forward(L, L->xdev + t0 * H, cn, L->odev + t0 * H, nullptr, ks, flags & ~DMOE_F_HOST_PTRS)) != DMOE_OK)
      return s;
    kernels += L->stats.kernels;
    DMOE_CUDA(cudaEventRecord(L->ev_done[c], ks));
    DMOE_CUDA(cudaStreamWaitEvent(L->d2h_stream, L->ev_done[c], 0));
    DMOE_CUDA(cudaMemcpyAsync(out + t0 * H, L->odev + t0 * H, (size_t)cn * H * 4, cudaMemcpyDeviceToHost, L->d2h_stream));
  }
  DMOE_CUDA(cudaStreamSynchronize(L->d2h_stream));
  L->stats.kernels = kernels;
  L->last_stream = ks;
  return dmoe_sync(L);
}

}  // namespace

extern "C" {

int32_t dmoe_abi_version(void) { return DMOE_ABI_VERSION; }

size_t dmoe_last_error(char* buf, size_t len) {
  if (buf && len) {
    const size_t n = std::min(len - 1, g_last_error.size());
    std::memcpy(buf, g_last_error.data(), n);
    buf[n] = 0;
  }
  return g_last_error.size();
}

// dmoe_create; with `parent` (an expert-parallel layer of the same ranks) the new layer's
// communicator is split from the parent's instead of initialised from dist->nccl_id, so that
// one unique id serves every layer of a model.
static dmoe_status create_layer(const dmoe_layer_desc* d, const dmoe_dist_cfg* dist, const dmoe_layer* parent,
                                dmoe_layer** out) {
  if (!out) return fail(DMOE_ERR_INVALID_ARG, "null output handle");
  *out = nullptr;
  dmoe_status st = validate(d);
  if (st != DMOE_OK) return st;
  const int world = dist ? std::max(1, dist->world_size) : 1;
  if (parent && world <= 1)
    return fail(DMOE_ERR_INVALID_ARG, "a split communicator needs an expert-parallel dist (world_size > 1)");
  if (world > 1) {
    if (world > kMaxRanks) return fail(DMOE_ERR_UNSUPPORTED, "world_size %d > %d", world, kMaxRanks);
    if (dist->rank < 0 || dist->rank >= world) return fail(DMOE_ERR_INVALID_ARG, "rank %d of %d", dist->rank, world);
    if (d->n_expert % world) return fail(DMOE_ERR_UNSUPPORTED, "n_expert %lld not divisible by world_size %d",
                                         (long long)d->n_expert, world);
    if (!dist->nccl_id && !parent) return fail(DMOE_ERR_INVALID_ARG, "expert parallelism needs dist->nccl_id");
    if (parent && (!parent->comm || parent->world != world || parent->rank != dist->rank))
      return fail(DMOE_ERR_INVALID_ARG, "parent layer is not an expert-parallel layer of the same ranks");
    if (!nccl().ok) return fail(DMOE_ERR_NCCL, "NCCL unavailable: %s", nccl().why);
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    return fail(DMOE_ERR_NO_DEVICE, "no CUDA device (libdiffuse_moe has no CPU fallback)");
  }
  dmoe_layer* L = new dmoe_layer();
  L->device = dist ? dist->device : 0;
  if (L->device < 0 || L->device >= ndev) {
    delete L;
    return fail(DMOE_ERR_INVALID_ARG, "device %d out of range", dist ? dist->device : 0);
  }
  auto bail = [&](dmoe_status s) {
    dmoe_destroy(L);
    return s;
  };
  if (cudaSetDevice(L->device) != cudaSuccess) return bail(fail(DMOE_ERR_CUDA, "cudaSetDevice"));
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, L->device) != cudaSuccess) return bail(fail(DMOE_ERR_CUDA, "device props"));
  if (prop.major != 10) return bail(fail(DMOE_ERR_UNSUPPORTED, "device sm_%d%d is not sm_100", prop.major, prop.minor));
  L->sms = prop.multiProcessorCount;
  L->H = d->n_embd;
  L->I = d->n_ff_exp;
  L->Is = d->n_ff_shexp;
  L->E = d->n_expert;
  L->K = d->n_expert_used;
  L->cap = d->expert_capacity;
  L->blk = d->moe_block_size;
  L->scale = d->routed_scaling;
  L->norm_topk = d->norm_topk_prob;
  L->etype = d->expert_type;
  L->stype = d->shared_type;
  L->has_shared = d->n_ff_shexp > 0;
  L->has_bias = d->b_router != nullptr;
  L->world = world;
  L->rank = world > 1 ? dist->rank : 0;
  L->e_local = L->E / world;
  L->timeout_ms = (dist && dist->timeout_ms > 0) ? dist->timeout_ms : 60000;
  if (cudaStreamCreateWithFlags(&L->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&L->h2d_stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&L->d2h_stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail(fail(DMOE_ERR_CUDA, "stream create"));
  for (int c = 0; c < dmoe_layer::kMaxChunks; ++c)
    if (cudaEventCreateWithFlags(&L->ev_in[c], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&L->ev_done[c], cudaEventDisableTiming) != cudaSuccess)
      return bail(fail(DMOE_ERR_CUDA, "event create"));
  if (cudaEventCreateWithFlags(&L->ev_start, cudaEventDisableTiming) != cudaSuccess)
    return bail(fail(DMOE_ERR_CUDA, "event create"));
  for (auto& e : L->ev)
    if (cudaEventCreate(&e) != cudaSuccess) return bail(fail(DMOE_ERR_CUDA, "event create"));
  {
    // router weight, stored transposed [H][E] so the logits kernel reads contiguous weight rows
    std::vector<float> wrt((size_t)L->E * L->H);
    for (int64_t e = 0; e < L->E; ++e)
      for (int64_t k = 0; k < L->H; ++k) wrt[(size_t)k * L->E + e] = d->w_router[(size_t)e * L->H + k];
    if (cudaMalloc(&L->wr, (size_t)L->E * L->H * 4) != cudaSuccess) return bail(fail(DMOE_ERR_OOM, "router alloc"));
    if (cudaMemcpy(L->wr, wrt.data(), (size_t)L->E * L->H * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return bail(fail(DMOE_ERR_CUDA, "router upload"));
  }
  if (L->has_bias) {
    if (cudaMalloc(&L->br, (size_t)L->E * 4) != cudaSuccess) return bail(fail(DMOE_ERR_OOM, "bias alloc"));
    if (cudaMemcpy(L->br, d->b_router, (size_t)L->E * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return bail(fail(DMOE_ERR_CUDA, "bias upload"));
  }
  {
    // this rank's experts: a contiguous slice of each [E][rows][k] GGUF tensor
    const int64_t e0 = (int64_t)L->rank * L->e_local;
    const uint8_t* g = static_cast<const uint8_t*>(d->w_gate) + (size_t)e0 * L->I * row_size(L->etype, L->H);
    const uint8_t* u = static_cast<const uint8_t*>(d->w_up) + (size_t)e0 * L->I * row_size(L->etype, L->H);
    const uint8_t* dn = static_cast<const uint8_t*>(d->w_down) + (size_t)e0 * L->H * row_size(L->etype, L->I);
    if ((st = upload_weight(L->gate, L->etype, g, L->e_local * L->I, L->H)) != DMOE_OK) return bail(st);
    if ((st = upload_weight(L->up, L->etype, u, L->e_local * L->I, L->H)) != DMOE_OK) return bail(st);
    if ((st = upload_weight(L->down, L->etype, dn, L->e_local * L->H, L->I)) != DMOE_OK) return bail(st);
  }
  if (L->has_shared) {
    if ((st = upload_weight(L->sgate, L->stype, d->sw_gate, L->Is, L->H)) != DMOE_OK) return bail(st);
    if ((st = upload_weight(L->sup, L->stype, d->sw_up, L->Is, L->H)) != DMOE_OK) return bail(st);
    if ((st = upload_weight(L->sdown, L->stype, d->sw_down, L->H, L->Is)) != DMOE_OK) return bail(st);
  }
  if (cudaMalloc(&L->err, 64) != cudaSuccess) return bail(fail(DMOE_ERR_OOM, "err alloc"));
  if (cudaMemset(L->err, 0, 64) != cudaSuccess) return bail(fail(DMOE_ERR_CUDA, "err memset"));
  if (cudaMallocHost(&L->host_counters, 64) != cudaSuccess) return bail(fail(DMOE_ERR_OOM, "pinned alloc"));
  std::memset(L->host_counters, 0, 64);
  if (world > 1) {
    if (cudaMallocHost(&L->ep_host, sizeof(int32_t) * 2 * kMaxRanks * dmoe_layer::kMaxChunks) != cudaSuccess)
      return bail(fail(DMOE_ERR_OOM, "pinned alloc"));
    // pipeline chunks of the exchange (every rank must use the same count) and the SMs the GEMMs
    // leave to NCCL's kernels so that the exchange runs beside the shared expert's GEMMs (and, with
    // chunks, beside another chunk's GEMMs). Measured on 2 B200s (c3, 8192 tokens per rank):
    // 3.65 ms per forward with one chunk, 3.92 with two, 4.60 with four (the smaller GEMMs of a
    // chunk lose more than the overlap gains), so one chunk by default.
    L->ep_chunks = std::min(dmoe_layer::kMaxChunks, std::max(1, env_int("DMOE_EP_CHUNKS", 1)));
    L->gemm_sm_reserve = std::min(L->sms / 4, std::max(0, env_int("DMOE_EP_SM_RESERVE", 8)));
    if (cudaStreamCreateWithFlags(&L->comm_stream, cudaStreamNonBlocking) != cudaSuccess)
      return bail(fail(DMOE_ERR_CUDA, "stream create"));
    // per-expert loads of the last forward, their sum over ranks, replica slots (none yet)
    if (cudaMalloc(&L->ep_load, sizeof(int32_t) * (size_t)L->E) != cudaSuccess ||
        cudaMalloc(&L->ep_load_sum, sizeof(int32_t) * (size_t)L->E) != cudaSuccess ||
        cudaMalloc(&L->hot_slot, sizeof(int32_t) * (size_t)L->E) != cudaSuccess)
      return bail(fail(DMOE_ERR_OOM, "cudaMalloc expert loads"));
    if (cudaMemset(L->ep_load, 0, sizeof(int32_t) * (size_t)L->E) != cudaSuccess ||
        cudaMemset(L->hot_slot, 0xff, sizeof(int32_t) * (size_t)L->E) != cudaSuccess)
      return bail(fail(DMOE_ERR_CUDA, "cudaMemset expert loads"));
    for (int c = 0; c < dmoe_layer::kMaxChunks; ++c)
      if (cudaEventCreateWithFlags(&L->ev_pack[c], cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&L->ev_disp[c], cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&L->ev_exp[c], cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&L->ev_comb[c], cudaEventDisableTiming) != cudaSuccess)
        return bail(fail(DMOE_ERR_CUDA, "event create"));
    // non-blocking communicator: init and every group are polled against the layer's deadline
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r;
    if (parent) {
      r = nccl().CommSplit(parent->comm, 0, L->rank, &L->comm, &cfg);
    } else {
      ncclUniqueId id;
      std::memcpy(&id, dist->nccl_id, sizeof(id));
      r = nccl().CommInitRankConfig(&L->comm, world, id, L->rank, &cfg);
    }
    if (r != ncclSuccess && r != ncclInProgress) {
      L->comm = nullptr;
      return bail(fail(DMOE_ERR_NCCL, "%s: %s", parent ? "ncclCommSplit" : "ncclCommInitRankConfig",
                       nccl().GetErrorString(r)));
    }
    if ((st = nccl_settle(L, r, "communicator init (all ranks must call dmoe_create)")) != DMOE_OK) return bail(st);
  }
  *out = L;
  return DMOE_OK;
}

dmoe_status dmoe_create(const dmoe_layer_desc* d, const dmoe_dist_cfg* dist, dmoe_layer** out) {
  return create_layer(d, dist, nullptr, out);
}

dmoe_status dmoe_create_split(const dmoe_layer_desc* d, const dmoe_dist_cfg* dist, const dmoe_layer* parent,
                              dmoe_layer** out) {
  if (!parent) return fail(DMOE_ERR_INVALID_ARG, "null parent layer");
  return create_layer(d, dist, parent, out);
}

dmoe_status dmoe_nccl_unique_id(void* id128) {
  if (!id128) return fail(DMOE_ERR_INVALID_ARG, "null id buffer");
  if (!nccl().ok) return fail(DMOE_ERR_NCCL, "NCCL unavailable: %s", nccl().why);
  ncclUniqueId id;
  const ncclResult_t r = nccl().GetUniqueId(&id);
  if (r != ncclSuccess) return fail(DMOE_ERR_NCCL, "ncclGetUniqueId: %s", nccl().GetErrorString(r));
  std::memcpy(id128, &id, sizeof(id));
  return DMOE_OK;
}

void dmoe_destroy(dmoe_layer* L) {
  if (!L) return;
  cudaSetDevice(L->device);
  if (L->comm) {
    // drain this rank's work (bounded by the deadline), then release the communicator without
    // waiting on the other ranks: destroy never blocks on a peer that is gone
    ep_wait(L, L->last_stream, "destroy");
    if (L->comm) nccl().CommAbort(L->comm);
    L->comm = nullptr;
  }
  if (L->own_stream) cudaStreamSynchronize(L->own_stream);
  cudaStreamSynchronize(L->last_stream);
  cudaFree(L->wr);
  cudaFree(L->br);
  for (DevWeight* w : {&L->gate, &L->up, &L->down, &L->sgate, &L->sup, &L->sdown}) free_weight(*w);
  cudaFree(L->parts);
  cudaFree(L->arrivals);
  cudaFree(L->idx);
  cudaFree(L->wts);
  cudaFree(L->allowed);
  cudaFree(L->ints);
  cudaFree(L->tiles);
  cudaFree(L->xg);
  cudaFree(L->hbuf);
  cudaFree(L->gu);
  cudaFree(L->pair_tok);
  cudaFree(L->pair_w);
  cudaFree(L->pair_row);
  cudaFree(L->ybuf);
  cudaFree(L->tt_done);
  cudaFree(L->xdev);
  cudaFree(L->odev);
  cudaFree(L->err);
  for (void* p : {(void*)L->ep_mask, (void*)L->ep_pos, (void*)L->ep_cnt, (void*)L->ep_xs, (void*)L->ep_ms,
                  (void*)L->ep_xr, (void*)L->ep_mr, (void*)L->ep_part, (void*)L->ep_back, (void*)L->ep_load,
                  (void*)L->ep_load_sum, (void*)L->hot_slot})
    cudaFree(p);
  if (L->ep_host) cudaFreeHost(L->ep_host);
  if (L->host_counters) cudaFreeHost(L->host_counters);
  for (auto& e : L->ev)
    if (e) cudaEventDestroy(e);
  if (L->own_stream) cudaStreamDestroy(L->own_stream);
  for (cudaStream_t cs : {L->h2d_stream, L->d2h_stream})
    if (cs) {
      cudaStreamSynchronize(cs);
      cudaStreamDestroy(cs);
    }
  for (int c = 0; c < dmoe_layer::kMaxChunks; ++c) {
    if (L->ev_in[c]) cudaEventDestroy(L->ev_in[c]);
    if (L->ev_done[c]) cudaEventDestroy(L->ev_done[c]);
  }
  if (L->ev_start) cudaEventDestroy(L->ev_start);
  if (L->comm_stream) {
    cudaStreamSynchronize(L->comm_stream);  // the communicator is aborted: its kernels have ended
    cudaStreamDestroy(L->comm_stream);
  }
  for (int c = 0; c < dmoe_layer::kMaxChunks; ++c)
    for (cudaEvent_t e : {L->ev_pack[c], L->ev_disp[c], L->ev_exp[c], L->ev_comb[c]})
      if (e) cudaEventDestroy(e);
  delete L;
}

dmoe_status dmoe_forward(dmoe_layer* L, const float* x, int64_t n, float* out, const dmoe_route_out* route,
                         void* stream, uint32_t flags) {
  if (!L) return fail(DMOE_ERR_INVALID_ARG, "null layer");
  if (L->broken) return fail(DMOE_ERR_NCCL, "a collective of this layer failed earlier; re-create it on every rank");
  if (n < 0 || (n > 0 && !x)) return fail(DMOE_ERR_INVALID_ARG, "bad input");
  const bool route_only = flags & DMOE_F_ROUTE_ONLY;
  const bool host = flags & DMOE_F_HOST_PTRS;
  const bool prof = flags & DMOE_F_PROFILE;
  if (!route_only && n > 0 && !out) return fail(DMOE_ERR_INVALID_ARG, "null output");
  if (n * (1 + L->K) >= (1ll << 31)) return fail(DMOE_ERR_UNSUPPORTED, "too many tokens in one call");
  const NvtxRange nvtx_call("dmoe_forward");
  DMOE_CUDA(cudaSetDevice(L->device));
  // device mode: the caller's stream as given (NULL = the CUDA default stream);
  // host mode without a stream: the layer's own stream
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (host && !stream) st = L->own_stream;
  L->last_stream = st;
  L->profiled = prof;
  set_pdl_for_call(n < 1024);
  std::memset(&L->stats, 0, sizeof(L->stats));
  if (n == 0) {
    if (L->world == 1 || route_only) return DMOE_OK;
    // expert parallelism: a rank without tokens still takes its part in the exchange (the other
    // ranks' rows for its experts arrive all the same)
    dmoe_status s0;
    if ((s0 = grow(L->ints, L->ints_cap, (size_t)3 * L->E + 8)) != DMOE_OK) return s0;
    int kernels = 0;
    const NvtxRange nvtx_experts("dmoe experts (expert parallel, no local tokens)");
    if ((s0 = ep_experts(L, st, nullptr, 0, nullptr, nullptr, nullptr, flags, kernels)) != DMOE_OK) return s0;
    L->stats.kernels = kernels;
    return host ? dmoe_sync(L) : DMOE_OK;
  }
  {
    int64_t sizes[dmoe_layer::kMaxChunks];
    if (const int nc = host_chunk_plan(L, n, host, route, flags, sizes); nc > 0)
      return forward_chunked(L, x, n, out, sizes, nc, flags);
  }

  const int64_t H = L->H, E = L->E, K = L->K;
  const bool use_block = L->blk > 1 && L->cap > 0 && L->cap < E && n % L->blk == 0;
  const int nseg = (int)((H + kRouterSeg - 1) / kRouterSeg);
  RouterPlan rl_plan = router_plan(n, (int)E, (int)H, L->sms);  // too few whole-K tiles: split by segment
  if (const int f = env_int("DMOE_ROUTER_SPLIT", -1); f >= 0 && f <= 3) rl_plan = (RouterPlan)f;
  const bool rl_split = rl_plan == ROUTER_SPLIT2 || rl_plan == ROUTER_SPLIT8;
  const int nparts = rl_split ? nseg : 1;

  dmoe_status s;
  size_t dummy_cap;
  (void)dummy_cap;
  if ((s = grow(L->parts, L->parts_cap, (size_t)nparts * n * E)) != DMOE_OK) return s;
  if (rl_split) {
    // per-tile arrival counters: zeroed when (re)allocated, re-armed by the kernel after use
    const size_t need = (size_t)router_arrivals(n, (int)E);
    if (need > L->arrivals_cap) {
      cudaFree(L->arrivals);
      L->arrivals = nullptr;
      L->arrivals_cap = 0;
      if ((s = grow(L->arrivals, L->arrivals_cap, need)) != DMOE_OK) return s;
      DMOE_CUDA(cudaMemsetAsync(L->arrivals, 0, L->arrivals_cap * sizeof(int32_t), st));
    }
  }
  if ((s = grow(L->idx, L->idx_cap, (size_t)n * K)) != DMOE_OK) return s;
  if ((s = grow(L->wts, L->wts_cap, (size_t)n * K)) != DMOE_OK) return s;
  if ((s = grow(L->ints, L->ints_cap, (size_t)3 * E + 8)) != DMOE_OK) return s;
  if (use_block && (s = grow(L->allowed, L->allowed_cap, (size_t)(n / L->blk) * E)) != DMOE_OK) return s;
  int32_t* counts = L->ints;

  const float* xd = x;
  float* od = out;
  if (host) {
    if ((s = grow(L->xdev, L->xdev_cap, (size_t)n * H)) != DMOE_OK) return s;
    DMOE_CUDA(cudaMemcpyAsync(L->xdev, x, (size_t)n * H * 4, cudaMemcpyHostToDevice, st));
    xd = L->xdev;
    if (!route_only) {
      if ((s = grow(L->odev, L->odev_cap, (size_t)n * H)) != DMOE_OK) return s;
      od = L->odev;
    }
  }
  int kernels = 0;
  if (prof) DMOE_CUDA(cudaEventRecord(L->ev[0], st));

  // ---- router (src/diffuse-moe-graph.cpp:203-262)
  auto nvtx_router = std::make_unique<NvtxRange>("dmoe router");
  DMOE_CUDA(launch_router(xd, L->wr, L->parts, n, (int)H, (int)E, rl_plan, L->arrivals, counts, st));
  ++kernels;
  RouteArgs ra{};
  ra.probs = L->parts;
  ra.bias = L->br;
  ra.n = n;
  ra.e = (int)E;
  ra.top_k = (int)K;
  ra.cap = (int)L->cap;
  ra.blk = (int)L->blk;
  ra.use_block = use_block ? 1 : 0;
  ra.norm_topk = L->norm_topk;
  ra.scale = L->scale;
  ra.idx = (route && route->idx && !host) ? route->idx : L->idx;
  ra.w = (route && route->weights && !host) ? route->weights : L->wts;
  ra.allowed = use_block ? ((route && route->allowed && !host) ? route->allowed : L->allowed) : nullptr;
  ra.counts = counts;
  DMOE_CUDA(launch_route(ra, st));
  ++kernels;
  // expert parallelism: keep this forward's per-expert pair counts for dmoe_replicate_experts
  if (L->world > 1 && !route_only)
    DMOE_CUDA(cudaMemcpyAsync(L->ep_load, counts, sizeof(int32_t) * (size_t)E, cudaMemcpyDeviceToDevice, st));
  if (prof) DMOE_CUDA(cudaEventRecord(L->ev[1], st));
  nvtx_router.reset();

  if (!route_only) {
    const NvtxRange nvtx_experts(L->world == 1 ? "dmoe experts" : "dmoe experts (expert parallel)");
    s = L->world == 1 ? single_gpu_experts(L, st, xd, n, ra.idx, ra.w, counts, od, flags, kernels)
                      : ep_experts(L, st, xd, n, ra.idx, ra.w, od, flags, kernels);
    if (s != DMOE_OK) return s;
  }
  L->stats.router_parts = nparts;
  L->stats.kernels = kernels;
  L->stats.used_block_routing = use_block ? 1 : 0;

  if (host) {
    if (!route_only) DMOE_CUDA(cudaMemcpyAsync(out, od, (size_t)n * H * 4, cudaMemcpyDeviceToHost, st));
    if (route) {
      if (route->idx) DMOE_CUDA(cudaMemcpyAsync(route->idx, ra.idx, (size_t)n * K * 4, cudaMemcpyDeviceToHost, st));
      if (route->weights)
        DMOE_CUDA(cudaMemcpyAsync(route->weights, ra.w, (size_t)n * K * 4, cudaMemcpyDeviceToHost, st));
      if (route->allowed && use_block)
        DMOE_CUDA(cudaMemcpyAsync(route->allowed, ra.allowed, (size_t)(n / L->blk) * E, cudaMemcpyDeviceToHost, st));
    }
    return dmoe_sync(L);
  }
  return DMOE_OK;
}

dmoe_status dmoe_sync(dmoe_layer* L) {
  if (!L) return fail(DMOE_ERR_INVALID_ARG, "null layer");
  DMOE_CUDA(cudaSetDevice(L->device));
  if (L->comm) {
    dmoe_status s = ep_wait(L, L->last_stream, "forward");
    if (s != DMOE_OK) return s;
  } else {
    DMOE_CUDA(cudaStreamSynchronize(L->last_stream));
  }
  uint32_t e = 0;
  DMOE_CUDA(cudaMemcpy(&e, L->err, 4, cudaMemcpyDeviceToHost));
  L->stats.n_routed_tiles = L->host_counters[0];
  L->stats.n_active = L->host_counters[1];
  if (L->profiled) {
    float a = 0, b = 0, c = 0, d = 0;
    cudaEventElapsedTime(&a, L->ev[0], L->ev[1]);
    if (L->stats.token_tile) {
      cudaEventElapsedTime(&b, L->ev[1], L->ev[2]);
      cudaEventElapsedTime(&c, L->ev[2], L->ev[3]);
      cudaEventElapsedTime(&d, L->ev[3], L->ev[4]);
    }
    L->stats.ms_router = a;
    L->stats.ms_dispatch = b;
    L->stats.ms_gateup = c;
    L->stats.ms_down = d;
    L->stats.ms_total = a + b + c + d;
  }
  if (e) {
    // a timeout wins over an out-of-bounds tile (the status a caller retries on); the message
    // names every condition that was seen
    cudaMemset(L->err, 0, 4);
    const bool bad = e & ERRBIT_BAD_TILE, timeout = e & ~(uint32_t)ERRBIT_BAD_TILE;
    if (timeout)
      return fail(DMOE_ERR_TIMEOUT, "device wait timed out; the kernel gave up%s (error bits 0x%x)",
                  bad ? "; a device-built token tile (or tile count) was also out of bounds and skipped" : "", e);
    return fail(DMOE_ERR_CUDA, "a device-built token tile (or tile count) was out of bounds and skipped (error bits 0x%x)",
                e);
  }
  return DMOE_OK;
}

dmoe_status dmoe_replicate_experts(dmoe_layer* L, const int32_t* ids, int32_t n_hot) {
  if (!L) return fail(DMOE_ERR_INVALID_ARG, "null layer");
  if (n_hot < 0 || n_hot > DMOE_MAX_HOT)
    return fail(DMOE_ERR_INVALID_ARG, "n_hot %d outside [0, %d]", n_hot, DMOE_MAX_HOT);
  if (L->world == 1) return DMOE_OK;  // one GPU holds every expert already
  if (L->broken) return fail(DMOE_ERR_NCCL, "a collective of this layer failed earlier; re-create it on every rank");
  const int64_t E = L->E, El = L->e_local;
  if (n_hot > E - El)
    return fail(DMOE_ERR_INVALID_ARG, "n_hot %d > n_expert - experts per rank (%lld)", n_hot, (long long)(E - El));
  DMOE_CUDA(cudaSetDevice(L->device));
  const NcclApi& api = nccl();
  cudaStream_t st = L->own_stream;
  dmoe_status s = ep_wait(L, L->last_stream, "earlier forwards");  // weights and loads settle first
  if (s != DMOE_OK) return s;
  std::vector<int32_t> chosen;
  if (n_hot > 0 && ids) {
    std::vector<char> seen((size_t)E, 0);
    for (int j = 0; j < n_hot; ++j) {
      if (ids[j] < 0 || ids[j] >= E || seen[(size_t)ids[j]])
        return fail(DMOE_ERR_INVALID_ARG, "hot expert ids must be distinct and in [0, %lld)", (long long)E);
      seen[(size_t)ids[j]] = 1;
    }
    chosen.assign(ids, ids + n_hot);
  } else if (n_hot > 0) {
    // the busiest experts of the last forward over all ranks, ties to the lower id (every rank
    // computes the same choice from the same sums)
    DMOE_NCCL(api.AllReduce(L->ep_load, L->ep_load_sum, (size_t)E, ncclInt32, ncclSum, L->comm, st),
              "ncclAllReduce(expert loads)");
    if ((s = ep_wait(L, st, "expert load sum")) != DMOE_OK) return s;
    std::vector<int32_t> load((size_t)E), order((size_t)E);
    DMOE_CUDA(cudaMemcpy(load.data(), L->ep_load_sum, sizeof(int32_t) * (size_t)E, cudaMemcpyDeviceToHost));
    for (int64_t e = 0; e < E; ++e) order[(size_t)e] = (int32_t)e;
    std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return load[(size_t)a] > load[(size_t)b]; });
    chosen.assign(order.begin(), order.begin() + n_hot);
  }
  // new weight families: this rank's experts, then the replicas (broadcast from their owners)
  DevWeight* fam[3] = {&L->gate, &L->up, &L->down};
  const int64_t rpe[3] = {L->I, L->I, L->H};  // rows per expert
  DevWeight nw[3];
  auto drop_new = [&]() {
    for (DevWeight& w : nw) free_weight(w);
  };
  for (int f = 0; f < 3; ++f) {
    const DevWeight& o = *fam[f];
    nw[f].type = o.type;
    nw[f].k = o.k;
    nw[f].rows = (El + n_hot) * rpe[f];
    const size_t rb = dev_row_bytes(o), own = (size_t)(El * rpe[f]);
    if (cudaMalloc(&nw[f].q, (size_t)nw[f].rows * rb) != cudaSuccess) {
      drop_new();
      return fail(DMOE_ERR_OOM, "cudaMalloc replica weights");
    }
    DMOE_CUDA(cudaMemcpyAsync(nw[f].q, o.q, own * rb, cudaMemcpyDeviceToDevice, st));
    if (o.type == DMOE_TYPE_Q8_0) {
      if (cudaMalloc(&nw[f].s, (size_t)nw[f].rows * (o.k / 32) * 4) != cudaSuccess) {
        drop_new();
        return fail(DMOE_ERR_OOM, "cudaMalloc replica scales");
      }
      DMOE_CUDA(cudaMemcpyAsync(nw[f].s, o.s, own * (o.k / 32) * 4, cudaMemcpyDeviceToDevice, st));
    }
  }
  if (n_hot > 0) {
    DMOE_NCCL(api.GroupStart(), "ncclGroupStart");
    for (int j = 0; j < n_hot; ++j) {
      const int owner = (int)(chosen[(size_t)j] / El);
      const int64_t local = chosen[(size_t)j] - owner * El;
      for (int f = 0; f < 3; ++f) {
        const DevWeight& o = *fam[f];
        const size_t rb = dev_row_bytes(o), nbytes = (size_t)rpe[f] * rb;
        uint8_t* dst = static_cast<uint8_t*>(nw[f].q) + (size_t)(El + j) * nbytes;
        const uint8_t* src = L->rank == owner ? static_cast<const uint8_t*>(o.q) + (size_t)local * nbytes : dst;
        DMOE_NCCL(api.Broadcast(src, dst, nbytes, ncclUint8, owner, L->comm, st), "ncclBroadcast(expert weights)");
        if (o.type == DMOE_TYPE_Q8_0) {
          const size_t ns = (size_t)rpe[f] * (o.k / 32);
          float* sd = nw[f].s + (size_t)(El + j) * ns;
          const float* ss = L->rank == owner ? o.s + (size_t)local * ns : sd;
          DMOE_NCCL(api.Broadcast(ss, sd, ns, ncclFloat32, owner, L->comm, st), "ncclBroadcast(expert scales)");
        }
      }
    }
    DMOE_NCCL(api.GroupEnd(), "replica broadcast");
  }
  if ((s = ep_wait(L, st, "replica broadcast")) != DMOE_OK) {
    drop_new();
    return s;
  }
  for (int f = 0; f < 3; ++f)
    if ((s = map_weight(nw[f])) != DMOE_OK) {
      drop_new();
      return s;
    }
  for (int f = 0; f < 3; ++f) {
    free_weight(*fam[f]);
    *fam[f] = nw[f];
  }
  std::vector<int32_t> slot((size_t)E, -1);
  for (int j = 0; j < n_hot; ++j) slot[(size_t)chosen[(size_t)j]] = j;
  DMOE_CUDA(cudaMemcpy(L->hot_slot, slot.data(), sizeof(int32_t) * (size_t)E, cudaMemcpyHostToDevice));
  L->n_hot = n_hot;
  L->hot_ids = chosen;
  L->last_stream = st;
  return DMOE_OK;
}

dmoe_status dmoe_get_stats(const dmoe_layer* L, dmoe_stats* s) {
  if (!L || !s) return fail(DMOE_ERR_INVALID_ARG, "null argument");
  *s = L->stats;
  return DMOE_OK;
}

}  // extern "C"
