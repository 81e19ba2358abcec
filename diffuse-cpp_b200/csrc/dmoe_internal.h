// dmoe_internal.h — device-side parameter blocks shared by the host library and the kernels.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <nvtx3/nvToolsExt.h>

#include <cstdint>
#include <utility>

#include "tile_check.h"

namespace dmoe {

// ggml_type ids of the formats on this path (ggml.h enum ggml_type)
enum WType : int { WT_F32 = 0, WT_F16 = 1, WT_Q8_0 = 8, WT_Q4_K = 12 };

// The GEMM kernel's two epilogues.
// MODE_FUSED: one launch runs every gate/up tile, then every down tile (token tiles <= 64).
enum GemmMode : int { MODE_GATEUP = 0, MODE_DOWN = 1, MODE_FUSED = 2 };

constexpr int kRouterSeg = 256;  // canonical router segment length (fma chain per segment)
constexpr int kMTile = 128;      // weight rows per MMA tile (tcgen05 M)
constexpr int kMaxTopK = 16;     // n_expert_used limit
constexpr int kMaxRanks = 32;    // expert-parallel world size limit (one mask bit per rank)

// Per-rank row offsets, passed by value to the expert-parallel kernels.
struct RankOffsets {
  int32_t v[kMaxRanks];
};

// A weight family processed by one GEMM launch. Group 0 is the shared expert (token rows
// [0, n_tokens) in natural order, weight 1), group 1 the routed experts (token tiles from the
// device tile list). Every flattened tile index maps to (group, token tile, m-tile, k-split).
struct GemmGroup {
  int32_t n_mt;          // output m-tiles per expert (rows_out / 128)
  int32_t k_stages;      // K / STAGE_K
  int32_t rows_per_exp;  // weight rows per expert in the tensor map (row coordinate stride)
  int32_t present;       // 0 if this group has no work
};

struct GemmParams {
  CUtensorMap tm_w[2][2];  // [group][matrix] quant / f16 tiles
  CUtensorMap tm_s[2][2];  // [group][matrix] q8_0 scale tiles (fp32, repacked)
  CUtensorMap tm_b;        // fp16 activations [rows][K] (xg for gate/up, hbuf for down)
  GemmGroup grp[2];
  const TokTile* tiles;        // routed token tiles (device)
  const int32_t* n_tiles;      // number of routed token tiles (device)
  int32_t n_shared_tt;         // shared-expert token tiles (host-known: ceil(N / NT))
  int32_t ksplit;              // split-K factor
  int32_t w_keep;              // 1: weight tiles are re-read by several token tiles (L2 evict normal)
  int64_t n_tokens;
  // gate/up epilogue
  __half* hbuf;
  int64_t h_ld;
  int32_t h_quad_swap;  // bit g: group g's down matrix is q4_K, write its h with the quad swap
  float* gu_acc;        // split-K partial accumulators [rows][2 * gu_half], or null
  int64_t gu_half;
  // down epilogue: with y == null every row is reduced into out (fp32 vector atomics);
  // otherwise shared rows store into out and routed row r stores w_r * (W_d h_r) into
  // y[r - n_tokens] for combine_kernel (deterministic slot-order sum)
  float* out;           // shared rows (group 0), token = row
  int64_t out_ld;
  float* out_routed;    // routed rows (group 1) reduce into out_routed[pair_tok[r]] (atomic path)
  float* y;
  int64_t y_ld;
  const int32_t* pair_tok;
  const float* pair_w;
  // fused launch: the down phase's operands (tiles numbered after all gate/up tiles) and, per
  // token tile (shared tiles first, then routed), the gate/up epilogue warps that have written
  // its h rows; a down tile starts once all of them have (zeroed by scan_tiles_kernel)
  CUtensorMap tm_w_dn[2];  // [group] down weight (quant / f16)
  CUtensorMap tm_s_dn[2];  // [group] q8_0 scales
  CUtensorMap tm_b_dn;     // fp16 h rows
  GemmGroup grp_dn[2];
  int32_t* tt_done;
  uint32_t* err;
  // bounds of the routed token tiles (built on the device): rows [n_tokens, rows_total) and
  // experts [0, n_experts) of group 1; a tile outside them is skipped and reported
  int64_t rows_total;
  int32_t n_experts;
  int32_t tiles_cap;  // capacity of `tiles` and of the routed part of `tt_done`: the count is clamped to it
  // resident-activation down launches (BRES): each routed list tile splits into tile_div tiles of
  // the launch's NT rows; a unit (group, token tile) runs its m-tiles in bres_chunks chunks
  int32_t tile_div;
  int32_t bres_chunks;
};

// Router: one routing block per CTA (src/diffuse-moe-graph.cpp:203-262).
struct RouteArgs {
  const float* probs;  // [n][e] p = sigmoid(router logit), canonical bits
  const float* bias;   // [e] expert bias for the selection, or null
  int64_t n;
  int e, top_k, cap, blk;
  int use_block;       // block routing switch, evaluated on the host (:215-216)
  int norm_topk;
  float scale;
  int32_t* idx;        // [n][top_k]
  float* w;            // [n][top_k]
  uint8_t* allowed;    // [n / blk][e] or null
  int32_t* counts;     // [e] per-expert pair counts (atomics; zeroed by the caller)
  int tok_split;       // CTAs per routing block (set by launch_route)
};

// router logits launch: whole-K 128- or 112-token tiles, or per-256-k-segment partials of 128-
// or 32-token tiles summed by each tile's last CTA (part[1 ..] and `arrivals` in use)
enum RouterPlan { ROUTER_WHOLE = 0, ROUTER_SPLIT2 = 1, ROUTER_SPLIT8 = 2, ROUTER_WHOLE7 = 3 };
cudaError_t launch_router(const float* x, const float* wrt, float* part, int64_t n, int h, int e, RouterPlan plan,
                          int32_t* arrivals, int32_t* zero_counts, cudaStream_t st);
RouterPlan router_plan(int64_t n, int e, int h, int sms);
int64_t router_arrivals(int64_t n, int e);  // split plans: per-tile arrival counters needed
// shared memory of route_kernel for `tpb` tokens per CTA and e experts; at most kRouteSmemMax
constexpr size_t kRouteSmemMax = 200 * 1024;
size_t route_smem_bytes(int64_t tpb, int64_t e);
cudaError_t launch_route(const RouteArgs& a, cudaStream_t st);
cudaError_t launch_scan_tiles(const int32_t* counts, int e, int64_t n, int nt, int32_t* off, int32_t* fill,
                              TokTile* tiles, int32_t* n_tiles, int32_t* n_active, int32_t* tt_done, int n_sh_tt,
                              cudaStream_t st);
cudaError_t launch_gather(const float* x, int64_t n, int h, int top_k, const int32_t* idx, const float* w,
                          const int32_t* off, int32_t* fill, __half* xg, int32_t* pair_tok, float* pair_w,
                          int32_t* pair_row, int swap_shared, int swap_routed, int with_shared, float* zero_out,
                          cudaStream_t st);
cudaError_t launch_combine(const float* y, int64_t y_ld, int64_t n, const int32_t* pair_row, int top_k, float* out,
                           int64_t h, int add_out, cudaStream_t st);
// expert parallelism (ep.cu)
// hot_slot: [n_expert] replica slot of each expert held by every rank, -1 otherwise (or null)
cudaError_t launch_ep_plan(const int32_t* idx, int64_t n, int top_k, int e_local, const int32_t* hot_slot,
                           int my_rank, int world, uint32_t* mask, int32_t* pos, int32_t* cnt, int cnt_stride,
                           cudaStream_t st);
cudaError_t launch_ep_pack(const float* x, int64_t n, int h, int top_k, const int32_t* idx, const float* w,
                           int e_local, const int32_t* hot_slot, int my_rank, const uint32_t* mask, const int32_t* pos,
                           const RankOffsets& soff, int swap, __half* xs, int32_t* meta, cudaStream_t st);
cudaError_t launch_ep_count(const int32_t* meta, int64_t rows, int top_k, int32_t* counts, cudaStream_t st);
cudaError_t launch_gather_rows(const __half* xr, int64_t rows, int h, int top_k, const int32_t* meta,
                               const int32_t* off, int32_t* fill, __half* xg, int32_t* pair_tok, float* pair_w,
                               cudaStream_t st);
cudaError_t launch_gather_shared(const float* x, int64_t n, int h, int swap, __half* xg, cudaStream_t st);
cudaError_t launch_ep_final(float* out, const float* back, int64_t n, int h, const uint32_t* mask, const int32_t* pos,
                            const RankOffsets& soff, cudaStream_t st);
cudaError_t launch_swiglu_finish(const float* gu, int64_t gu_half, int64_t rows, int64_t n, int is, int iw,
                                 __half* hbuf, int64_t h_ld, int swap_shared, int swap_routed, cudaStream_t st);
// pair: clusters of two CTAs sharing 256-row tiles (tcgen05 cta_group::2); gemm_pair_ok says
// which launches have that form (quantised weights, NT = 128, separate gate/up and down launches)
cudaError_t launch_moe_gemm(int wtype, int mode, int nt, int ndq, bool pair, const GemmParams& p, int grid,
                            cudaStream_t st);
bool gemm_pair_ok(int wtype, int mode, int nt);
// down launch with resident activation tiles (quantised weights), kBresNT token rows per CTA,
// K <= kBresK: single CTAs on token tiles of kBresNT rows, or (pair) CTA pairs on token tiles of
// 2 kBresNT rows; p.tile_div = list tile rows / launch tile rows, p.bres_chunks = m-chunks per
// token tile
constexpr int kBresNT = 64;
constexpr int kBresK = 1024;
cudaError_t launch_moe_gemm_bres(int wtype, bool pair, int ndq, const GemmParams& p, int grid, cudaStream_t st);
int gemm_stage_k(int wtype);
int gemm_out_rows(int mode, int nt, bool pair);  // output rows per tile of one expert matrix

// Launch with programmatic stream serialization: the kernel may start while its predecessor in
// the stream finishes; every such kernel calls pdl_wait() before touching global memory.
// dmoe_forward turns it on for calls below 1024 tokens on this thread (measured: 2-3 % faster
// at 1-8 blocks, slower from 64 blocks, where early-launched CTAs hold SMs the predecessor's
// later CTAs need); DMOE_PDL=0 in the environment turns it off entirely.
bool pdl_enabled();
void set_pdl_for_call(bool on);
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

// NVTX range over a host scope: the layer's stages show up by name in Nsight timelines and can
// filter ncu captures (--nvtx); a no-op when no tool is attached.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

// records the message returned by dmoe_last_error on this thread (dmoe_api.cu)
void set_last_error(const char* msg);

// host-side codecs (quant.cpp)
uint16_t f32_to_f16_bits(float f);
float f16_bits_to_f32(uint16_t h);
size_t row_size(int32_t type, int64_t k);

}  // namespace dmoe
