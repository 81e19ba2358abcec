// noalloc.cu — routing without any device allocation (dmoe_route_static).
//
// Some callers cannot call cudaMalloc at all: a process whose device memory is owned by another
// allocator (a serving stack that reserves its whole budget at start-up, or a host framework
// that hands out every buffer itself) may forbid any allocation outside that allocator. For
// them this entry point runs the router (the same kernels and canonical arithmetic as
// dmoe_forward with DMOE_F_ROUTE_ONLY) with its working memory in a fixed array that is part
// of the library image, so the call itself allocates nothing.
//
// The array is a file-scope __device__ object: every GPU that loads the library holds its
// DMOE_STATIC_SCRATCH_BYTES until the process exits. Its name is only a host-side stand-in in
// host code, so the device address is looked up once per device with cudaGetSymbolAddress (on
// the first call made on that device, with that device current) and passed to the kernels.
// All calls share the one array and it keeps the previous call's contents: the per-expert
// counters are cleared on every call, and calls that overlap on the GPU (other streams, other
// threads) race on it.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/diffuse_moe.h"
#include "dmoe_internal.h"

namespace dmoe {

namespace {

constexpr int64_t kStaticMaxTokens = DMOE_STATIC_MAX_TOKENS;
constexpr int64_t kStaticMaxExperts = DMOE_STATIC_MAX_EXPERTS;
constexpr int64_t kStaticMaxEmbd = DMOE_STATIC_MAX_EMBD;

// layout (floats): logits [T][E] | router weight transposed [H][E] | counts [E]
constexpr size_t kLogitsOff = 0;
constexpr size_t kWrtOff = kLogitsOff + (size_t)kStaticMaxTokens * kStaticMaxExperts;
constexpr size_t kCountsOff = kWrtOff + (size_t)kStaticMaxEmbd * kStaticMaxExperts;
constexpr size_t kScratchFloats = kCountsOff + (size_t)kStaticMaxExperts;
static_assert(kScratchFloats * sizeof(float) == DMOE_STATIC_SCRATCH_BYTES, "header states the scratch size");

static __device__ __align__(256) float g_route_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_route_scratch on the current device (looked up once per device).
cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_route_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

// w [e][h] (GGUF ne = [H, E]) -> wt [h][e], the layout the logits kernel reads.
__global__ void transpose_router_kernel(const float* __restrict__ w, float* __restrict__ wt, int e, int h) {
  __shared__ float tile[32][33];
  const int h0 = blockIdx.x * 32, e0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int ee = e0 + r, hh = h0 + threadIdx.x;
    tile[r][threadIdx.x] = (ee < e && hh < h) ? w[(int64_t)ee * h + hh] : 0.0f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int hh = h0 + r, ee = e0 + threadIdx.x;
    if (hh < h && ee < e) wt[(int64_t)hh * e + ee] = tile[threadIdx.x][r];
  }
}

}  // namespace
}  // namespace dmoe

using namespace dmoe;

extern "C" dmoe_status dmoe_route_static(const float* x, int64_t n_tokens, int64_t n_embd, const float* w_router,
                                         const float* b_router, int64_t n_expert, int64_t n_expert_used,
                                         int64_t expert_capacity, int64_t moe_block_size, float routed_scaling,
                                         int32_t norm_topk_prob, int32_t* idx, float* weights, void* stream) {
  char msg[256];
  if (n_tokens < 0 || n_embd <= 0 || n_expert <= 0 || n_expert_used <= 0 || expert_capacity < 0 ||
      moe_block_size < 0) {
    set_last_error("dmoe_route_static: non-positive size");
    return DMOE_ERR_INVALID_ARG;
  }
  if (n_tokens > kStaticMaxTokens || n_expert > kStaticMaxExperts || n_embd > kStaticMaxEmbd) {
    snprintf(msg, sizeof(msg),
             "dmoe_route_static: n_tokens %lld / n_expert %lld / n_embd %lld exceed the fixed scratch limits "
             "%lld / %lld / %lld",
             (long long)n_tokens, (long long)n_expert, (long long)n_embd, (long long)kStaticMaxTokens,
             (long long)kStaticMaxExperts, (long long)kStaticMaxEmbd);
    set_last_error(msg);
    return DMOE_ERR_UNSUPPORTED;
  }
  if (n_embd % kRouterSeg || n_expert % 4 || n_expert_used > 16 || n_expert_used > n_expert) {
    set_last_error("dmoe_route_static: n_embd must be a multiple of 256, n_expert of 4, n_expert_used <= 16");
    return DMOE_ERR_UNSUPPORTED;
  }
  // block routing switch (src/diffuse-moe-graph.cpp:215-216); without it the routing kernel
  // runs 32-token CTAs whatever moe_block_size is
  const bool use_block = moe_block_size > 1 && expert_capacity > 0 && expert_capacity < n_expert &&
                         n_tokens % moe_block_size == 0;
  if (route_smem_bytes(use_block ? moe_block_size : 32, n_expert) > kRouteSmemMax) {
    set_last_error("dmoe_route_static: moe_block_size x n_expert too large for the routing kernel");
    return DMOE_ERR_UNSUPPORTED;
  }
  if (n_tokens > 0 && (!x || !w_router || !idx || !weights)) {
    set_last_error("dmoe_route_static: null pointer");
    return DMOE_ERR_INVALID_ARG;
  }
  // the logits kernel reads x with 16-byte copies and the routing kernel reads the bias as float4
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(b_router)) & 15u ||
      (reinterpret_cast<uintptr_t>(w_router) | reinterpret_cast<uintptr_t>(idx) |
       reinterpret_cast<uintptr_t>(weights)) & 3u) {
    set_last_error("dmoe_route_static: x and b_router must be 16-byte aligned, w_router / idx / weights 4-byte aligned");
    return DMOE_ERR_INVALID_ARG;
  }
  if (n_tokens == 0) return DMOE_OK;
  float* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "dmoe_route_static: scratch address lookup failed: %s", cudaGetErrorString(e));
    set_last_error(msg);
    return DMOE_ERR_CUDA;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  set_pdl_for_call(false);
  float* logits = scratch + kLogitsOff;
  float* wrt = scratch + kWrtOff;
  int32_t* counts = reinterpret_cast<int32_t*>(scratch + kCountsOff);
  const int H = (int)n_embd, E = (int)n_expert;
  transpose_router_kernel<<<dim3((unsigned)((H + 31) / 32), (unsigned)((E + 31) / 32)), dim3(32, 8), 0, st>>>(
      w_router, wrt, E, H);
  e = cudaGetLastError();
  if (e == cudaSuccess) e = launch_router(x, wrt, logits, n_tokens, H, E, ROUTER_WHOLE, nullptr, counts, st);
  if (e == cudaSuccess) {
    RouteArgs ra{};
    ra.probs = logits;
    ra.bias = b_router;
    ra.n = n_tokens;
    ra.e = E;
    ra.top_k = (int)n_expert_used;
    ra.cap = (int)expert_capacity;
    ra.blk = (int)moe_block_size;
    ra.use_block = use_block ? 1 : 0;
    ra.norm_topk = norm_topk_prob;
    ra.scale = routed_scaling;
    ra.idx = idx;
    ra.w = weights;
    ra.allowed = nullptr;
    ra.counts = counts;
    e = launch_route(ra, st);
  }
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "dmoe_route_static: launch failed: %s", cudaGetErrorString(e));
    set_last_error(msg);
    return DMOE_ERR_CUDA;
  }
  return DMOE_OK;
}
