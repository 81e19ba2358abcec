// sampler.cu — one denoising step's greedy sampling and commit on the GPU (dmoe_sample_step).
//
// Reference: src/diffuse-sampler.cpp. For every masked position of the block being denoised,
// sample_token with temperature 0 (:29-49) takes the argmax of the position's logits (a strict
// `>` scan, so the lowest vocabulary index wins a tie) and its probability 1 / sum_v
// exp(l_v - max); the step then sorts the candidates by probability, highest first, and commits
// the first n_transfer of them and every further one whose probability is at least the
// threshold, at least one (:183-237). The reference copies every position's n_vocab logits to
// the host for this (diffuse-moe-graph.cpp:331-332); here they stay on the device and only the
// committed tokens change.
//
// sample_rows_kernel: one cluster of kClusterCtas CTAs per position. Each CTA scans its slice of
// the row once, keeping a running (max, lowest index of the max, sum of exp(l - max)) per thread
// (the sum is rescaled by exp(old max - new max) when the max grows); the threads' triples merge
// in the CTA, and CTA 0 merges the CTAs' triples (read through distributed shared memory) in a
// fixed shuffle tree.
// The row is read once: the kernel is HBM-bound (4 n_vocab bytes per masked position).
// sample_commit_kernel: one CTA ranks the candidates (probability descending, position ascending
// among equal probabilities, where the reference's std::sort leaves the order unspecified) and
// applies the commit rule.
#include <cstdio>

#include "../../include/diffuse_moe.h"
#include "dmoe_internal.h"
#include "sm100.cuh"

namespace dmoe {

namespace {

constexpr int kClusterCtas = 8;
constexpr int kRowThreads = 512;
constexpr int kCommitThreads = 1024;
constexpr int kUnroll = 10;  // 16-byte loads in flight per thread: a 157,184-value row in one batch
static_assert(DMOE_SAMPLE_MAX_POS <= kCommitThreads, "one commit thread per position");

struct Best {
  float m;    // running max
  int32_t i;  // lowest index holding it
  float s;    // sum of exp(l - m)
};

// Merge of two partial triples; `a` covers lower indices than `b` only matters for equal maxima,
// where the lower index is kept either way.
__device__ __forceinline__ Best merge(Best a, Best b) {
  if (b.s == 0.0f) return a;  // empty partial
  if (a.s == 0.0f) return b;
  Best r;
  if (a.m > b.m) {
    r.m = a.m;
    r.i = a.i;
    r.s = a.s + b.s * expf(b.m - a.m);
  } else if (b.m > a.m) {
    r.m = b.m;
    r.i = b.i;
    r.s = b.s + a.s * expf(a.m - b.m);
  } else {
    r.m = a.m;
    r.i = min(a.i, b.i);
    r.s = a.s + b.s;
  }
  return r;
}

__device__ __forceinline__ void visit(Best& t, float x, int32_t v) {
  if (x > t.m) {  // strict: an equal later value keeps the earlier index
    t.s = t.s * expf(t.m - x) + 1.0f;
    t.m = x;
    t.i = v;
  } else {
    t.s += expf(x - t.m);
  }
}

__device__ __forceinline__ Best shfl_best(Best b, int off) {
  Best r;
  r.m = __shfl_down_sync(0xffffffffu, b.m, off);
  r.i = __shfl_down_sync(0xffffffffu, b.i, off);
  r.s = __shfl_down_sync(0xffffffffu, b.s, off);
  return r;
}

// grid (kClusterCtas, n_pos), clusters of kClusterCtas along x: cluster = one position.
__global__ void __cluster_dims__(kClusterCtas, 1, 1) __launch_bounds__(kRowThreads)
    sample_rows_kernel(const float* __restrict__ logits, int64_t n_vocab, const int32_t* __restrict__ seq,
                       int32_t mask_id, int32_t* __restrict__ token, float* __restrict__ prob) {
  __shared__ Best warp_best[kRowThreads / 32];
  __shared__ Best cta_best;
  const int64_t row = blockIdx.y;
  const uint32_t rank = cluster_ctarank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // the whole cluster sees the same position: it leaves together, before any cluster barrier
  if (seq && seq[row] != mask_id) {
    if (rank == 0 && tid == 0) {
      token[row] = -1;
      prob[row] = 0.0f;
    }
    return;
  }
  // this CTA's slice: whole float4s, the ragged tail in the last slice
  const int64_t per = ((n_vocab + kClusterCtas - 1) / kClusterCtas + 3) & ~int64_t(3);
  const int64_t v0 = (int64_t)rank * per, v1 = min(n_vocab, v0 + per);
  const float* r = logits + row * n_vocab;
  Best t{-INFINITY, 0, 0.0f};
  if (v0 < v1) {
    // thread tid takes the 4-value groups tid, tid + 512, ... of the slice (increasing indices
    // within a thread), as one float4 load where the row is 16-byte aligned and as four loads
    // where it is not: the same values in the same order either way, so equal rows give equal bits
    // kUnroll groups are loaded before any is consumed (enough bytes in flight to cover the
    // memory latency), then visited in index order
    const int64_t n4 = (v1 - v0) / 4;
    const bool vec = ((reinterpret_cast<uintptr_t>(r + v0) & 15) == 0);
    for (int64_t q0 = tid; q0 < n4; q0 += kUnroll * kRowThreads) {
      float4 x[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t q = q0 + (int64_t)u * kRowThreads;
        const int64_t b = v0 + 4 * q;
        if (q >= n4) {
          x[u] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        } else if (vec) {
          x[u] = __ldcs(reinterpret_cast<const float4*>(r + b));
        } else {
          x[u].x = __ldcs(r + b);
          x[u].y = __ldcs(r + b + 1);
          x[u].z = __ldcs(r + b + 2);
          x[u].w = __ldcs(r + b + 3);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t q = q0 + (int64_t)u * kRowThreads;
        if (q >= n4) break;
        const int32_t b = (int32_t)(v0 + 4 * q);
        visit(t, x[u].x, b);
        visit(t, x[u].y, b + 1);
        visit(t, x[u].z, b + 2);
        visit(t, x[u].w, b + 3);
      }
    }
    for (int64_t q = v0 + 4 * n4 + tid; q < v1; q += kRowThreads) visit(t, __ldcs(r + q), (int32_t)q);
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) t = merge(t, shfl_best(t, off));
  if (lane == 0) warp_best[warp] = t;
  __syncthreads();
  if (warp == 0) {
    t = lane < kRowThreads / 32 ? warp_best[lane] : Best{-INFINITY, 0, 0.0f};
#pragma unroll
    for (int off = 16; off; off >>= 1) t = merge(t, shfl_best(t, off));
    if (lane == 0) cta_best = t;
  }
  cluster_sync();  // every CTA's cta_best is written
  if (rank == 0 && warp == 0) {
    // lane c < kClusterCtas reads CTA c's triple (all at once), then a fixed shuffle tree merges
    // them: the same order every time, so the bits do not depend on timing
    Best o{-INFINITY, 0, 0.0f};
    if (lane < kClusterCtas) {
      const uint32_t a = mapa_shared(smem_u32(&cta_best), (uint32_t)lane);
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(o.m) : "r"(a));
      asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(o.i) : "r"(a + 4));
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(o.s) : "r"(a + 8));
    }
#pragma unroll
    for (int off = kClusterCtas / 2; off; off >>= 1) o = merge(o, shfl_best(o, off));
    if (lane == 0) {
      token[row] = o.i;
      prob[row] = 1.0f / o.s;  // exp(max - max) / sum
    }
  }
  cluster_sync();  // CTA 0 has read every peer's shared memory before they exit
  pdl_trigger();
}

// One CTA: rank the candidates and commit (src/diffuse-sampler.cpp:212-237).
__global__ void __launch_bounds__(kCommitThreads)
    sample_commit_kernel(int n_pos, int32_t* __restrict__ seq, const int32_t* __restrict__ token,
                         const float* __restrict__ prob, int32_t n_transfer, float threshold,
                         int32_t* __restrict__ n_committed) {
  __shared__ float p_s[kCommitThreads];
  __shared__ int32_t cand_s[kCommitThreads];
  __shared__ int32_t committed, top;
  const int i = threadIdx.x;
  pdl_wait();  // the rows kernel's token / prob are complete and visible
  const bool cand = i < n_pos && token[i] >= 0;
  const float p = cand ? prob[i] : 0.0f;
  p_s[i] = p;
  cand_s[i] = cand ? 1 : 0;
  if (i == 0) {
    committed = 0;
    top = -1;
  }
  __syncthreads();
  int rank = 0;
  if (cand)
    for (int j = 0; j < n_pos; ++j)
      rank += (cand_s[j] && (p_s[j] > p || (p_s[j] == p && j < i))) ? 1 : 0;
  // sorted order: the first n_transfer always; after them, the loop runs while prob >= threshold,
  // and every candidate before one at or above it is at or above it too
  const bool take = cand && (rank < n_transfer || p >= threshold);
  if (take) {
    seq[i] = token[i];
    atomicAdd(&committed, 1);
  }
  if (cand && rank == 0) top = i;
  __syncthreads();
  if (i == 0) {
    int c = committed;
    if (c == 0 && top >= 0) {  // at least one (:231-235)
      seq[top] = token[top];
      c = 1;
    }
    if (n_committed) *n_committed = c;
  }
}

}  // namespace

}  // namespace dmoe

using namespace dmoe;

extern "C" dmoe_status dmoe_sample_step(const float* logits, int64_t n_pos, int64_t n_vocab, int32_t* seq,
                                        int32_t mask_id, int32_t n_transfer, float threshold, int32_t* token,
                                        float* prob, int32_t* n_committed, void* stream) {
  char msg[256];
  if (n_pos < 0 || n_vocab <= 0 || n_vocab > INT32_MAX) {
    set_last_error("dmoe_sample_step: n_pos must be >= 0 and 0 < n_vocab < 2^31");
    return DMOE_ERR_INVALID_ARG;
  }
  if (n_pos > DMOE_SAMPLE_MAX_POS) {
    snprintf(msg, sizeof(msg), "dmoe_sample_step: n_pos %lld above %d", (long long)n_pos, DMOE_SAMPLE_MAX_POS);
    set_last_error(msg);
    return DMOE_ERR_UNSUPPORTED;
  }
  if (n_pos > 0 && (!logits || !token || !prob)) {
    set_last_error("dmoe_sample_step: null pointer");
    return DMOE_ERR_INVALID_ARG;
  }
  if (n_pos == 0) return DMOE_OK;
  const NvtxRange nvtx_call("dmoe_sample_step");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  sample_rows_kernel<<<dim3(kClusterCtas, (unsigned)n_pos), dim3(kRowThreads), 0, st>>>(logits, n_vocab, seq, mask_id,
                                                                                      token, prob);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && seq) {
    // programmatic dependent launch: the commit CTA starts while the rows kernel drains and
    // waits for it in griddepcontrol.wait
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kCommitThreads);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, sample_commit_kernel, (int)n_pos, seq, (const int32_t*)token, (const float*)prob,
                           n_transfer, threshold, n_committed);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "dmoe_sample_step: launch failed: %s", cudaGetErrorString(e));
    set_last_error(msg);
    return DMOE_ERR_CUDA;
  }
  return DMOE_OK;
}
