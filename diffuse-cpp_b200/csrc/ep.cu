// ep.cu — expert-parallel dispatch and combine kernels (one process per GPU).
//
// Rank d owns experts [d * e_local, (d + 1) * e_local); router, bias and shared expert are
// replicated, and each rank routes its own token blocks (capacity sets are per block, so
// routing needs no communication). One forward on rank r:
//   ep_mask_kernel     mask[t]: bit d set iff a slot of token t selects an expert of rank d
//                      (an expert replicated on every rank counts as this rank's: hot_slot)
//   ep_scan_kernel     pos[d][t]: slot of token t in the rows sent to rank d; cnt[d]
//   (a forward runs these per chunk of its tokens; chunk k's GEMMs overlap the next chunk's
//   dispatch and the previous chunk's combine, which run on a communication stream)
//   ep_pack_kernel     one fp16 row per (token, destination) plus its slot list: the rank-local
//                      expert id (or -1) and the gate weight of each of the top_k slots
//   (NCCL: counts, then rows and slot lists, grouped ncclSend / ncclRecv)
//   ep_count_kernel    pairs per local expert over the received rows
//   gather_rows_kernel / gather_shared_kernel   the gathered GEMM layout (dispatch.cu's rows
//                      [0, n) shared expert, then the routed pairs expert-contiguously)
//   (grouped GEMMs: the down epilogue reduces w * y into one fp32 partial row per received row)
//   (NCCL: partial rows back to their owners, same offsets mirrored)
//   ep_final_kernel    out[t] = (sum over destinations d ascending of partial_d[t]) + shared[t]
#include "dmoe_internal.h"

namespace dmoe {

// Where a (token, slot) is computed: the owner of its expert, or this rank when every rank holds
// a replica of the expert (hot_slot[e] >= 0); and the expert's index among that rank's local
// experts (owned ones first, then the replicas).
struct SlotDest {
  int rank, local;
};
__device__ __forceinline__ SlotDest slot_dest(int e, int e_local, const int32_t* hot_slot, int my_rank) {
  const int hs = hot_slot ? hot_slot[e] : -1;
  if (hs >= 0) return {my_rank, e_local + hs};
  const int d = e / e_local;
  return {d, e - d * e_local};
}

__global__ void ep_mask_kernel(const int32_t* __restrict__ idx, int64_t n, int top_k, int e_local,
                               const int32_t* __restrict__ hot_slot, int my_rank, uint32_t* __restrict__ mask) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n) return;
  uint32_t m = 0;
  for (int s = 0; s < top_k; ++s) m |= 1u << slot_dest(idx[t * top_k + s], e_local, hot_slot, my_rank).rank;
  mask[t] = m;
}

// One CTA (1024 threads) per destination rank: exclusive scan over tokens of bit d; the count
// of rank d goes to cnt[d * cnt_stride] (per-chunk counts interleaved by destination).
__global__ void __launch_bounds__(1024) ep_scan_kernel(const uint32_t* __restrict__ mask, int64_t n,
                                                       int32_t* __restrict__ pos, int32_t* __restrict__ cnt,
                                                       int cnt_stride) {
  __shared__ int32_t warp_sum[32];
  __shared__ int32_t s_total;
  const int d = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int32_t running = 0;
  for (int64_t base = 0; base < n; base += 1024) {
    const int64_t t = base + tid;
    const int bit = t < n ? (int)((mask[t] >> d) & 1u) : 0;
    const uint32_t bal = __ballot_sync(0xffffffffu, bit);
    const int in_warp = __popc(bal & ((1u << lane) - 1u));
    if (lane == 0) warp_sum[warp] = __popc(bal);
    __syncthreads();
    if (warp == 0) {
      const int v = warp_sum[lane];
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      warp_sum[lane] = incl - v;  // exclusive prefix of the warp totals
      if (lane == 31) s_total = incl;
    }
    __syncthreads();
    if (t < n) pos[(int64_t)d * n + t] = bit ? running + warp_sum[warp] + in_warp : -1;
    running += s_total;
    __syncthreads();
  }
  if (tid == 0) cnt[(int64_t)d * cnt_stride] = running;
}

// One CTA per token: its fp16 row (quad-swapped when the routed matrices are q4_K) and slot list
// to every destination in its mask. meta row = top_k int32 local expert ids (-1: other rank)
// followed by top_k fp32 gate weights.
__global__ void __launch_bounds__(256) ep_pack_kernel(const float* __restrict__ x, int64_t n, int h, int top_k,
                                                      const int32_t* __restrict__ idx, const float* __restrict__ w,
                                                      int e_local, const int32_t* __restrict__ hot_slot, int my_rank,
                                                      const uint32_t* __restrict__ mask,
                                                      const int32_t* __restrict__ pos, RankOffsets soff, int swap,
                                                      __half* __restrict__ xs, int32_t* __restrict__ meta) {
  __shared__ int64_t rows[kMaxRanks];
  __shared__ int nrows;
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const uint32_t m = mask[t];
  if (tid == 0) {
    int k = 0;
    for (int d = 0; d < kMaxRanks; ++d)
      if ((m >> d) & 1u) rows[k++] = soff.v[d] + pos[(int64_t)d * n + t];
    nrows = k;
  }
  __syncthreads();
  // slot lists: thread s < top_k handles slot s for every destination
  if (tid < top_k) {
    const SlotDest sd = slot_dest(idx[t * top_k + tid], e_local, hot_slot, my_rank);
    const float wv = w[t * top_k + tid];
    int k = 0;
    for (int d = 0; d < kMaxRanks; ++d) {
      if (!((m >> d) & 1u)) continue;
      int32_t* mr = meta + rows[k] * (2 * top_k);
      mr[tid] = sd.rank == d ? sd.local : -1;
      mr[top_k + tid] = __float_as_int(wv);
      ++k;
    }
  }
  const float4* xr = reinterpret_cast<const float4*>(x + t * h);
  for (int q = tid; q < h / 4; q += blockDim.x) {
    const float4 v = xr[q];
    const __half2 a = swap ? __floats2half2_rn(v.x, v.z) : __floats2half2_rn(v.x, v.y);
    const __half2 b = swap ? __floats2half2_rn(v.y, v.w) : __floats2half2_rn(v.z, v.w);
    uint2 pk;
    memcpy(&pk.x, &a, 4);
    memcpy(&pk.y, &b, 4);
    for (int r = 0; r < nrows; ++r) reinterpret_cast<uint2*>(xs + rows[r] * h)[q] = pk;
  }
}

__global__ void ep_count_kernel(const int32_t* __restrict__ meta, int64_t rows, int top_k,
                                int32_t* __restrict__ counts) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * top_k) return;
  const int64_t r = i / top_k;
  const int s = (int)(i - r * top_k);
  const int e = meta[r * 2 * top_k + s];
  if (e >= 0) atomicAdd(&counts[e], 1);
}

// One CTA per received row: its (already fp16, already swapped) row to each of its local pairs.
__global__ void __launch_bounds__(256) gather_rows_kernel(const __half* __restrict__ xr, int64_t rows, int h,
                                                          int top_k, const int32_t* __restrict__ meta,
                                                          const int32_t* __restrict__ off, int32_t* __restrict__ fill,
                                                          __half* __restrict__ xg, int32_t* __restrict__ pair_tok,
                                                          float* __restrict__ pair_w) {
  __shared__ int64_t dst[kMaxTopK];
  __shared__ int ndst;
  const int64_t r = blockIdx.x;
  const int tid = threadIdx.x;
  if (tid == 0) {
    int k = 0;
    const int32_t* mr = meta + r * 2 * top_k;
    for (int s = 0; s < top_k; ++s) {
      const int e = mr[s];
      if (e < 0) continue;
      const int64_t p = off[e] + atomicAdd(&fill[e], 1);
      pair_tok[p] = (int32_t)r;
      pair_w[p] = __int_as_float(mr[top_k + s]);
      dst[k++] = p;
    }
    ndst = k;
  }
  __syncthreads();
  const uint4* src = reinterpret_cast<const uint4*>(xr + r * h);
  for (int q = tid; q < h / 8; q += blockDim.x) {
    const uint4 v = src[q];
    for (int k = 0; k < ndst; ++k) reinterpret_cast<uint4*>(xg + dst[k] * h)[q] = v;
  }
}

// Shared-expert rows [0, n) of the gathered layout from the local fp32 tokens.
__global__ void __launch_bounds__(256) gather_shared_kernel(const float* __restrict__ x, int64_t n, int h, int swap,
                                                            __half* __restrict__ xg) {
  const int64_t t = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + t * h);
  for (int q = threadIdx.x; q < h / 4; q += blockDim.x) {
    const float4 v = xr[q];
    const __half2 a = swap ? __floats2half2_rn(v.x, v.z) : __floats2half2_rn(v.x, v.y);
    const __half2 b = swap ? __floats2half2_rn(v.y, v.w) : __floats2half2_rn(v.z, v.w);
    uint2 pk;
    memcpy(&pk.x, &a, 4);
    memcpy(&pk.y, &b, 4);
    reinterpret_cast<uint2*>(xg + t * h)[q] = pk;
  }
}

// out[t] = (partial_{d0} + partial_{d1} + ...) + out[t], destinations ascending; out holds the
// shared expert's rows on entry.
__global__ void __launch_bounds__(256) ep_final_kernel(float* __restrict__ out, const float* __restrict__ back,
                                                       int64_t n, int h, const uint32_t* __restrict__ mask,
                                                       const int32_t* __restrict__ pos, RankOffsets soff) {
  __shared__ int64_t rows[kMaxRanks];
  __shared__ int nrows;
  const int64_t t = blockIdx.x;
  if (threadIdx.x == 0) {
    const uint32_t m = mask[t];
    int k = 0;
    for (int d = 0; d < kMaxRanks; ++d)
      if ((m >> d) & 1u) rows[k++] = (int64_t)(soff.v[d] + pos[(int64_t)d * n + t]) * h;
    nrows = k;
  }
  __syncthreads();
  float4* o = reinterpret_cast<float4*>(out + t * h);
  for (int q = threadIdx.x; q < h / 4; q += blockDim.x) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < nrows; ++k) {
      const float4 v = reinterpret_cast<const float4*>(back + rows[k])[q];
      if (k == 0) {
        a = v;
      } else {
        a.x = __fadd_rn(a.x, v.x);
        a.y = __fadd_rn(a.y, v.y);
        a.z = __fadd_rn(a.z, v.z);
        a.w = __fadd_rn(a.w, v.w);
      }
    }
    const float4 sh = o[q];
    if (nrows > 0) {
      a.x = __fadd_rn(a.x, sh.x);
      a.y = __fadd_rn(a.y, sh.y);
      a.z = __fadd_rn(a.z, sh.z);
      a.w = __fadd_rn(a.w, sh.w);
      o[q] = a;
    }
  }
}

cudaError_t launch_ep_plan(const int32_t* idx, int64_t n, int top_k, int e_local, const int32_t* hot_slot,
                           int my_rank, int world, uint32_t* mask, int32_t* pos, int32_t* cnt, int cnt_stride,
                           cudaStream_t st) {
  if (world > kMaxRanks) return cudaErrorInvalidValue;
  if (n > 0)
    ep_mask_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(idx, n, top_k, e_local, hot_slot, my_rank, mask);
  ep_scan_kernel<<<(unsigned)world, 1024, 0, st>>>(mask, n, pos, cnt, cnt_stride);  // n = 0: zero counts
  return cudaGetLastError();
}

cudaError_t launch_ep_pack(const float* x, int64_t n, int h, int top_k, const int32_t* idx, const float* w,
                           int e_local, const int32_t* hot_slot, int my_rank, const uint32_t* mask, const int32_t* pos,
                           const RankOffsets& soff, int swap, __half* xs, int32_t* meta, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  if (top_k > 256) return cudaErrorInvalidValue;
  ep_pack_kernel<<<(unsigned)n, 256, 0, st>>>(x, n, h, top_k, idx, w, e_local, hot_slot, my_rank, mask, pos, soff,
                                              swap, xs, meta);
  return cudaGetLastError();
}

cudaError_t launch_ep_count(const int32_t* meta, int64_t rows, int top_k, int32_t* counts, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  const int64_t items = rows * top_k;
  ep_count_kernel<<<(unsigned)((items + 255) / 256), 256, 0, st>>>(meta, rows, top_k, counts);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(const __half* xr, int64_t rows, int h, int top_k, const int32_t* meta,
                               const int32_t* off, int32_t* fill, __half* xg, int32_t* pair_tok, float* pair_w,
                               cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  if (top_k > kMaxTopK || h % 8) return cudaErrorInvalidValue;
  gather_rows_kernel<<<(unsigned)rows, 256, 0, st>>>(xr, rows, h, top_k, meta, off, fill, xg, pair_tok, pair_w);
  return cudaGetLastError();
}

cudaError_t launch_gather_shared(const float* x, int64_t n, int h, int swap, __half* xg, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  gather_shared_kernel<<<(unsigned)n, 256, 0, st>>>(x, n, h, swap, xg);
  return cudaGetLastError();
}

cudaError_t launch_ep_final(float* out, const float* back, int64_t n, int h, const uint32_t* mask, const int32_t* pos,
                            const RankOffsets& soff, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  ep_final_kernel<<<(unsigned)n, 256, 0, st>>>(out, back, n, h, mask, pos, soff);
  return cudaGetLastError();
}

}  // namespace dmoe
