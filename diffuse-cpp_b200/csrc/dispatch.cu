// dispatch.cu — token dispatch between the router and the expert GEMMs.
//
// The reference multiplies every (token, slot) pair through ggml_mul_mat_id with the
// expert index per slot (src/diffuse-moe-graph.cpp:265-269). Here the pairs are laid out
// expert-contiguously so each expert's tokens form dense GEMM tiles:
//
//   rows [0, n)                         shared expert: token t at row t (weight 1)
//   rows [n + off[e], n + off[e] + c_e)  routed expert e: its (token, slot) pairs
//
// scan_tiles_kernel  exclusive scan of the per-expert counts + the token-tile list
// gather_kernel      x (fp32) -> fp16 rows of the gathered buffer, pair -> token / weight maps
// swiglu_finish      split-K path: h = silu(g) * u from the fp32 partial sums
// combine_kernel     out[t] = ((y_0 + y_1) + ... + y_{k-1}) + shared[t], the slot sum and the
//                    shared-expert add of src/diffuse-moe-graph.cpp:273-286 in that order
#include "dmoe_internal.h"
#include "sm100.cuh"

namespace dmoe {

// One CTA; e <= 1024 threads (one per expert).
__global__ void __launch_bounds__(1024) scan_tiles_kernel(const int32_t* __restrict__ counts, int e, int64_t n, int nt,
                                                          int32_t* __restrict__ off, int32_t* __restrict__ fill,
                                                          TokTile* __restrict__ tiles, int32_t* __restrict__ n_tiles,
                                                          int32_t* __restrict__ n_active, int32_t* __restrict__ tt_done,
                                                          int n_sh_tt) {
  __shared__ int32_t s_cnt[1024];
  pdl_wait();
  pdl_trigger();
  __shared__ int32_t s_tt[1024];
  const int tid = threadIdx.x;
  const int c = tid < e ? counts[tid] : 0;
  const int tt = (c + nt - 1) / nt;
  s_cnt[tid] = c;
  s_tt[tid] = tt;
  __syncthreads();
  // Hillis-Steele inclusive scans (both arrays)
  for (int o = 1; o < 1024; o <<= 1) {
    const int a = tid >= o ? s_cnt[tid - o] : 0;
    const int b = tid >= o ? s_tt[tid - o] : 0;
    __syncthreads();
    s_cnt[tid] += a;
    s_tt[tid] += b;
    __syncthreads();
  }
  const int excl_c = s_cnt[tid] - c;
  const int excl_t = s_tt[tid] - tt;
  if (tid < e) {
    off[tid] = (int32_t)n + excl_c;
    fill[tid] = 0;
    for (int j = 0; j < tt; ++j) {
      TokTile t;
      t.expert = tid;
      t.row0 = (int32_t)n + excl_c + j * nt;
      t.nrows = min(nt, c - j * nt);
      t.pad = 0;
      tiles[excl_t + j] = t;
    }
  }
  if (tid == 1023) {
    *n_tiles = s_tt[1023];
  }
  if (tt_done)  // the fused GEMM's per-token-tile completion counters
    for (int i = tid; i < n_sh_tt + s_tt[1023]; i += 1024) tt_done[i] = 0;
  // active expert count (experts with at least one pair)
  __syncthreads();
  s_cnt[tid] = (tid < e && c > 0) ? 1 : 0;
  __syncthreads();
  for (int o = 512; o > 0; o >>= 1) {
    if (tid < o) s_cnt[tid] += s_cnt[tid + o];
    __syncthreads();
  }
  if (tid == 0) *n_active = s_cnt[0];
}

// One CTA per token. Writes the token's fp16 row to the shared-expert segment and to each of
// its routed pairs. `swap_shared` / `swap_routed` select the q4_K K order (elements 1 and 2 of
// each quad swapped) for rows that feed a q4_K weight matrix.
__global__ void __launch_bounds__(256) gather_kernel(const float* __restrict__ x, int64_t n, int h, int top_k,
                                                     const int32_t* __restrict__ idx, const float* __restrict__ w,
                                                     const int32_t* __restrict__ off, int32_t* __restrict__ fill,
                                                     __half* __restrict__ xg, int32_t* __restrict__ pair_tok,
                                                     float* __restrict__ pair_w, int32_t* __restrict__ pair_row,
                                                     int swap_shared, int swap_routed, int with_shared,
                                                     float* __restrict__ zero_out) {
  __shared__ int64_t rows[kMaxTopK + 1];
  pdl_wait();
  pdl_trigger();
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const int r0 = with_shared ? 1 : 0;
  if (tid == 0 && with_shared) rows[0] = t;
  if (tid < top_k) {  // one lane per slot: the slots' atomics are in flight together
    const int s = tid;
    const int ee = idx[t * top_k + s];
    const int64_t pos = off[ee] + atomicAdd(&fill[ee], 1);
    pair_tok[pos] = (int32_t)t;
    pair_w[pos] = w[t * top_k + s];
    pair_row[t * top_k + s] = (int32_t)pos;
    rows[r0 + s] = pos;
  }
  __syncthreads();
  const int nrows = r0 + top_k;
  const float4* xr = reinterpret_cast<const float4*>(x + t * h);
  for (int q = tid; q < h / 4; q += blockDim.x) {
    const float4 v = xr[q];
    const __half2 a0 = __floats2half2_rn(v.x, v.y), b0 = __floats2half2_rn(v.z, v.w);  // natural
    const __half2 a1 = __floats2half2_rn(v.x, v.z), b1 = __floats2half2_rn(v.y, v.w);  // quad swap
    uint2 pk_nat, pk_swp;
    memcpy(&pk_nat.x, &a0, 4);
    memcpy(&pk_nat.y, &b0, 4);
    memcpy(&pk_swp.x, &a1, 4);
    memcpy(&pk_swp.y, &b1, 4);
    for (int r = 0; r < nrows; ++r) {
      const bool shared_row = with_shared && r == 0;
      const bool swp = shared_row ? swap_shared : swap_routed;
      reinterpret_cast<uint2*>(xg + rows[r] * h)[q] = swp ? pk_swp : pk_nat;
    }
    if (zero_out) reinterpret_cast<float4*>(zero_out + t * h)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

__device__ __forceinline__ int quad_swap_i(int i) { return (i & ~3) | ((i & 1) << 1) | ((i >> 1) & 1); }

// h[r][i'] = silu(g[r][i]) * u[r][i] for rows [0, rows) and i < width_of(row): shared rows
// (r < n) have width is, routed rows width i.
__global__ void swiglu_finish_kernel(const float* __restrict__ gu, int64_t gu_half, int64_t rows, int64_t n, int is,
                                     int iw, __half* __restrict__ hbuf, int64_t h_ld, int swap_shared,
                                     int swap_routed) {
  const int64_t r = blockIdx.x;
  if (r >= rows) return;
  const int width = r < n ? is : iw;
  const float* g = gu + r * 2 * gu_half;
  const float* u = g + gu_half;
  const bool swp = r < n ? swap_shared : swap_routed;
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const float gv = g[i];
    const float hv = gv / (1.0f + __expf(-gv)) * u[i];
    hbuf[r * h_ld + (swp ? quad_swap_i(i) : i)] = __float2half_rn(hv);
  }
}

// One CTA per token. y holds the weighted routed rows (row r of the gathered layout at
// y + (r - n) * y_ld); out holds the shared expert's rows when add_out is set.
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ y, int64_t y_ld, int64_t n,
                                                      const int32_t* __restrict__ pair_row, int top_k,
                                                      float* __restrict__ out, int64_t h, int add_out) {
  __shared__ int64_t rows[kMaxTopK];
  pdl_wait();
  pdl_trigger();
  const int64_t t = blockIdx.x;
  if (threadIdx.x < top_k) rows[threadIdx.x] = (int64_t)(pair_row[t * top_k + threadIdx.x] - n) * y_ld;
  __syncthreads();
  float4* o = reinterpret_cast<float4*>(out + t * h);
  for (int64_t q = threadIdx.x; q < h / 4; q += blockDim.x) {
    float4 v[kMaxTopK];
#pragma unroll
    for (int s = 0; s < kMaxTopK; ++s)
      if (s < top_k) v[s] = __ldcs(reinterpret_cast<const float4*>(y + rows[s]) + q);
    float4 a = v[0];
#pragma unroll
    for (int s = 1; s < kMaxTopK; ++s)
      if (s < top_k) {
        a.x = __fadd_rn(a.x, v[s].x);
        a.y = __fadd_rn(a.y, v[s].y);
        a.z = __fadd_rn(a.z, v[s].z);
        a.w = __fadd_rn(a.w, v[s].w);
      }
    if (add_out) {
      const float4 b = o[q];
      a.x = __fadd_rn(a.x, b.x);
      a.y = __fadd_rn(a.y, b.y);
      a.z = __fadd_rn(a.z, b.z);
      a.w = __fadd_rn(a.w, b.w);
    }
    o[q] = a;
  }
}

cudaError_t launch_combine(const float* y, int64_t y_ld, int64_t n, const int32_t* pair_row, int top_k, float* out,
                           int64_t h, int add_out, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  if (top_k < 1 || top_k > kMaxTopK || h % 4) return cudaErrorInvalidValue;
  return launch_pdl(combine_kernel, dim3((unsigned)n), dim3(256), 0, st, y, y_ld, n, pair_row, top_k, out, h, add_out);
}

cudaError_t launch_scan_tiles(const int32_t* counts, int e, int64_t n, int nt, int32_t* off, int32_t* fill,
                              TokTile* tiles, int32_t* n_tiles, int32_t* n_active, int32_t* tt_done, int n_sh_tt,
                              cudaStream_t st) {
  return launch_pdl(scan_tiles_kernel, dim3(1), dim3(1024), 0, st, counts, e, n, nt, off, fill, tiles, n_tiles, n_active,
                    tt_done, n_sh_tt);
}

cudaError_t launch_gather(const float* x, int64_t n, int h, int top_k, const int32_t* idx, const float* w,
                          const int32_t* off, int32_t* fill, __half* xg, int32_t* pair_tok, float* pair_w,
                          int32_t* pair_row, int swap_shared, int swap_routed, int with_shared, float* zero_out,
                          cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  return launch_pdl(gather_kernel, dim3((unsigned)n), dim3(256), 0, st, x, n, h, top_k, idx, w, off, fill, xg, pair_tok,
                    pair_w, pair_row, swap_shared, swap_routed, with_shared, zero_out);
}

cudaError_t launch_swiglu_finish(const float* gu, int64_t gu_half, int64_t rows, int64_t n, int is, int iw,
                                 __half* hbuf, int64_t h_ld, int swap_shared, int swap_routed, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  swiglu_finish_kernel<<<(unsigned)rows, 256, 0, st>>>(gu, gu_half, rows, n, is, iw, hbuf, h_ld, swap_shared,
                                                       swap_routed);
  return cudaGetLastError();
}

}  // namespace dmoe
