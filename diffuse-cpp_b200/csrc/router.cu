// router.cu — the MoE router of diffuse-cpp's block-routed layer on sm_100a.
//
// Reference: src/diffuse-moe-graph.cpp:203-262 (router GEMM, sigmoid, expert bias for the
// selection only, per-block capacity mask, per-token top-k, unbiased renormalised weights).
//
// Routing must be bit-exact against the CPU restatement, so every floating-point step below
// uses explicitly rounded intrinsics (no contraction) in this canonical order:
//   logit[n][e] = P_0 + P_1 + ... (float adds, left to right); P_s = fma chain over
//                 h in [256 s, 256 s + 256) in order, starting from 0
//   p   = 1 / (1 + e),  e = (float) exp(-(double) logit)  [own double-precision exp, below]
//   sel = p + bias[e]
//   bmax = sel[t0]; bmax = sel[t] + relu(bmax - sel[t]) for t = t0+1 .. t0+31   (:223-229)
//   thr  = value at position cap-1 of bmax sorted descending                     (:231-236)
//   keep = (bmax - (thr * 1 + (-1e-6f))) > 0;  sel += keep ? 0 : -1e30            (:238-248)
//   idx  = top-k of sel, descending, ties to the lower expert id                   (:252)
//   w    = p[idx] / (float)(sum_s (double) p[idx_s]) * scale                       (:253-262)
#include "dmoe_internal.h"
#include "sm100.cuh"

namespace dmoe {

// ------------------------------------------------------------------------------------------
// exp(-l) as float: Cody-Waite reduction x = k ln2 + r (|r| <= ln2 / 2) and the degree-12
// Taylor polynomial of e^r evaluated by Horner with fused multiply-adds, then scaled by 2^k.
// Written from the series; every operation is IEEE double, so host and device agree bitwise.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ float exp_neg_canonical(float l) {
  const double x = -(double)l;
  if (x > 104.0) return __int_as_float(0x7f800000);
  if (x < -110.0) return 0.0f;
  const double kd = rint(__dmul_rn(x, 1.4426950408889634));
  double r = __fma_rn(-kd, 0x1.62e42fefa39efp-1, x);
  r = __fma_rn(-kd, 2.3190468138462996e-17, r);
  double p = 2.08767569878681e-09;
  p = __fma_rn(p, r, 2.505210838544172e-08);
  p = __fma_rn(p, r, 2.755731922398589e-07);
  p = __fma_rn(p, r, 2.7557319223985893e-06);
  p = __fma_rn(p, r, 2.48015873015873e-05);
  p = __fma_rn(p, r, 0.0001984126984126984);
  p = __fma_rn(p, r, 0.001388888888888889);
  p = __fma_rn(p, r, 0.008333333333333333);
  p = __fma_rn(p, r, 0.041666666666666664);
  p = __fma_rn(p, r, 0.16666666666666666);
  p = __fma_rn(p, r, 0.5);
  p = __fma_rn(p, r, 1.0);
  p = __fma_rn(p, r, 1.0);
  const long long k = (long long)kd;
  const double s = __longlong_as_double((k + 1023ll) << 52);
  return __double2float_rn(__dmul_rn(p, s));
}

__device__ __forceinline__ float sigmoid_canonical(float l) {
  const float e = exp_neg_canonical(l);
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
}

// ------------------------------------------------------------------------------------------
// Router logits: one CTA = 64 threads computing a 32-token x 64-expert tile; thread (ty, tx)
// owns tokens 4 ty .. 4 ty + 3 and experts {4 tx .. 4 tx + 3} u {32 + 4 tx .. 32 + 4 tx + 3}.
// Tiles of x [token][k] and of the transposed router weight wrt [k][expert] (transposed once at
// bind time) arrive by cp.async into a double-buffered shared-memory ring.
//   SPLIT = false: one CTA runs every segment, keeping tot = P_0 + P_1 + ... (large N).
//   SPLIT = true:  one CTA per (tile, segment) writes its segment partial P_s, and
//                  router_finish_kernel sums P_0 .. P_{S-1} left to right (small N, where the
//                  tiles alone cannot fill the GPU).
// Both produce the canonical logits, turned into probs = sigmoid(logit) and selection scores
// sel = probs + bias (src/diffuse-moe-graph.cpp:204-210).
// ------------------------------------------------------------------------------------------
constexpr int RL_TOK = 32, RL_EXP = 64, RL_KC = 64, RL_THREADS = 64;
constexpr int RL_XP = RL_KC + 4;  // x tile row pitch (floats)
constexpr int RL_SMEM = 2 * (RL_TOK * RL_XP + RL_KC * RL_EXP) * 4;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <bool SPLIT>
__global__ void __launch_bounds__(RL_THREADS) router_logits_kernel(const float* __restrict__ x,
                                                                   const float* __restrict__ wrt,
                                                                   const float* __restrict__ bias,
                                                                   float* __restrict__ part, float* __restrict__ probs,
                                                                   float* __restrict__ sel, int64_t n, int h,
                                                                   int e) {
  extern __shared__ __align__(16) float rl_smem[];
  const uint32_t xs0 = smem_u32(rl_smem);                     // [2][32][RL_XP]
  const uint32_t ws0 = xs0 + 2 * RL_TOK * RL_XP * 4;          // [2][64 k][64 e]
  const int tid = threadIdx.x;
  const int ty = tid >> 3, tx = tid & 7;
  const int64_t t0 = (int64_t)blockIdx.x * RL_TOK;
  const int e0 = blockIdx.y * RL_EXP;
  const int nseg = h / kRouterSeg;
  const int s_begin = SPLIT ? (int)blockIdx.z : 0;
  const int s_end = SPLIT ? s_begin + 1 : nseg;
  const int kc0 = s_begin * kRouterSeg, nchunks = (s_end - s_begin) * (kRouterSeg / RL_KC);

  auto load_chunk = [&](int c, int buf) {
    const int kc = kc0 + c * RL_KC;
    const uint32_t xs = xs0 + buf * RL_TOK * RL_XP * 4, ws = ws0 + buf * RL_KC * RL_EXP * 4;
#pragma unroll
    for (int r = 0; r < (RL_TOK * RL_KC / 4) / RL_THREADS; ++r) {  // 8 per thread
      const int q = tid + r * RL_THREADS, t = q >> 4, k4 = q & 15;
      const bool ok = t0 + t < n;
      const float* src = ok ? x + (t0 + t) * h + kc + 4 * k4 : x;
      cp_async16(xs + (t * RL_XP + 4 * k4) * 4, src, ok);
    }
#pragma unroll
    for (int r = 0; r < (RL_KC * RL_EXP / 4) / RL_THREADS; ++r) {  // 16 per thread
      const int q = tid + r * RL_THREADS, k = q >> 4, e4 = q & 15;
      const bool ok = e0 + 4 * e4 < e;
      const float* src = ok ? wrt + (int64_t)(kc + k) * e + e0 + 4 * e4 : wrt;
      cp_async16(ws + (k * RL_EXP + 4 * e4) * 4, src, ok);
    }
    cp_async_commit();
  };

  float tot[4][8], acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) tot[i][j] = acc[i][j] = 0.0f;

  load_chunk(0, 0);
  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    if (c + 1 < nchunks) {
      load_chunk(c + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t xs = xs0 + buf * RL_TOK * RL_XP * 4, ws = ws0 + buf * RL_KC * RL_EXP * 4;
#pragma unroll 2
    for (int k4 = 0; k4 < RL_KC / 4; ++k4) {
      float4 xv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) xv[i] = lds128f(xs + ((4 * ty + i) * RL_XP + 4 * k4) * 4);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t wrow = ws + ((4 * k4 + kk) * RL_EXP) * 4;
        const float4 wa = lds128f(wrow + (4 * tx) * 4), wb = lds128f(wrow + (32 + 4 * tx) * 4);
        const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float xi = kk == 0 ? xv[i].x : kk == 1 ? xv[i].y : kk == 2 ? xv[i].z : xv[i].w;
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(xi, wv[j], acc[i][j]);
        }
      }
    }
    __syncthreads();  // buffer `buf` is refilled by the next iteration's prefetch
    if (((c + 1) % (kRouterSeg / RL_KC)) == 0) {  // end of a segment: fold its partial in order
      const bool first = (c + 1) == (kRouterSeg / RL_KC);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          tot[i][j] = first ? acc[i][j] : __fadd_rn(tot[i][j], acc[i][j]);
          acc[i][j] = 0.0f;
        }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t tok = t0 + 4 * ty + i;
    if (tok >= n) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int ee = e0 + (j < 4 ? 4 * tx + j : 32 + 4 * tx + (j - 4));
      if (ee >= e) continue;
      if constexpr (SPLIT) {
        part[(int64_t)s_begin * n * e + tok * e + ee] = tot[i][j];
      } else {
        const float pv = sigmoid_canonical(tot[i][j]);
        probs[tok * e + ee] = pv;
        sel[tok * e + ee] = bias ? __fadd_rn(pv, bias[ee]) : pv;
      }
    }
  }
}

// Small-N finish: one thread per (token, expert) logit; all segment partials are loaded before
// the left-to-right sum.
__global__ void __launch_bounds__(256) router_finish_kernel(const float* __restrict__ part,
                                                            const float* __restrict__ bias, float* __restrict__ probs,
                                                            float* __restrict__ sel, int64_t n, int e, int nseg) {
  const int64_t off = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (off >= n * e) return;
  const int64_t ps = n * e;
  float pp[16];
  float l = __ldcs(part + off);
  for (int s0 = 1; s0 < nseg; s0 += 16) {
#pragma unroll
    for (int u = 0; u < 16; ++u) pp[u] = (s0 + u < nseg) ? __ldcs(part + (int64_t)(s0 + u) * ps + off) : 0.0f;
#pragma unroll
    for (int u = 0; u < 16; ++u)
      if (s0 + u < nseg) l = __fadd_rn(l, pp[u]);
  }
  const float pv = sigmoid_canonical(l);
  probs[off] = pv;
  sel[off] = bias ? __fadd_rn(pv, bias[off % e]) : pv;
}

// ------------------------------------------------------------------------------------------
// Routing: one CTA of 1024 threads per block of `blk` tokens (32 tokens when block routing is
// off), from the probs / selection scores of the logits kernel.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

constexpr int RT_THREADS = 1024;

__global__ void __launch_bounds__(RT_THREADS) route_kernel(RouteArgs a) {
  extern __shared__ float rsm[];
  const int tpb = a.use_block ? a.blk : 32;  // tokens per CTA
  float* ss = rsm;                           // [tpb][e] selection scores (masked in place)
  float* bmax = ss + tpb * a.e;              // [e] block max of the selection scores
  float* addv = bmax + a.e;                  // [e] 0 or -1e30
  int* gt_s = reinterpret_cast<int*>(addv + a.e);  // [e]
  int* eq_s = gt_s + a.e;                          // [e]
  __shared__ float thr_s;
  const int tid = threadIdx.x;
  const int64_t t0 = (int64_t)blockIdx.x * tpb;
  const int ntok = (int)min((int64_t)tpb, a.n - t0);
  const int cnt = ntok * a.e;
  // stage the block's selection scores (coalesced, 4 loads in flight per thread)
  const float* sg = a.sel + t0 * a.e;
  for (int base = 0; base < cnt; base += 4 * RT_THREADS) {
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int idx = base + u * RT_THREADS + tid;
      v[u] = idx < cnt ? sg[idx] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int idx = base + u * RT_THREADS + tid;
      if (idx < cnt) ss[idx] = v[u];
    }
  }
  for (int ee = tid; ee < a.e; ee += RT_THREADS) {
    gt_s[ee] = 0;
    eq_s[ee] = 0;
  }
  __syncthreads();
  if (a.use_block) {
    // block max by the fold m = s_t + relu(m - s_t), t = 1 .. blk-1 in order (:223-229)
    for (int ee = tid; ee < a.e; ee += RT_THREADS) {
      float m = ss[ee];
      for (int t = 1; t < tpb; ++t) {
        const float st = ss[t * a.e + ee];
        const float d = __fsub_rn(m, st);
        const float rl = d > 0.0f ? d : 0.0f;
        m = __fadd_rn(st, rl);
      }
      bmax[ee] = m;
    }
    __syncthreads();
    // thr = value at position cap-1 of bmax sorted descending (:231-236): rank counts split
    // over `nsp` threads per expert
    const int nsp = max(1, RT_THREADS / a.e);
    const int chunk = (a.e + nsp - 1) / nsp;
    if (tid < nsp * a.e) {
      const int ee = tid % a.e, q = tid / a.e;
      const float v = bmax[ee];
      int gt = 0, eq = 0;
      const int j1 = min(a.e, (q + 1) * chunk);
      for (int j = q * chunk; j < j1; ++j) {
        const float u = bmax[j];
        gt += u > v;
        eq += u == v;
      }
      atomicAdd(&gt_s[ee], gt);
      atomicAdd(&eq_s[ee], eq);
    }
    __syncthreads();
    for (int ee = tid; ee < a.e; ee += RT_THREADS) {
      const int gt = gt_s[ee], eq = eq_s[ee];
      if (gt <= a.cap - 1 && a.cap - 1 < gt + eq) thr_s = bmax[ee];  // all writers store the same value
    }
    __syncthreads();
    // keep = step(bmax - (thr - 1e-6)); masked scores += -1e30 (:238-248)
    const float thr_m = __fadd_rn(__fmul_rn(thr_s, 1.0f), -1e-6f);
    for (int ee = tid; ee < a.e; ee += RT_THREADS) {
      const float dlt = __fsub_rn(bmax[ee], thr_m);
      const bool keep = dlt > 0.0f;
      if (a.allowed) a.allowed[(int64_t)blockIdx.x * a.e + ee] = keep ? 1 : 0;
      addv[ee] = keep ? 0.0f : -1e30f;
    }
    __syncthreads();
    for (int idx = tid; idx < cnt; idx += RT_THREADS) ss[idx] = __fadd_rn(ss[idx], addv[idx % a.e]);
    __syncthreads();
  }
  // per-token top-k (:252): one warp per token, ties to the lower expert id
  const int warp = tid >> 5, lane = tid & 31;
  for (int t = warp; t < ntok; t += RT_THREADS / 32) {
    const float* st = ss + t * a.e;
    uint32_t taken = 0;  // bit j: candidate lane + 32 j already selected (e <= 1024)
    int sel_idx[16];
    for (int s = 0; s < a.top_k; ++s) {
      float bv = 0.0f;
      int bi = -1;
      for (int j = 0; j * 32 + lane < a.e; ++j) {
        if (taken & (1u << j)) continue;
        const int ee = j * 32 + lane;
        const float v = st[ee];
        if (bi < 0 || better(v, ee, bv, bi)) {
          bv = v;
          bi = ee;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || better(ov, oi, bv, bi))) {
          bv = ov;
          bi = oi;
        }
      }
      if (bi >= 0 && (bi & 31) == lane) taken |= 1u << (bi >> 5);
      sel_idx[s] = bi;
    }
    // gates from the unbiased probs, renormalised (sum in double) and scaled (:253-262)
    if (lane == 0) {
      const int64_t tok = t0 + t;
      float wv[16];
      double sum = 0.0;
      for (int s = 0; s < a.top_k; ++s) {
        wv[s] = a.probs[tok * a.e + sel_idx[s]];
        sum = __dadd_rn(sum, (double)wv[s]);
      }
      const float fs = __double2float_rn(sum);
      for (int s = 0; s < a.top_k; ++s) {
        float v = wv[s];
        if (a.norm_topk) v = __fdiv_rn(v, fs);
        if (a.scale != 1.0f) v = __fmul_rn(v, a.scale);
        a.idx[tok * a.top_k + s] = sel_idx[s];
        a.w[tok * a.top_k + s] = v;
        atomicAdd(&a.counts[sel_idx[s]], 1);
      }
    }
  }
}

// Fills probs and sel [n][e]. split = true: one CTA per (tile, segment) with partials in `part`
// [h / 256][n][e], then the elementwise finish.
cudaError_t launch_router(const float* x, const float* wrt, const float* bias, float* part, float* probs, float* sel,
                          int64_t n, int h, int e, bool split, cudaStream_t st) {
  if (h % kRouterSeg) return cudaErrorInvalidValue;
  const int nseg = h / kRouterSeg;
  dim3 grid((unsigned)((n + RL_TOK - 1) / RL_TOK), (unsigned)((e + RL_EXP - 1) / RL_EXP), split ? (unsigned)nseg : 1u);
  if (split) {
    cudaFuncSetAttribute(router_logits_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, RL_SMEM);
    router_logits_kernel<true><<<grid, RL_THREADS, RL_SMEM, st>>>(x, wrt, bias, part, probs, sel, n, h, e);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    const int64_t cnt = n * e;
    router_finish_kernel<<<(unsigned)((cnt + 255) / 256), 256, 0, st>>>(part, bias, probs, sel, n, e, nseg);
  } else {
    cudaFuncSetAttribute(router_logits_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, RL_SMEM);
    router_logits_kernel<false><<<grid, RL_THREADS, RL_SMEM, st>>>(x, wrt, bias, part, probs, sel, n, h, e);
  }
  return cudaGetLastError();
}

cudaError_t launch_route(const RouteArgs& a, cudaStream_t st) {
  const int tpb = a.use_block ? a.blk : 32;
  const int64_t nblocks = (a.n + tpb - 1) / tpb;
  const size_t smem = sizeof(float) * ((size_t)tpb * a.e + 4 * (size_t)a.e);
  cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  route_kernel<<<(unsigned)nblocks, RT_THREADS, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace dmoe
