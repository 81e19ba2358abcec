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
// Router logits: a 32-token x 64-expert tile per CTA over router segments [s_begin, s_end).
// `wrt` is the router weight transposed to [h][e] (done once at bind time) so weight tiles are
// contiguous rows. Two shapes of the same arithmetic:
//   <4, 4, 128>: 128 threads x (4 tokens x 4 experts); one segment per CTA (grid.z = #segments),
//                writing the segment partials P_s that route_kernel sums in order (small N);
//   <8, 8, 32>:  32 threads x (8 tokens x 8 experts); all segments in one CTA with the running
//                sum tot = P_0 + P_1 + ... (large N, 1024+ CTAs).
// Both produce the canonical bits.
// ------------------------------------------------------------------------------------------
constexpr int RL_TOK = 32, RL_EXP = 64, RL_KC = 64;

template <int TM, int TN, int NTH>
__global__ void __launch_bounds__(NTH) router_logits_kernel(const float* __restrict__ x, const float* __restrict__ wrt,
                                                            float* __restrict__ part, int64_t n, int h, int e,
                                                            int segs_per_cta) {
  static_assert((RL_TOK / TM) * (RL_EXP / TN) == NTH, "thread tiles cover the CTA tile");
  __shared__ __align__(16) float xs[RL_KC][RL_TOK + 4];
  __shared__ __align__(16) float ws[RL_KC][RL_EXP];
  const int tid = threadIdx.x;
  constexpr int NX = RL_EXP / TN;
  const int ty = tid / NX;  // tokens TM ty ..
  const int tx = tid % NX;  // experts TN tx ..
  const int64_t t0 = (int64_t)blockIdx.x * RL_TOK;
  const int e0 = blockIdx.y * RL_EXP;
  const int nseg = (h + kRouterSeg - 1) / kRouterSeg;
  const int s_begin = blockIdx.z * segs_per_cta;
  const int s_end = min(nseg, s_begin + segs_per_cta);
  float tot[TM][TN], acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) tot[i][j] = 0.0f;
  for (int s = s_begin; s < s_end; ++s) {
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;
    const int k_end = min(h, (s + 1) * kRouterSeg);
    for (int kc = s * kRouterSeg; kc < k_end; kc += RL_KC) {
      const int klen = min(RL_KC, k_end - kc);
      __syncthreads();
      // x tile: 32 tokens x 64 k (float4 along k) -> xs[k][t]
      for (int q = tid; q < RL_TOK * (RL_KC / 4); q += NTH) {
        const int t = q / (RL_KC / 4), k4 = q % (RL_KC / 4);
        const int64_t tok = t0 + t;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tok < n && 4 * k4 < klen) v = *reinterpret_cast<const float4*>(x + tok * h + kc + 4 * k4);
        xs[4 * k4 + 0][t] = v.x;
        xs[4 * k4 + 1][t] = v.y;
        xs[4 * k4 + 2][t] = v.z;
        xs[4 * k4 + 3][t] = v.w;
      }
      // weight tile: 64 k rows x 64 experts, contiguous in wrt
      for (int q = tid; q < RL_KC * (RL_EXP / 4); q += NTH) {
        const int k = q / (RL_EXP / 4), e4 = q % (RL_EXP / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k < klen && e0 + 4 * e4 < e) v = *reinterpret_cast<const float4*>(wrt + (int64_t)(kc + k) * e + e0 + 4 * e4);
        *reinterpret_cast<float4*>(&ws[k][4 * e4]) = v;
      }
      __syncthreads();
      for (int k = 0; k < klen; ++k) {
        float xa[TM], wa[TN];
#pragma unroll
        for (int i = 0; i < TM; i += 4) {
          const float4 v = *reinterpret_cast<const float4*>(&xs[k][TM * ty + i]);
          xa[i] = v.x; xa[i + 1] = v.y; xa[i + 2] = v.z; xa[i + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < TN; j += 4) {
          const float4 v = *reinterpret_cast<const float4*>(&ws[k][TN * tx + j]);
          wa[j] = v.x; wa[j + 1] = v.y; wa[j + 2] = v.z; wa[j + 3] = v.w;
        }
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) acc[i][j] = __fmaf_rn(xa[i], wa[j], acc[i][j]);
      }
    }
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) tot[i][j] = (s == s_begin) ? acc[i][j] : __fadd_rn(tot[i][j], acc[i][j]);
  }
  float* dst = part + (int64_t)blockIdx.z * n * e;
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t tok = t0 + TM * ty + i;
    if (tok >= n) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int ee = e0 + TN * tx + j;
      if (ee < e) dst[tok * e + ee] = tot[i][j];
    }
  }
}

// ------------------------------------------------------------------------------------------
// Routing: one CTA per block of `rblk` tokens (32 tokens when block routing is off).
// ------------------------------------------------------------------------------------------

__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

__global__ void __launch_bounds__(256) route_kernel(RouteArgs a) {
  extern __shared__ float rsm[];
  const int tpb = a.use_block ? a.blk : 32;  // tokens per CTA
  float* ps = rsm;                           // [tpb][e] probs
  float* ss = rsm + tpb * a.e;               // [tpb][e] selection scores
  float* bmax = ss + tpb * a.e;              // [e]
  __shared__ float thr_s;
  const int tid = threadIdx.x;
  const int64_t t0 = (int64_t)blockIdx.x * tpb;
  const int ntok = (int)min((int64_t)tpb, a.n - t0);
  // logits -> probs, selection scores
  for (int idx = tid; idx < ntok * a.e; idx += blockDim.x) {
    const int t = idx / a.e, ee = idx % a.e;
    const int64_t off = (t0 + t) * a.e + ee;
    // partials P_0 .. P_{nparts-1}: loads issued together, summed left to right
    const int64_t pstride = a.n * a.e;
    float l = a.part[off];
    for (int q0 = 1; q0 < a.nparts; q0 += 8) {
      float pv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) pv[u] = (q0 + u < a.nparts) ? a.part[(int64_t)(q0 + u) * pstride + off] : 0.0f;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (q0 + u < a.nparts) l = __fadd_rn(l, pv[u]);
    }
    const float pv = sigmoid_canonical(l);
    ps[t * a.e + ee] = pv;
    ss[t * a.e + ee] = a.bias ? __fadd_rn(pv, a.bias[ee]) : pv;
    if (a.probs) a.probs[off] = pv;
  }
  __syncthreads();
  if (a.use_block) {
    for (int ee = tid; ee < a.e; ee += blockDim.x) {
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
    for (int ee = tid; ee < a.e; ee += blockDim.x) {
      const float v = bmax[ee];
      int gt = 0, eq = 0;
      for (int j = 0; j < a.e; ++j) {
        const float u = bmax[j];
        gt += u > v;
        eq += u == v;
      }
      if (gt <= a.cap - 1 && a.cap - 1 < gt + eq) thr_s = v;  // all writers store the same value
    }
    __syncthreads();
    const float thr_m = __fadd_rn(__fmul_rn(thr_s, 1.0f), -1e-6f);
    for (int ee = tid; ee < a.e; ee += blockDim.x) {
      const float dlt = __fsub_rn(bmax[ee], thr_m);
      const bool keep = dlt > 0.0f;
      if (a.allowed) a.allowed[(int64_t)blockIdx.x * a.e + ee] = keep ? 1 : 0;
      const float add = keep ? 0.0f : -1e30f;
      for (int t = 0; t < tpb; ++t) ss[t * a.e + ee] = __fadd_rn(ss[t * a.e + ee], add);
    }
    __syncthreads();
  }
  // per-token top-k: one warp per token
  const int warp = tid >> 5, lane = tid & 31;
  const int nwarps = blockDim.x >> 5;
  for (int t = warp; t < ntok; t += nwarps) {
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
    if (lane == 0) {
      const int64_t tok = t0 + t;
      float wv[16];
      double sum = 0.0;
      for (int s = 0; s < a.top_k; ++s) {
        wv[s] = ps[t * a.e + sel_idx[s]];
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

// nparts must be 1 (running sum) or the number of segments (one partial per segment).
cudaError_t launch_router(const float* x, const float* wrt, float* part, int64_t n, int h, int e, int nparts,
                          cudaStream_t st) {
  const int nseg = (h + kRouterSeg - 1) / kRouterSeg;
  if (nparts != 1 && nparts != nseg) return cudaErrorInvalidValue;
  dim3 grid((unsigned)((n + RL_TOK - 1) / RL_TOK), (unsigned)((e + RL_EXP - 1) / RL_EXP), (unsigned)nparts);
  if (nparts == 1)
    router_logits_kernel<8, 8, 32><<<grid, 32, 0, st>>>(x, wrt, part, n, h, e, nseg);
  else
    router_logits_kernel<4, 4, 128><<<grid, 128, 0, st>>>(x, wrt, part, n, h, e, 1);
  return cudaGetLastError();
}

cudaError_t launch_route(const RouteArgs& a, cudaStream_t st) {
  const int tpb = a.use_block ? a.blk : 32;
  const int64_t nblocks = (a.n + tpb - 1) / tpb;
  const size_t smem = sizeof(float) * ((size_t)2 * tpb * a.e + a.e);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr = true;
  }
  route_kernel<<<(unsigned)nblocks, 256, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace dmoe
