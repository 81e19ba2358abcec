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
//
// Two launches: the router GEMM (router_logits_wide_kernel: whole logits on 128-expert tiles at
// large N; router_logits_split_kernel: per-segment partials P_s summed by the tile's last CTA),
// then p = sigmoid(logit); and route_kernel (bias, then the routing of one block per CTA).
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
// Router logits split by segment (small and mid N, where whole-K tiles cannot fill the GPU).
// CTA = 256 threads on a (16 TM) token x 64 expert tile and one 256-k segment s (blockIdx.z);
// thread (ty, tx) = (tid / 16, tid % 16) owns tokens TM ty .. TM ty + TM - 1 and experts
// 4 tx .. 4 tx + 3: TM x 4 independent fma chains. x [token][k] and the transposed router weight
// wrt [k][expert] (transposed once at bind time) arrive in 32-k chunks by cp.async. Each CTA
// writes its partial P_s to part[s]; the last CTA of a tile to finish (per-tile arrival counter)
// adds P_0 .. P_{S-1} left to right, writes p = sigmoid(logit) to part[0] and re-arms the counter.
// TM = 8 from ~1000 tokens (fewer shared-memory reads per fma), TM = 2 below (more CTAs).
// ------------------------------------------------------------------------------------------
constexpr int RL_EXP = 64, RL_KC = 32, RL_EPT = 4, RL_TX = RL_EXP / RL_EPT, RL_THREADS = 16 * RL_TX;
static_assert(RL_EPT == 4, "a thread's experts are one 16-byte weight load and one float4 store per token");
constexpr int RL_XP = RL_KC + 4;  // x tile row pitch (floats)

template <int TM>
constexpr int rl_tok() { return 16 * TM; }
template <int TM>
constexpr int rl_stage_floats() { return rl_tok<TM>() * RL_XP + RL_KC * RL_EXP; }
// ring depth: TM = 2 tiles prefetch their whole 256-k segment at once (one memory latency
// instead of eight); TM = 8 tiles (four times the shared memory per chunk) keep a 3-deep ring
template <int TM>
constexpr int rl_stages() { return TM <= 2 ? kRouterSeg / RL_KC : 3; }
template <int TM>
constexpr int rl_smem() { return rl_stages<TM>() * rl_stage_floats<TM>() * 4; }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Packed fp32 pairs (low word = first value) for sm_100's fma.rn.f32x2: each lane is an IEEE
// round-to-nearest fma, bitwise the same as fmaf, at half the issue slots. Accumulators and
// weight pairs stay packed in 64-bit registers; each x value is duplicated once per k.
typedef unsigned long long f32x2;
__device__ __forceinline__ void ffma2(f32x2& d, f32x2 a, f32x2 b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}
__device__ __forceinline__ f32x2 dup2(float x) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float2 unpack2(f32x2 v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ void lds2x64(uint32_t a, f32x2& lo, f32x2& hi) {
  asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(lo), "=l"(hi) : "r"(a));
}

template <int TM>
__global__ void __launch_bounds__(RL_THREADS, 2) router_logits_split_kernel(const float* __restrict__ x,
                                                                          const float* __restrict__ wrt,
                                                                          float* __restrict__ part, int64_t n, int h,
                                                                          int e, int32_t* __restrict__ arrivals,
                                                                          int32_t* __restrict__ zero_counts) {
  extern __shared__ __align__(16) float rl_smem_f[];
  pdl_wait();
  pdl_trigger();
  if (zero_counts && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)  // route_kernel's counters
    for (int i = threadIdx.x; i < e; i += RL_THREADS) zero_counts[i] = 0;
  constexpr int TT = rl_tok<TM>();
  constexpr int RL_STAGES = rl_stages<TM>();
  constexpr int NCHUNKS = kRouterSeg / RL_KC;
  const uint32_t sm0 = smem_u32(rl_smem_f);
  const int tid = threadIdx.x;
  const int ty = tid / RL_TX, tx = tid % RL_TX;
  const int64_t t0 = (int64_t)blockIdx.x * TT;
  const int e0 = blockIdx.y * RL_EXP;
  const int nseg = h / kRouterSeg;
  const int seg = (int)blockIdx.z;
  const int kc0 = seg * kRouterSeg;

  auto xs_of = [&](int buf) { return sm0 + buf * rl_stage_floats<TM>() * 4; };
  auto ws_of = [&](int buf) { return xs_of(buf) + TT * RL_XP * 4; };
  auto load_chunk = [&](int c, int buf) {
    const int kc = kc0 + c * RL_KC;
    const uint32_t xs = xs_of(buf), ws = ws_of(buf);
    for (int q = tid; q < TT * (RL_KC / 4); q += RL_THREADS) {
      const int t = q / (RL_KC / 4), k4 = q % (RL_KC / 4);
      const bool ok = t0 + t < n;
      const float* src = ok ? x + (t0 + t) * h + kc + 4 * k4 : x;
      cp_async16(xs + (t * RL_XP + 4 * k4) * 4, src, ok);
    }
#pragma unroll
    for (int r = 0; r < (RL_KC * RL_EXP / 4) / RL_THREADS; ++r) {
      const int q = tid + r * RL_THREADS, k = q >> 4, e4 = q & 15;
      const bool ok = e0 + 4 * e4 < e;
      const float* src = ok ? wrt + (int64_t)(kc + k) * e + e0 + 4 * e4 : wrt;
      cp_async16(ws + (k * RL_EXP + 4 * e4) * 4, src, ok);
    }
  };

  constexpr int NJP = RL_EPT / 2;
  f32x2 acc[TM][NJP];  // experts (2 jp, 2 jp + 1) of the thread's RL_EPT, packed: P_s
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int jp = 0; jp < NJP; ++jp) acc[i][jp] = 0ull;  // (+0.0f, +0.0f)

#pragma unroll
  for (int c = 0; c < RL_STAGES - 1; ++c) {
    if (c < NCHUNKS) load_chunk(c, c);
    cp_async_commit();
  }
  for (int c = 0; c < NCHUNKS; ++c) {
    const int buf = c % RL_STAGES;
    cp_async_wait<RL_STAGES - 2>();
    __syncthreads();  // chunk c landed for every thread; chunk c - 1's buffer is free
    if (c + RL_STAGES - 1 < NCHUNKS) load_chunk(c + RL_STAGES - 1, (c + RL_STAGES - 1) % RL_STAGES);
    cp_async_commit();
    const uint32_t xs = xs_of(buf), ws = ws_of(buf);
#pragma unroll 2
    for (int k4 = 0; k4 < RL_KC / 4; ++k4) {
      float4 xv[TM];
#pragma unroll
      for (int i = 0; i < TM; ++i) xv[i] = lds128f(xs + ((TM * ty + i) * RL_XP + 4 * k4) * 4);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t wrow = ws + ((4 * k4 + kk) * RL_EXP) * 4;
        f32x2 wp[NJP];
        lds2x64(wrow + (RL_EPT * tx) * 4, wp[0], wp[1]);
#pragma unroll
        for (int i = 0; i < TM; ++i) {
          const f32x2 xx = dup2(kk == 0 ? xv[i].x : kk == 1 ? xv[i].y : kk == 2 ? xv[i].z : xv[i].w);
#pragma unroll
          for (int jp = 0; jp < NJP; ++jp) ffma2(acc[i][jp], xx, wp[jp]);
        }
      }
    }
  }
  cp_async_wait<0>();
  float* dst = part + (int64_t)seg * n * e;
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t tok = t0 + TM * ty + i;
    const int ee = e0 + RL_EPT * tx;
    if (tok >= n || ee >= e) continue;  // e is a multiple of 4: the thread's 4 experts are whole or absent
    const float2 a = unpack2(acc[i][0]), b = unpack2(acc[i][1]);
    *reinterpret_cast<float4*>(dst + tok * e + ee) = make_float4(a.x, a.y, b.x, b.y);
  }
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  const int tile = blockIdx.y * gridDim.x + blockIdx.x;
  if (tid == 0) s_last = atomicAdd(&arrivals[tile], 1) == nseg - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // this tile's logits = P_0 + P_1 + ... in segment order; p = sigmoid(logit) into part[0]
  const int64_t ps = n * e;
  for (int q = tid; q < TT * (RL_EXP / 4); q += RL_THREADS) {
    const int t = q / (RL_EXP / 4), e4 = q % (RL_EXP / 4);
    const int64_t tok = t0 + t;
    const int ee = e0 + 4 * e4;
    if (tok >= n || ee >= e) continue;
    const float4* src = reinterpret_cast<const float4*>(part + tok * e + ee);
    float4 l = __ldcg(src);
    for (int s0 = 1; s0 < nseg; s0 += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (s0 + u < nseg) v[u] = __ldcg(src + (int64_t)(s0 + u) * (ps / 4));
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (s0 + u < nseg) {
          l.x = __fadd_rn(l.x, v[u].x);
          l.y = __fadd_rn(l.y, v[u].y);
          l.z = __fadd_rn(l.z, v[u].z);
          l.w = __fadd_rn(l.w, v[u].w);
        }
    }
    *reinterpret_cast<float4*>(part + tok * e + ee) =
        make_float4(sigmoid_canonical(l.x), sigmoid_canonical(l.y), sigmoid_canonical(l.z), sigmoid_canonical(l.w));
  }
  if (tid == 0) arrivals[tile] = 0;  // re-armed for the next launch on this stream
}

// ------------------------------------------------------------------------------------------
// Router logits on wide whole-K tiles (large N): CTA = 256 threads, one CTA per SM, on a (16 TM)
// token x 128 expert tile. Warp w takes expert half w & 1 and token-row group w >> 1; lane =
// (tyl, tx) = (lane / 8, lane % 8), token row ty = 4 (w >> 1) + tyl. A thread owns tokens ty + 16 i
// (i < TM) and experts 4 tx .. 4 tx + 3 and 32 + 4 tx .. 32 + 4 tx + 3 of its half: TM x 8
// independent fma chains, the segment sums in registers. Against the 64-expert tiles (measured
// at 8192 tokens: 8.3 shared-memory wavefronts per warp and k, fma pipe 64 % active) each
// half-warp (the unit a 16-byte shared load is served in) reads two adjacent token rows and 128
// contiguous weight bytes per load, one wavefront each instead of one and two, for twice the fmas
// per load; the 68-float x pitch puts adjacent rows 4 banks apart. x [token][k] and wrt
// [k][expert] arrive in 64-k chunks through a 3-deep cp.async ring (198 KB at TM = 8). Same
// canonical order as router_logits_split_kernel: per 256-k segment an fma chain from 0, the segment
// sums added left to right, then p = sigmoid(logit) into probs [n][e].
// ------------------------------------------------------------------------------------------
constexpr int RW_EXP = 128, RW_KC = 64, RW_XP = RW_KC + 4, RW_THREADS = 256, RW_STAGES = 3;
template <int TM>
constexpr int rw_tok() { return 16 * TM; }
template <int TM>
constexpr int rw_stage_floats() { return rw_tok<TM>() * RW_XP + RW_KC * RW_EXP; }
template <int TM>
constexpr int rw_smem() { return RW_STAGES * rw_stage_floats<TM>() * 4; }
static_assert(kRouterSeg % RW_KC == 0, "a chunk lies in one segment");

template <int TM>
__global__ void __launch_bounds__(RW_THREADS, 1) router_logits_wide_kernel(const float* __restrict__ x,
                                                                         const float* __restrict__ wrt,
                                                                         float* __restrict__ probs, int64_t n, int h,
                                                                         int e, int32_t* __restrict__ zero_counts) {
  extern __shared__ __align__(16) float rw_smem_f[];
  pdl_wait();
  pdl_trigger();
  if (zero_counts && blockIdx.x == 0 && blockIdx.y == 0)  // route_kernel's counters
    for (int i = threadIdx.x; i < e; i += RW_THREADS) zero_counts[i] = 0;
  constexpr int TT = rw_tok<TM>();
  constexpr int CH_PER_SEG = kRouterSeg / RW_KC;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tx = lane & 7, ty = 4 * (warp >> 1) + (lane >> 3), eh = warp & 1;
  const int64_t t0 = (int64_t)blockIdx.x * TT;
  const int e0 = blockIdx.y * RW_EXP;
  const int nchunks = h / RW_KC;
  const uint32_t sm0 = smem_u32(rw_smem_f);
  auto xs_of = [&](int buf) { return sm0 + buf * rw_stage_floats<TM>() * 4; };
  auto ws_of = [&](int buf) { return xs_of(buf) + TT * RW_XP * 4; };
  auto load_chunk = [&](int c, int buf) {
    const int kc = c * RW_KC;
    const uint32_t xs = xs_of(buf), ws = ws_of(buf);
#pragma unroll
    for (int r = 0; r < TT * (RW_KC / 4) / RW_THREADS; ++r) {
      const int q = tid + r * RW_THREADS, t = q / (RW_KC / 4), k4 = q % (RW_KC / 4);
      const bool ok = t0 + t < n;
      cp_async16(xs + (t * RW_XP + 4 * k4) * 4, ok ? x + (t0 + t) * h + kc + 4 * k4 : x, ok);
    }
#pragma unroll
    for (int r = 0; r < (RW_KC * RW_EXP / 4) / RW_THREADS; ++r) {
      const int q = tid + r * RW_THREADS, k = q / (RW_EXP / 4), e4 = q % (RW_EXP / 4);
      const bool ok = e0 + 4 * e4 < e;
      cp_async16(ws + (k * RW_EXP + 4 * e4) * 4, ok ? wrt + (int64_t)(kc + k) * e + e0 + 4 * e4 : wrt, ok);
    }
  };
  static_assert(TT * (RW_KC / 4) % RW_THREADS == 0, "whole x loads per thread");

  // acc[i][j]: experts (4 tx + 2 j, + 1) for j = 0, 1 and (32 + 4 tx + 2 (j - 2), + 1) for j = 2, 3
  // of the half, packed; tot[i][2 j], tot[i][2 j + 1] their segment sums
  f32x2 acc[TM][4];
  float tot[TM][8];
#pragma unroll
  for (int i = 0; i < TM; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0ull;  // (+0.0f, +0.0f)
#pragma unroll
    for (int j = 0; j < 8; ++j) tot[i][j] = 0.0f;
  }
#pragma unroll
  for (int c = 0; c < RW_STAGES - 1; ++c) {
    if (c < nchunks) load_chunk(c, c);
    cp_async_commit();
  }
  for (int c = 0; c < nchunks; ++c) {
    const int buf = c % RW_STAGES;
    cp_async_wait<RW_STAGES - 2>();
    __syncthreads();  // chunk c landed for every thread; chunk c - 1's buffer is free
    if (c + RW_STAGES - 1 < nchunks) load_chunk(c + RW_STAGES - 1, (c + RW_STAGES - 1) % RW_STAGES);
    cp_async_commit();
    const uint32_t xrow = xs_of(buf) + ty * RW_XP * 4;              // token row ty + 16 i at + 16 i RW_XP floats
    const uint32_t wcol = ws_of(buf) + (eh * (RW_EXP / 2) + 4 * tx) * 4;  // k row at + k RW_EXP floats
#pragma unroll 2
    for (int k4 = 0; k4 < RW_KC / 4; ++k4) {
      float4 xv[TM];
#pragma unroll
      for (int i = 0; i < TM; ++i) xv[i] = lds128f(xrow + (16 * i * RW_XP + 4 * k4) * 4);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t wk = wcol + (4 * k4 + kk) * RW_EXP * 4;
        f32x2 wp[4];
        lds2x64(wk, wp[0], wp[1]);
        lds2x64(wk + 32 * 4, wp[2], wp[3]);
#pragma unroll
        for (int i = 0; i < TM; ++i) {
          const f32x2 xx = dup2(kk == 0 ? xv[i].x : kk == 1 ? xv[i].y : kk == 2 ? xv[i].z : xv[i].w);
#pragma unroll
          for (int j = 0; j < 4; ++j) ffma2(acc[i][j], xx, wp[j]);
        }
      }
    }
    if (((c + 1) % CH_PER_SEG) == 0) {  // end of a segment: fold its partial in order
      const bool first = (c + 1) == CH_PER_SEG;
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 a = unpack2(acc[i][j]);
          tot[i][2 * j] = first ? a.x : __fadd_rn(tot[i][2 * j], a.x);
          tot[i][2 * j + 1] = first ? a.y : __fadd_rn(tot[i][2 * j + 1], a.y);
          acc[i][j] = 0ull;
        }
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t tok = t0 + ty + 16 * i;
    if (tok >= n) continue;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const int ee = e0 + eh * (RW_EXP / 2) + 32 * g + 4 * tx;
      if (ee >= e) continue;  // e is a multiple of 4: the group is whole or absent
      *reinterpret_cast<float4*>(probs + tok * e + ee) =
          make_float4(sigmoid_canonical(tot[i][4 * g]), sigmoid_canonical(tot[i][4 * g + 1]),
                      sigmoid_canonical(tot[i][4 * g + 2]), sigmoid_canonical(tot[i][4 * g + 3]));
    }
  }
}

// ------------------------------------------------------------------------------------------
// Routing: `tok_split` CTAs of 1024 threads per block of `blk` tokens (32 tokens when block
// routing is off), from p = sigmoid(logit). Every CTA of a block stages the block's p and derives
// the block's capacity set (fold, threshold, mask: the same bits in each); CTA j then takes the
// top-k of tokens [j tpb / tok_split, (j + 1) tpb / tok_split). Splitting spreads the per-token
// work over more SMs when there are few blocks.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

// monotonic map of a float onto unsigned order (-0 below +0; every non-NaN float above 0)
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

constexpr int RT_THREADS = 1024;

__global__ void __launch_bounds__(RT_THREADS) route_kernel(RouteArgs a) {
  extern __shared__ float rsm[];
  pdl_wait();
  pdl_trigger();
  const int tpb = a.use_block ? a.blk : 32;  // tokens per CTA
  const int E = a.e;
  float* ss = rsm;                                 // [tpb][E] selection scores (masked in place)
  float* pp = ss + tpb * E;                        // [tpb][E] probabilities
  float* bmax = pp + tpb * E;                      // [E] block max of the selection scores
  float* addv = bmax + E;                          // [E] 0 or -1e30
  int* gt_s = reinterpret_cast<int*>(addv + E);    // [E]
  int* eq_s = gt_s + E;                            // [E]
  int* cnt_s = eq_s + E;                           // [E] pairs per expert in this CTA
  __shared__ float thr_s;
  const int tid = threadIdx.x;
  const int64_t blk_id = blockIdx.x / a.tok_split;
  const int part = blockIdx.x % a.tok_split;
  const int64_t t0 = blk_id * tpb;
  const int ntok = (int)min((int64_t)tpb, a.n - t0);
  const int cnt = ntok * E;
  // p and sel = p + bias (:204-210); 16-byte loads, all issued before use
  {
    const float4* pg = reinterpret_cast<const float4*>(a.probs + t0 * E);
    constexpr int PF = 4;
    for (int base = 0; base < cnt / 4; base += PF * RT_THREADS) {
      float4 v[PF], b[PF];
#pragma unroll
      for (int u = 0; u < PF; ++u) {
        const int i4 = base + u * RT_THREADS + tid;
        if (i4 < cnt / 4) {
          v[u] = __ldcg(pg + i4);
          b[u] = a.bias ? __ldg(reinterpret_cast<const float4*>(a.bias) + (4 * i4 % E) / 4) : make_float4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < PF; ++u) {
        const int i4 = base + u * RT_THREADS + tid;
        if (i4 >= cnt / 4) continue;
        reinterpret_cast<float4*>(pp)[i4] = v[u];
        if (a.bias)
          v[u] = make_float4(__fadd_rn(v[u].x, b[u].x), __fadd_rn(v[u].y, b[u].y), __fadd_rn(v[u].z, b[u].z),
                             __fadd_rn(v[u].w, b[u].w));
        reinterpret_cast<float4*>(ss)[i4] = v[u];
      }
    }
  }
  for (int ee = tid; ee < E; ee += RT_THREADS) {
    gt_s[ee] = 0;
    eq_s[ee] = 0;
    cnt_s[ee] = 0;
  }
  __syncthreads();
  if (a.use_block) {
    // block max by the fold m = s_t + relu(m - s_t), t = 1 .. blk-1 in order (:223-229); the
    // scores are loaded 8 tokens ahead of the dependent chain
    auto fold = [](float m, float st) {
      const float d = __fsub_rn(m, st);
      return __fadd_rn(st, d > 0.0f ? d : 0.0f);
    };
    for (int ee = tid; ee < E; ee += RT_THREADS) {
      float m = ss[ee];
      int t = 1;
      for (; t + 8 <= tpb; t += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = ss[(t + u) * E + ee];
#pragma unroll
        for (int u = 0; u < 8; ++u) m = fold(m, v[u]);
      }
      for (; t < tpb; ++t) m = fold(m, ss[t * E + ee]);
      bmax[ee] = m;
    }
    __syncthreads();
    // thr = value at position cap-1 of bmax sorted descending (:231-236): rank counts split
    // over `nsp` threads per expert
    // (chunks of whole float4s: E is a multiple of 4, so a float4 below E lies inside)
    const int nsp = max(1, RT_THREADS / E);
    const int chunk = ((E + nsp - 1) / nsp + 3) & ~3;
    if (tid < nsp * E) {
      const int ee = tid % E, q = tid / E;
      const float v = bmax[ee];
      int gt = 0, eq = 0;
      const int j1 = min(E, (q + 1) * chunk);
      const float4* b4 = reinterpret_cast<const float4*>(bmax);
#pragma unroll 4
      for (int j = q * chunk; j < j1; j += 4) {
        const float4 u = b4[j >> 2];
        gt += (u.x > v) + (u.y > v) + (u.z > v) + (u.w > v);
        eq += (u.x == v) + (u.y == v) + (u.z == v) + (u.w == v);
      }
      atomicAdd(&gt_s[ee], gt);
      atomicAdd(&eq_s[ee], eq);
    }
    __syncthreads();
    for (int ee = tid; ee < E; ee += RT_THREADS) {
      const int gt = gt_s[ee], eq = eq_s[ee];
      if (gt <= a.cap - 1 && a.cap - 1 < gt + eq) thr_s = bmax[ee];  // all writers store the same value
    }
    __syncthreads();
    // keep = step(bmax - (thr - 1e-6)); masked scores += -1e30 (:238-248)
    const float thr_m = __fadd_rn(__fmul_rn(thr_s, 1.0f), -1e-6f);
    for (int ee = tid; ee < E; ee += RT_THREADS) {
      const float dlt = __fsub_rn(bmax[ee], thr_m);
      const bool keep = dlt > 0.0f;
      if (a.allowed && part == 0) a.allowed[blk_id * E + ee] = keep ? 1 : 0;
      addv[ee] = keep ? 0.0f : -1e30f;
    }
    __syncthreads();
    if (RT_THREADS % E == 0) {  // a thread's scores are all of one expert
      const float av = addv[tid % E];
      for (int i = tid; i < cnt; i += RT_THREADS) ss[i] = __fadd_rn(ss[i], av);
    } else {
      for (int i = tid; i < cnt; i += RT_THREADS) ss[i] = __fadd_rn(ss[i], addv[i % E]);
    }
    __syncthreads();
  }
  // per-token top-k (:252): one warp per token, ties to the lower expert id. Each lane keeps
  // the best of its candidates (experts lane, lane + 32, ...); every round the warp reduces the
  // lanes' bests, and only the winning lane marks its candidate taken and rescans. With E <= 256
  // a lane's (at most 8) candidates sit in registers, so a rescan reads no shared memory.
  constexpr int RC = 8;
  const int warp = tid >> 5, lane = tid & 31;
  const int ncand = (E - lane + 31) / 32;  // this lane's candidates (<= 32)
  const bool regs = E <= 32 * RC;
  const int per = (tpb + a.tok_split - 1) / a.tok_split;
  const int tb = part * per, te = min(ntok, tb + per);
  for (int t = tb + warp; t < te; t += RT_THREADS / 32) {
    const float* st = ss + t * E;
    uint32_t taken = 0;
    float hv = 0.0f;
    int hi = -1;
    float cv[RC];
#pragma unroll
    for (int j = 0; j < RC; ++j) cv[j] = (regs && j < ncand) ? st[j * 32 + lane] : 0.0f;
    auto rescan = [&]() {
      hv = 0.0f;
      hi = -1;
      if (regs) {
#pragma unroll
        for (int j = 0; j < RC; ++j) {
          const int ee = j * 32 + lane;
          if (j < ncand && !(taken & (1u << j)) && (hi < 0 || better(cv[j], ee, hv, hi))) {
            hv = cv[j];
            hi = ee;
          }
        }
        return;
      }
      for (int j = 0; j < ncand; ++j) {
        if (taken & (1u << j)) continue;
        const int ee = j * 32 + lane;
        const float v = st[ee];
        if (hi < 0 || better(v, ee, hv, hi)) {
          hv = v;
          hi = ee;
        }
      }
    };
    rescan();
    int sel_idx = -1;  // lane s < top_k keeps slot s
    for (int s = 0; s < a.top_k; ++s) {
      // the warp's best (value, then lowest id): the largest order key (keys order floats as the
      // comparisons do; NaN scores, whose routing the reference leaves unspecified too, aside),
      // then the lowest id among the lanes holding it; 0 = no candidate left
      const uint32_t key = hi >= 0 ? order_key(hv) : 0u;
      const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
      const uint32_t bu = __reduce_min_sync(0xffffffffu, (hi >= 0 && key == kmax) ? (uint32_t)hi : 0xffffffffu);
      const int bi = kmax ? (int)bu : -1;
      if (lane == s) sel_idx = bi;
      if (bi >= 0 && (bi & 31) == lane) {
        taken |= 1u << (bi >> 5);
        rescan();
      }
    }
    // gates from the unbiased probs, renormalised (sum in double, slot order) and scaled (:253-262)
    const float pv = lane < a.top_k ? pp[t * E + sel_idx] : 0.0f;
    double sum = 0.0;
    for (int s = 0; s < a.top_k; ++s) sum = __dadd_rn(sum, (double)__shfl_sync(0xffffffffu, pv, s));
    if (lane < a.top_k) {
      const float fs = __double2float_rn(sum);
      float v = pv;
      if (a.norm_topk) v = __fdiv_rn(v, fs);
      if (a.scale != 1.0f) v = __fmul_rn(v, a.scale);
      const int64_t tok = t0 + t;
      a.idx[tok * a.top_k + lane] = sel_idx;
      a.w[tok * a.top_k + lane] = v;
      atomicAdd(&cnt_s[sel_idx], 1);
    }
  }
  __syncthreads();
  for (int ee = tid; ee < E; ee += RT_THREADS)
    if (cnt_s[ee]) atomicAdd(&a.counts[ee], cnt_s[ee]);
}

// p = sigmoid(logit) into part[0] ([n][e]); the split path also uses part[1 .. h/256 - 1] for
// partials and `arrivals` (router_arrivals(n, e) zeroed ints, left zeroed again).
template <int TM>
static cudaError_t launch_logits_split(const float* x, const float* wrt, float* part, int64_t n, int h, int e,
                                       int32_t* arrivals, int32_t* zero_counts, cudaStream_t st) {
  auto kern = router_logits_split_kernel<TM>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, rl_smem<TM>());
  if (err != cudaSuccess) return err;
  const dim3 grid((unsigned)((n + rl_tok<TM>() - 1) / rl_tok<TM>()), (unsigned)((e + RL_EXP - 1) / RL_EXP),
                  (unsigned)(h / kRouterSeg));
  return launch_pdl(kern, grid, dim3(RL_THREADS), rl_smem<TM>(), st, x, wrt, part, n, h, e, arrivals, zero_counts);
}

template <int TM>
static cudaError_t launch_logits_wide(const float* x, const float* wrt, float* probs, int64_t n, int h, int e,
                                      int32_t* zero_counts, cudaStream_t st) {
  auto kern = router_logits_wide_kernel<TM>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, rw_smem<TM>());
  if (err != cudaSuccess) return err;
  const dim3 grid((unsigned)((n + rw_tok<TM>() - 1) / rw_tok<TM>()), (unsigned)((e + RW_EXP - 1) / RW_EXP));
  return launch_pdl(kern, grid, dim3(RW_THREADS), rw_smem<TM>(), st, x, wrt, probs, n, h, e, zero_counts);
}

cudaError_t launch_router(const float* x, const float* wrt, float* part, int64_t n, int h, int e, RouterPlan plan,
                          int32_t* arrivals, int32_t* zero_counts, cudaStream_t st) {
  if (h % kRouterSeg) return cudaErrorInvalidValue;
  if ((plan == ROUTER_SPLIT2 || plan == ROUTER_SPLIT8) && !arrivals) return cudaErrorInvalidValue;
  switch (plan) {
    case ROUTER_WHOLE:
      return launch_logits_wide<8>(x, wrt, part, n, h, e, zero_counts, st);
    case ROUTER_WHOLE7:
      return launch_logits_wide<7>(x, wrt, part, n, h, e, zero_counts, st);
    case ROUTER_SPLIT8:
      return launch_logits_split<8>(x, wrt, part, n, h, e, arrivals, zero_counts, st);
    case ROUTER_SPLIT2:
      return launch_logits_split<2>(x, wrt, part, n, h, e, arrivals, zero_counts, st);
  }
  return cudaErrorInvalidValue;
}

// Wide whole-K tiles once they give at least every other SM one (a wide tile takes the same time
// whatever the grid: one per SM); below that, 128-token tiles split by 256-k segment while those
// give every SM one; below that, 32-token tiles split by segment. Measured on B200 with the
// 64-expert whole-K tiles (E = 256, H = 4096; router stage, logits + routing), whole / split 128 /
// split 32 tokens:
//   256 tokens   293 /  71 /  59 us        2048 tokens  307 / 175 / 220 us
//   512 tokens   303 /  82 /  86 us        3072 tokens  307 / 230 / 321 us
//   1024 tokens  304 / 117 / 130 us       4096 tokens  310 / 302 / 436 us
// 112-token wide tiles (TM = 7) where they put less work on the busiest SM than 128-token tiles:
// at 8192 tokens 148 tiles of 112 tokens, one per SM, where 128 of 128 tokens leave 20 SMs idle.
RouterPlan router_plan(int64_t n, int e, int h, int sms) {
  const int64_t etiles = (e + RL_EXP - 1) / RL_EXP;
  const int64_t wtiles = (e + RW_EXP - 1) / RW_EXP;
  const int64_t tiles8 = ((n + rl_tok<8>() - 1) / rl_tok<8>()) * etiles;
  const int64_t wide8 = ((n + rw_tok<8>() - 1) / rw_tok<8>()) * wtiles;
  const int64_t wide7 = ((n + rw_tok<7>() - 1) / rw_tok<7>()) * wtiles;
  if (2 * wide7 >= (int64_t)sms)
    return 7 * ((wide7 + sms - 1) / sms) < 8 * ((wide8 + sms - 1) / sms) ? ROUTER_WHOLE7 : ROUTER_WHOLE;
  if (tiles8 * (h / kRouterSeg) >= sms) return ROUTER_SPLIT8;
  return ROUTER_SPLIT2;
}

int64_t router_arrivals(int64_t n, int e) { return ((n + rl_tok<2>() - 1) / rl_tok<2>()) * ((e + RL_EXP - 1) / RL_EXP); }

size_t route_smem_bytes(int64_t tpb, int64_t e) { return sizeof(float) * (size_t)((2 * tpb + 5) * e); }

cudaError_t launch_route(const RouteArgs& a_in, cudaStream_t st) {
  RouteArgs a = a_in;
  const int tpb = a.use_block ? a.blk : 32;
  const int64_t nblocks = (a.n + tpb - 1) / tpb;
  if (a.e % 4) return cudaErrorInvalidValue;
  // few blocks: 4 CTAs per block share its tokens' top-k (each repeats the block-level steps)
  a.tok_split = nblocks < 64 ? 4 : 1;
  const size_t smem = route_smem_bytes(tpb, a.e);
  const cudaError_t err = cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)kRouteSmemMax);
  if (err != cudaSuccess) return err;
  return launch_pdl(route_kernel, dim3((unsigned)(nblocks * a.tok_split)), dim3(RT_THREADS), smem, st, a);
}

}  // namespace dmoe
