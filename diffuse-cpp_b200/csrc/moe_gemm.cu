// moe_gemm.cu — grouped expert GEMMs of the block-routed MoE layer on sm_100a tensor cores.
//
// Replaces the three ggml_mul_mat_id calls, the SwiGLU, the gating multiply, the slot sum and
// the shared expert of the reference layer (src/diffuse-moe-graph.cpp:264-286) with two
// launches of one persistent kernel template:
//
//   MODE_GATEUP: h[row][i] = silu(Wg_e[i] . x_row) * (Wu_e[i] . x_row)   -> fp16 hbuf
//   MODE_DOWN:   out[tok][o] += w_row * (Wd_e[o] . h_row)                  -> fp32 out (red.add)
//                (256 output rows per tile: two 128-row MMA tiles share one activation tile)
//                or, for large N, y[row][o] = w_row * (Wd_e[o] . h_row) summed by combine_kernel
//
// "Swap-AB" orientation: weights are the MMA's M side (128 rows per tile), the tokens of one
// expert the N side (NT per tile), K runs along the GGUF rows, so quantised weights stream
// through TMA in their native block layout.
//
// Warp roles (one CTA per SM, persistent over a device-side tile list):
//   warp 0      TMA producer: weight tiles (raw GGUF bytes / fp16) + activation tiles -> smem ring
//   warp 1      TMEM allocator + MMA issuer (tcgen05.mma kind::f16, fp32 accumulators in TMEM)
//   warps 2..9  epilogue: tcgen05.ld of the accumulators, SwiGLU (gate/up) or weighted rows /
//               reductions (down), stored straight from the accumulator lanes
//   warps 10..  dequant warpgroups: q4_K / q8_0 tile -> fp16 in registers -> tcgen05.st into
//               TMEM (the A operand of the TS-form MMA, no shared-memory round trip)
// F16 weights skip the dequant: TMA lands them 128B-swizzled and the SS-form MMA reads smem.
//
// q4_K K-order: a q4_K 32-bit word of quants holds bytes b0..b3 of weights (k, k+1, k+2, k+3)
// (low nibbles) and (k+32 .. k+35) (high nibbles). The masks 0x000F000F / (>>8) extract the
// pairs (k, k+2) and (k+1, k+3) with one LOP3 each, so the MMA's K order inside every aligned
// quad is (0, 2, 1, 3). The activations for a q4_K matrix are written with the same quad swap
// (gather kernel for x, gate/up epilogue for h); the dot products are unchanged.
#include <algorithm>
#include <atomic>

#include "dmoe_internal.h"
#include "sm100.cuh"

namespace dmoe {

// PAIR: a cluster of two CTAs shares each tile through tcgen05 cta_group::2 (M = 256): CTA r
// dequantises weight rows [128 r, 128 r + 128) of a 256-row tile into its own TMEM and loads its
// half of the NT tokens; the leader (rank 0) issues the MMAs, which read both CTAs' halves and
// write each CTA's 128 rows x NT accumulator. Each activation tile then crosses L2 once per 256
// rows instead of once per 128. Quantised weights at NT = 128 only.
// BRES (down launches, quantised weights, NT = 64): the CTA keeps one token tile's activations
// (NT rows x K <= kBresK, 128 KB) resident in shared memory and runs every 256-row m-tile of the
// down matrix against it, so the activations cross L2 once per token tile instead of once per
// m-tile; the stage ring carries weights only. The CTA walks whole units (group, token tile,
// m-chunk) of consecutive m-tiles.
static_assert(kBresK == 1024 && kBresNT == 64, "the host's BRES limits (dmoe_internal.h) match the kernel's");

template <int WT, int MODE, int NT, int NDQ_ = 2, bool PAIR_ = false, bool BRES_ = false>
struct GemmCfg {
  static constexpr bool QUANT = (WT != WT_F16);
  static constexpr bool FUSED = MODE == MODE_FUSED;
  static constexpr bool PAIR = PAIR_;
  static constexpr bool BRES = BRES_;
  static_assert(!BRES || (QUANT && MODE == MODE_DOWN && ((NT == kBresNT && !PAIR) || (NT == 2 * kBresNT && PAIR))),
                "resident activation tiles: quantised down launches, 64 token rows per CTA");
  static constexpr int B_ROWS = PAIR ? NT / 2 : NT;  // token rows of B this CTA loads
  // two weight tiles share each activation (B) tile: gate and up, or (down, NT <= 64) two
  // adjacent 128-row blocks of the down matrix, so B crosses L2 once per 256 output rows. At
  // NT = 128 the down tile keeps one block: two 128-column accumulators would leave TMEM no room
  // to double-buffer them, and the epilogue's overlap with the next tile is worth more there.
  static constexpr int MATS = (MODE != MODE_DOWN || NT <= 64) ? 2 : 1;
  static_assert(!FUSED || NT <= 64, "the fused launch needs the two-block down tiles");
  static_assert(!PAIR || (QUANT && !FUSED && NT == 128), "pair tiles: quantised weights, NT = 128, separate launches");
  // output rows per tile of one expert matrix, for a tile of mode `tmode`
  static constexpr int out_rows(int tmode) {
    return PAIR ? 2 * kMTile : (tmode == MODE_GATEUP ? kMTile : MATS * kMTile);
  }
  static constexpr int STAGE_K = (WT == WT_Q4_K) ? 256 : 128;
  // A block: the K range one dequant hand-off covers (TMEM columns ABK = AK / 2 per matrix).
  // CTA pairs use 64-K blocks: their single-buffered 256-column accumulator leaves room for only
  // two 128-K blocks, so each dequant warpgroup would own one buffer and strictly alternate with
  // the MMA; four 64-K buffers let a warpgroup fill its next buffer while the MMA reads the last.
  static constexpr int AK = (PAIR && QUANT) ? 64 : 128;
  static constexpr int ABK = AK / 2;
  static constexpr int KB_PER_STAGE = STAGE_K / AK;
  static constexpr int B_BYTES = STAGE_K * B_ROWS * 2;
  // per matrix per stage: q4_K 128 rows x one 144 B super-block; q8_0 128 x 128 int8 (SW128)
  // + 128 x 4 fp32 scales; f16 two SW128 boxes of 128 x 64.
  static constexpr int W_BYTES = (WT == WT_Q4_K) ? 128 * 144 : (WT == WT_Q8_0) ? (128 * 128 + 128 * 16) : (128 * 128 * 2);
  // BRES: the resident activation tile, K / 64 128B-swizzled boxes of NT rows, before the ring
  static constexpr int BRES_BYTES = BRES ? kBresK * B_ROWS * 2 : 0;
  static constexpr int STAGE_B = BRES ? 0 : B_BYTES;  // activation bytes carried by each stage
  static constexpr int STAGE_BYTES = STAGE_B + MATS * W_BYTES;
  // roles: warp 0 TMA producer, warp 1 MMA issuer, warps 2-9 epilogue (two per TMEM lane
  // quarter, one per column half), then NDQ dequant warpgroups
  static constexpr int NDQ = QUANT ? NDQ_ : 0;
  static constexpr int EPI_WARP0 = 2, EPI_WARPS = 8, DQ_WARP0 = EPI_WARP0 + EPI_WARPS;
  static constexpr int THREADS = 32 * (DQ_WARP0 + 4 * NDQ);
  static constexpr int EPI_COLS = NT / 2;  // accumulator columns per epilogue warp
  static constexpr int SMEM_BUDGET = 227 * 1024 - 2048;
  static constexpr int STAGES_RAW = (SMEM_BUDGET - BRES_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 6 ? 6 : STAGES_RAW;
  // TMEM: accumulators (double-buffered when they fit next to a 2+ deep A ring), A ring
  static constexpr int ACC_COLS = MATS * NT;
  static constexpr int A_COLS = MATS * ABK;
  static constexpr int ACC_BUFS = (2 * ACC_COLS + (QUANT ? 2 * A_COLS : 0) <= 512) ? 2 : 1;
  static constexpr int NA_RAW = QUANT ? (512 - ACC_BUFS * ACC_COLS) / A_COLS : 0;
  static constexpr int NA = NA_RAW > 4 ? 4 : NA_RAW;
  static constexpr int SMEM_BYTES = BRES_BYTES + STAGES * STAGE_BYTES + 1024 + 256;
  // gate/up launches: dequant warps convert a k-block's first matrix into 64 registers before
  // its A buffer is free, where the launch leaves each thread the registers (two dequant
  // warpgroups: 576 threads, up to 112 registers each). Measured on B200: gate/up 492 -> 471 us
  // at 64 x 32 tokens; the down launches (their epilogue holds more registers) lost 5-8 %.
  static constexpr bool PRECONVERT = QUANT && NDQ <= 2 && MODE == MODE_GATEUP;
  // every dequant warp arrives on each stage's `empty` (after its own k-blocks, if any)
  static constexpr int EMPTY_COUNT = 1 + 4 * NDQ;
  static_assert(STAGES >= 2, "smem ring needs two stages");
  static_assert(!QUANT || NA >= 2, "TMEM A ring needs two buffers");
  static_assert(B_BYTES % 1024 == 0 && W_BYTES % 1024 == 0 && BRES_BYTES % 1024 == 0, "1024-B aligned stage parts");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
  static_assert(NT % 32 == 0 && NT >= 32 && NT <= 256, "tcgen05 M=128 needs N % 16 == 0; two column halves");
  static_assert(ACC_BUFS * ACC_COLS + NA * A_COLS <= 512, "TMEM budget");
  // The dequant warpgroups share the A ring round-robin (k-block kbs -> group kbs % NDQ,
  // buffer kbs % NA). A group then waits for buffer use u only after the MMA has consumed
  // k-block kbs - NDQ - NA, which implies completion u - 1 of that buffer's `aempty` iff
  // NA >= NDQ; with fewer buffers a parity wait could alias two completions ahead.
  static constexpr bool RING_OK = !QUANT || NA >= NDQ;
};

// mode: MODE_GATEUP or MODE_DOWN (per tile in a fused launch); ttx: the token tile's index in
// the fused launch's completion counters (shared tiles first, then routed)
// bad: a routed tile whose rows or expert fall outside the buffers (a corrupt tile list); it is
// decoded as an empty tile, so every role skips it the same way, and the producer reports it
// BRES walk: skip = no work at this index (past the last unit, or the empty half of a list tile:
// every role skips it alike); bfirst / blast = first / last m-tile of its unit (the producer
// loads the unit's activation tile before the first, the MMA releases it after the last)
struct TileInfo {
  int group, expert, row0, nrows, mt, k0, k1, mode, ttx, bad, skip, bfirst, blast;
};

// routed token tiles in the device-built list, clamped to the list's capacity
__device__ __forceinline__ int routed_tiles(const GemmParams& p) {
  int over;
  return tile_count_checked(*p.n_tiles, p.tiles_cap, &over);
}

__device__ __forceinline__ int tiles_in(const GemmParams& p, const GemmGroup* gr) {
  const int n0 = gr[0].present ? p.n_shared_tt * gr[0].n_mt * p.ksplit : 0;
  const int n1 = gr[1].present ? routed_tiles(p) * gr[1].n_mt * p.ksplit : 0;
  return n0 + n1;
}

template <int MODE>
__device__ __forceinline__ int tiles_total(const GemmParams& p) {
  return tiles_in(p, p.grp) + (MODE == MODE_FUSED ? tiles_in(p, p.grp_dn) : 0);
}

template <int MODE, int NT>
__device__ __forceinline__ TileInfo decode_tile(const GemmParams& p, int t) {
  TileInfo ti;
  ti.bad = 0;
  ti.mode = MODE == MODE_FUSED ? MODE_GATEUP : MODE;
  const GemmGroup* gr = p.grp;
  if (MODE == MODE_FUSED) {
    const int ngu = tiles_in(p, p.grp);
    if (t >= ngu) {
      t -= ngu;
      ti.mode = MODE_DOWN;
      gr = p.grp_dn;
    }
  }
  const int n0 = gr[0].present ? p.n_shared_tt * gr[0].n_mt * p.ksplit : 0;
  int per_tt, r;
  if (t < n0) {
    ti.group = 0;
    per_tt = gr[0].n_mt * p.ksplit;
    const int tt = t / per_tt;
    r = t - tt * per_tt;
    ti.expert = 0;
    ti.row0 = tt * NT;
    const int64_t left = p.n_tokens - (int64_t)ti.row0;
    ti.nrows = left < NT ? (int)left : NT;
    ti.ttx = tt;
  } else {
    t -= n0;
    ti.group = 1;
    per_tt = gr[1].n_mt * p.ksplit;
    const int tt = t / per_tt;
    r = t - tt * per_tt;
    const TokTile tk = tile_checked(p.tiles[tt], p.n_experts, NT, p.n_tokens, p.rows_total, &ti.bad);
    ti.expert = tk.expert;
    ti.row0 = tk.row0;
    ti.nrows = tk.nrows;
    ti.ttx = p.n_shared_tt + tt;
  }
  ti.mt = r / p.ksplit;
  const int ks = r - ti.mt * p.ksplit;
  const int ksz = gr[ti.group].k_stages / p.ksplit;
  ti.k0 = ks * ksz;
  ti.k1 = ti.k0 + ksz;
  ti.skip = 0;
  ti.bfirst = ti.blast = 0;
  return ti;
}

// ---- BRES walk (resident activation tiles; down launches, no split-K) -----------------------
// Units: (group 0, shared token tile, chunk) first, then (group 1, routed token tile, chunk),
// a routed list tile of NT * tile_div rows giving tile_div token tiles of NT rows. Every unit
// has mpu = n_mt / bres_chunks consecutive m-tiles. CTA b of G takes units b, b + G, ... and
// runs each unit's m-tiles in order: walk index t = b + G k holds m-tile k % mpu of unit
// b + G (k / mpu).
__device__ __forceinline__ int bres_units(const GemmParams& p) {
  const int u0 = p.grp[0].present ? p.n_shared_tt * p.bres_chunks : 0;
  const int u1 = p.grp[1].present ? routed_tiles(p) * p.tile_div * p.bres_chunks : 0;
  return u0 + u1;
}
__device__ __forceinline__ int bres_mpu(const GemmParams& p) {
  return (p.grp[0].present ? p.grp[0].n_mt : p.grp[1].n_mt) / p.bres_chunks;
}
__device__ __forceinline__ int bres_total(const GemmParams& p, int G) {
  return (bres_units(p) + G - 1) / G * G * bres_mpu(p);
}

template <int NT>
__device__ __forceinline__ TileInfo decode_tile_bres(const GemmParams& p, int t, int G) {
  TileInfo ti;
  ti.bad = 0;
  ti.mode = MODE_DOWN;
  ti.ttx = 0;
  const int mpu = bres_mpu(p);
  const int b = t % G, k = t / G;
  int u = b + (k / mpu) * G;
  const int j = k % mpu;
  ti.bfirst = j == 0;
  ti.blast = j == mpu - 1;
  ti.skip = u >= bres_units(p);
  const int u0 = p.grp[0].present ? p.n_shared_tt * p.bres_chunks : 0;
  int tt, c;
  if (!ti.skip && u < u0) {
    ti.group = 0;
    tt = u / p.bres_chunks;
    c = u - tt * p.bres_chunks;
    ti.expert = 0;
    ti.row0 = tt * NT;
    const int64_t left = p.n_tokens - (int64_t)ti.row0;
    ti.nrows = left < NT ? (int)left : NT;
  } else {
    u -= u0;
    ti.group = 1;
    tt = ti.skip ? 0 : u / p.bres_chunks;
    c = ti.skip ? 0 : u - tt * p.bres_chunks;
    const int tl = tt / p.tile_div, half = tt - tl * p.tile_div;
    if (ti.skip) {
      ti.expert = 0;
      ti.row0 = (int)p.n_tokens;
      ti.nrows = 0;
    } else {
      const TokTile tk = tile_checked(p.tiles[tl], p.n_experts, NT * p.tile_div, p.n_tokens, p.rows_total, &ti.bad);
      ti.expert = tk.expert;
      ti.row0 = tk.row0 + half * NT;
      const int left = tk.nrows - half * NT;
      ti.nrows = left < 0 ? 0 : (left < NT ? left : NT);
      ti.skip = ti.nrows == 0;  // the empty half of a short list tile, or a tile out of bounds
    }
  }
  ti.mt = c * mpu + j;
  ti.k0 = 0;
  ti.k1 = p.grp[ti.group].k_stages;
  return ti;
}

__device__ __forceinline__ int ld_acquire_gpu(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
  return d;
}
__device__ __forceinline__ __half2 as_h2(uint32_t u) {
  __half2 h;
  memcpy(&h, &u, 4);
  return h;
}
__device__ __forceinline__ uint32_t as_u32(__half2 h) {
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}

// Bounded mbarrier wait that also gives up when another role of this CTA has aborted.
__device__ __forceinline__ bool role_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t errbit,
                                          volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > DMOE_WAIT_NS) {
      atomicOr(err, errbit);
      *abort_flag = 1;
      return false;
    }
  }
}

// Fused launch: waits (bounded, like every wait here) until `*ctr` reaches `target`, i.e. every
// gate/up epilogue warp of the token tile has published its h rows; then orders those generic-
// proxy writes before this thread's TMA reads of them.
__device__ __forceinline__ bool wait_count(const int32_t* ctr, int target, uint32_t* err, volatile int* abort_flag) {
  if (ld_acquire_gpu(ctr) < target) {
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_gpu(ctr) < target) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > DMOE_WAIT_NS) {
        atomicOr(err, ERRBIT_TIMEOUT_DEP);
        *abort_flag = 1;
        return false;
      }
      __nanosleep(64);
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// Warp-uniform forms for roles whose whole warp walks the schedule: every lane waits, and
// lane 0's verdict is the warp's, so the warp stays converged around its tcgen05 issue blocks.
__device__ __forceinline__ bool warp_role_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t errbit,
                                               volatile int* abort_flag) {
  const bool ok = role_wait(bar, parity, err, errbit, abort_flag);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}
__device__ __forceinline__ bool warp_abort(volatile int* abort_flag) {
  return __shfl_sync(0xffffffffu, *abort_flag, 0) != 0;
}

// ------------------------------------------------------------------------------------------
// dequantisation of one 128-K block of one weight row into 64 TMEM columns (fp16 pairs)
// ------------------------------------------------------------------------------------------
// q4_K: `rowp` = shared address of the row's 144-byte super-block; kb selects K half 0/1.
// Low nibbles: (q & 0x000F000F) | 0x6400 -> 1024 + q, exact; minus 1024 -> q; fma(q, d, -m).
// High nibbles: (q & 0x00F000F0) | 0x6400 -> 1024 + 16 q; minus 1024 -> 16 q (exact);
// fma(16 q, d / 16, -m) with d / 16 an exact power-of-two rescaling of d (no shift needed).
// Writes the row's 64 packed halves (TMEM columns 0..63 of the k-block's A block) into v.
// NGL = 2: the whole 128-K half kb (64 columns); NGL = 1: its 64-K quarter gl0 (32 columns).
template <int NGL>
__device__ __forceinline__ void q4k_convert(uint32_t rowp, int kb, int gl0, uint32_t (&v)[32 * NGL]) {
  const uint4 hdr = lds128(rowp);
  const __half2 dd = as_h2(__byte_perm(hdr.x, 0, 0x1010));    // {d, d}
  const __half2 dmn = as_h2(__byte_perm(hdr.x, 0, 0x3232));   // {dmin, dmin}
  uint32_t scw, mw;
  if (kb == 0) {
    scw = hdr.y & 0x3F3F3F3Fu;
    mw = hdr.z & 0x3F3F3F3Fu;
  } else {
    scw = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
    mw = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
  }
  const __half2 k1024 = __float2half2_rn(1024.0f);
  const __half2 k1_16 = __float2half2_rn(0.0625f);
  // 6-bit ints -> fp16 exactly (magic 1024), then one rounding of d*sc / dmin*m
  const __half2 sc01 = __hsub2(as_h2(__byte_perm(scw, 0x64646464u, 0x5140)), k1024);
  const __half2 sc23 = __hsub2(as_h2(__byte_perm(scw, 0x64646464u, 0x5342)), k1024);
  const __half2 mn01 = __hsub2(as_h2(__byte_perm(mw, 0x64646464u, 0x5140)), k1024);
  const __half2 mn23 = __hsub2(as_h2(__byte_perm(mw, 0x64646464u, 0x5342)), k1024);
  const __half2 dq01 = __hmul2(sc01, dd), dq23 = __hmul2(sc23, dd);
  const __half2 nm01 = __hneg2(__hmul2(mn01, dmn)), nm23 = __hneg2(__hmul2(mn23, dmn));
  // all of this K half's quants (64 bytes) are loaded before the first TMEM store
  const uint32_t qp = rowp + 16 + 64 * kb + 32 * gl0;
  const uint4 q0 = lds128(qp), q1 = lds128(qp + 16);
  uint4 q2 = q0, q3 = q1;
  if constexpr (NGL == 2) {
    q2 = lds128(qp + 32);
    q3 = lds128(qp + 48);
  }
#pragma unroll
  for (int gi = 0; gi < NGL; ++gi) {
    const int gl = gl0 + gi;
    // sub-blocks 2 gl (low nibbles) and 2 gl + 1 (high nibbles) of this K half
    const __half2 dlo = gl == 0 ? __low2half2(dq01) : __low2half2(dq23);
    const __half2 dhi = __hmul2(gl == 0 ? __high2half2(dq01) : __high2half2(dq23), k1_16);
    const __half2 mlo = gl == 0 ? __low2half2(nm01) : __low2half2(nm23);
    const __half2 mhi = gl == 0 ? __high2half2(nm01) : __high2half2(nm23);
    const uint4 qa = gi == 0 ? q0 : q2, qb = gi == 0 ? q1 : q3;
    const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    // columns [32 gi, 32 gi + 16): low nibbles; [32 gi + 16, 32 gi + 32): high nibbles
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t q = qw[w], q8 = q >> 8;
      const uint32_t v02 = lop3_and_or(q, 0x000F000Fu, 0x64006400u);
      const uint32_t v13 = lop3_and_or(q8, 0x000F000Fu, 0x64006400u);
      const uint32_t h02 = lop3_and_or(q, 0x00F000F0u, 0x64006400u);
      const uint32_t h13 = lop3_and_or(q8, 0x00F000F0u, 0x64006400u);
      v[32 * gi + 2 * w] = as_u32(__hfma2(__hsub2(as_h2(v02), k1024), dlo, mlo));
      v[32 * gi + 2 * w + 1] = as_u32(__hfma2(__hsub2(as_h2(v13), k1024), dlo, mlo));
      v[32 * gi + 16 + 2 * w] = as_u32(__hfma2(__hsub2(as_h2(h02), k1024), dhi, mhi));
      v[32 * gi + 16 + 2 * w + 1] = as_u32(__hfma2(__hsub2(as_h2(h13), k1024), dhi, mhi));
    }
  }
}

// q8_0 (repacked): `qtile` = shared address of a 128 x 128 int8 tile (128B-swizzled), `stile` =
// 128 x 4 fp32 scales. NB 32-quant blocks from blk0 (NB = 4: the whole row, 64 columns).
template <int NB>
__device__ __forceinline__ void q80_convert(uint32_t qtile, uint32_t stile, int row, int blk0, uint32_t (&v)[16 * NB]) {
  const float4 sc = lds128f(stile + row * 16);
  const float scv[4] = {sc.x, sc.y, sc.z, sc.w};
  const __half2 k1152 = __float2half2_rn(1152.0f);
  const uint32_t rp = qtile + row * 128;
  uint4 qv8[2 * NB];  // the blocks' quants, loaded before the first TMEM store
#pragma unroll
  for (int c = 0; c < 2 * NB; ++c) qv8[c] = lds128(rp + (((2 * blk0 + c) ^ (row & 7)) << 4));
#pragma unroll
  for (int bi = 0; bi < NB; ++bi) {  // columns [16 bi, 16 bi + 16): 32-quant block blk0 + bi
    const __half2 d2 = __float2half2_rn(scv[blk0 + bi]);
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const uint4 qv = qv8[2 * bi + cc];
      const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint32_t xq = qw[w] ^ 0x80808080u;
        const uint32_t v0 = __byte_perm(xq, 0x64646464u, 0x5140);
        const uint32_t v1 = __byte_perm(xq, 0x64646464u, 0x5342);
        v[16 * bi + 8 * cc + 2 * w] = as_u32(__hmul2(__hsub2(as_h2(v0), k1152), d2));
        v[16 * bi + 8 * cc + 2 * w + 1] = as_u32(__hmul2(__hsub2(as_h2(v1), k1152), d2));
      }
    }
  }
}

// one weight row's A block `ab` (ABK packed halves: 64 for 128 K, 32 for 64 K) of weight tile
// `wt` (q4_K super-block rows or a q8_0 tile)
template <int WT, int ABK>
__device__ __forceinline__ void convert_ablock(uint32_t wt, int row, int ab, uint32_t (&v)[ABK]) {
  static_assert(ABK == 64 || ABK == 32, "A blocks of 128 or 64 K");
  if constexpr (WT == WT_Q4_K) {
    if constexpr (ABK == 64) q4k_convert<2>(wt + row * 144, ab, 0, v);
    else q4k_convert<1>(wt + row * 144, ab >> 1, ab & 1, v);
  } else {
    if constexpr (ABK == 64) q80_convert<4>(wt, wt + 128 * 128, row, 0, v);
    else q80_convert<2>(wt, wt + 128 * 128, row, 2 * ab, v);
  }
}
template <int NC>
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t (&v)[NC]) {
#pragma unroll
  for (int j = 0; j < NC / 16; ++j) tmem_st16(taddr + 16 * j, *reinterpret_cast<const uint32_t(*)[16]>(&v[16 * j]));
}

// silu(g) = g * (1 / (1 + e^-g)); for g -> -inf the reciprocal of inf is 0 and the product -0
__device__ __forceinline__ float silu_f(float g) { return g * __frcp_rn(1.0f + __expf(-g)); }

__device__ __forceinline__ int quad_swap(int i) { return (i & ~3) | ((i & 1) << 1) | ((i >> 1) & 1); }

template <int WT, int MODE, int NT, int NDQ_, bool PAIR, bool BRES = false>
__global__ void __launch_bounds__(GemmCfg<WT, MODE, NT, NDQ_, PAIR, BRES>::THREADS, 1)
    moe_gemm_kernel(const __grid_constant__ GemmParams p) {
  using C = GemmCfg<WT, MODE, NT, NDQ_, PAIR, BRES>;
  static_assert(C::RING_OK, "A ring needs at least one buffer per dequant warpgroup");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // layout: [BRES: resident activation tile] [stage ring] [barriers]
  uint8_t* bres = smem;
  uint8_t* ring = smem + C::BRES_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + C::STAGES * C::STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = full + C::STAGES;
  uint64_t* afull = empty + C::STAGES;
  uint64_t* aempty = afull + 4;
  uint64_t* accfull = aempty + 4;
  uint64_t* accempty = accfull + 2;
  uint64_t* full_b = accempty + 2;  // PAIR: both CTAs' activation halves landed (leader's copy counts)
  // BRES: the resident tile has landed (TMA bytes) / is free again (MMA commit after a unit)
  uint64_t* bfull = full_b + (C::PAIR ? C::STAGES : 0);
  uint64_t* bempty = bfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bempty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = C::PAIR ? cluster_ctarank() : 0u;  // 0 = leader of the pair
  // PAIR: the leader's copy of barrier `b` (in the shared::cluster window)
  auto leader = [&](uint64_t* b) -> uint32_t { return mapa_shared(smem_u32(b), 0); };
  // waits: barriers that receive arrivals from the peer CTA acquire at cluster scope
  auto bwait = [&](uint64_t* bar, uint32_t parity, uint32_t errbit) -> bool {
    if constexpr (C::PAIR) {
      if (mbar_try_wait_cluster(bar, parity)) return true;
      const uint64_t t0 = globaltimer_ns();
      while (true) {
        for (int i = 0; i < 32; ++i)
          if (mbar_try_wait_cluster(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > DMOE_WAIT_NS) {
          atomicOr(p.err, errbit);
          *abort_flag = 1;
          return false;
        }
      }
    } else {
      return role_wait(bar, parity, p.err, errbit, abort_flag);
    }
  };
  auto wbwait = [&](uint64_t* bar, uint32_t parity, uint32_t errbit) -> bool {
    const bool ok = bwait(bar, parity, errbit);
    return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], C::EMPTY_COUNT);
    }
    for (int a = 0; a < 4; ++a) {
      mbar_init(&afull[a], C::PAIR ? 8 : 4);  // PAIR: both CTAs' dequant warps arrive on the leader's
      mbar_init(&aempty[a], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], C::PAIR ? 2 * C::EPI_WARPS : C::EPI_WARPS);
    }
    if (C::PAIR)
      for (int s = 0; s < C::STAGES; ++s) mbar_init(&full_b[s], 1);
    mbar_init(bfull, 1);
    mbar_init(bempty, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (C::PAIR) {
      tmem_alloc_pair(tmem_slot, 512);  // the same warp of both CTAs, same slot offset
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 512);
      tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    for (int g = 0; g < 2; ++g) {
      if (!p.grp[g].present) continue;
      tma_prefetch_desc(&p.tm_w[g][0]);
      if (MODE != MODE_DOWN) tma_prefetch_desc(&p.tm_w[g][1]);
      if (MODE == MODE_FUSED) tma_prefetch_desc(&p.tm_w_dn[g]);
    }
    tma_prefetch_desc(&p.tm_b);
    if (MODE == MODE_FUSED) tma_prefetch_desc(&p.tm_b_dn);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (C::PAIR) cluster_sync();  // the peer's barriers are initialised before any arrival
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  // everything above overlaps the previous kernel's tail; global memory only after this
  pdl_wait();
  pdl_trigger();
  // tile walk: one CTA per SM, or (PAIR) one pair per two SMs, both CTAs on the same tiles;
  // BRES: whole units per CTA (decode_tile_bres)
  const int t_first = C::PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int t_step = C::PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int total = C::BRES ? bres_total(p, t_step) : tiles_total<MODE>(p);
  auto decode = [&](int t) -> TileInfo {
    if constexpr (C::BRES) return decode_tile_bres<NT>(p, t, t_step);
    else return decode_tile<MODE, NT>(p, t);
  };

  auto stage_ptr = [&](int s) -> uint8_t* { return ring + s * C::STAGE_BYTES; };
  auto wtile_ptr = [&](int s, int m) -> uint8_t* { return ring + s * C::STAGE_BYTES + C::STAGE_B + m * C::W_BYTES; };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    // (whole warp walks the schedule; one elected lane issues each stage's copies)
    // weights read by one token tile stream through L2 (evict first); weights of experts with
    // several token tiles are re-read and kept (evict normal) -- chosen by the host
    const uint64_t pol_w = p.w_keep ? l2_policy_evict_normal() : l2_policy_evict_first();
    if (blockIdx.x == 0 && lane == 0 && (p.grp[1].present || (MODE == MODE_FUSED && p.grp_dn[1].present))) {
      int over;
      tile_count_checked(*p.n_tiles, p.tiles_cap, &over);
      if (over) atomicOr(p.err, ERRBIT_BAD_TILE);  // more routed tiles than the list holds
    }
    uint32_t stage_seq = 0, unit_seq = 0;
    for (int t = t_first; t < total && !warp_abort(abort_flag); t += t_step) {
      const TileInfo ti = decode(t);
      if (ti.bad && lane == 0) atomicOr(p.err, ERRBIT_BAD_TILE);
      if (ti.skip) continue;
      if (C::BRES && ti.bfirst) {
        // the unit's activation tile: all K of its NT rows, once the previous unit's MMAs are done
        // (PAIR: each CTA its half of the rows, counted on the leader's bfull, armed by the leader)
        if (!wbwait(bempty, (unit_seq & 1u) ^ 1u, ERRBIT_TIMEOUT_EMPTY)) break;
        if (elect_one()) {
          const int nbox = p.grp[ti.group].k_stages * C::STAGE_K / 64;
          if constexpr (C::PAIR) {
            if (rank == 0) mbar_arrive_expect_tx(bfull, (uint32_t)(2 * nbox * C::B_ROWS * 128));
            for (int bx = 0; bx < nbox; ++bx)
              tma_load_2d_pair(bres + bx * C::B_ROWS * 128, &p.tm_b, bx * 64, ti.row0 + (int)rank * C::B_ROWS,
                               leader(bfull));
          } else {
            mbar_arrive_expect_tx(bfull, (uint32_t)(nbox * NT * 128));
            for (int bx = 0; bx < nbox; ++bx) tma_load_2d(bres + bx * NT * 128, &p.tm_b, bx * 64, ti.row0, bfull);
          }
        }
        __syncwarp();
        ++unit_seq;
      }
      const bool dn = ti.mode == MODE_DOWN;
      const bool dn_fused = C::FUSED && dn;
      const GemmGroup& gg = dn_fused ? p.grp_dn[ti.group] : p.grp[ti.group];
      const int wrow = ti.expert * gg.rows_per_exp + ti.mt * C::out_rows(ti.mode);
      const CUtensorMap* tmb = dn_fused ? &p.tm_b_dn : &p.tm_b;
      if (dn_fused) {
        // the token tile's h rows: written by all of its gate/up tiles' epilogue warps
        bool ready = true;
        if (lane == 0) ready = wait_count(p.tt_done + ti.ttx, p.grp[ti.group].n_mt * C::EPI_WARPS, p.err, abort_flag);
        if (!__shfl_sync(0xffffffffu, ready ? 1 : 0, 0)) break;
      }
      bool ok = true;
      for (int kc = ti.k0; kc < ti.k1; ++kc) {
        const int s = stage_seq % C::STAGES;
        const uint32_t ph = (stage_seq / C::STAGES) & 1u;
        if (!wbwait(&empty[s], ph ^ 1u, ERRBIT_TIMEOUT_EMPTY)) { ok = false; break; }
        if (elect_one()) {
          if constexpr (C::PAIR) {
            // weights count on this CTA's full[s]; both CTAs' activation halves on the leader's
            // full_b[s] (its expected bytes are armed by the leader alone)
            mbar_arrive_expect_tx(&full[s], C::MATS * C::W_BYTES);
            if constexpr (!C::BRES) {
              if (rank == 0) mbar_arrive_expect_tx(&full_b[s], 2 * C::B_BYTES);
#pragma unroll
              for (int bx = 0; bx < C::STAGE_K / 64; ++bx)
                tma_load_2d_pair(stage_ptr(s) + bx * C::B_ROWS * 128, tmb, kc * C::STAGE_K + bx * 64,
                                 ti.row0 + (int)rank * C::B_ROWS, leader(&full_b[s]));
            }
          } else {
            mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
            if constexpr (!C::BRES) {
#pragma unroll
              for (int bx = 0; bx < C::STAGE_K / 64; ++bx)
                tma_load_2d(stage_ptr(s) + bx * NT * 128, tmb, kc * C::STAGE_K + bx * 64, ti.row0, &full[s]);
            }
          }
#pragma unroll
          for (int m = 0; m < C::MATS; ++m) {
            uint8_t* wt = wtile_ptr(s, m);
            // gate/up: matrix m at the tile's rows; down: the one matrix, row block m; a pair's
            // CTA r takes the 128-row half r of the tile
            const CUtensorMap* tw = dn_fused ? &p.tm_w_dn[ti.group] : &p.tm_w[ti.group][dn ? 0 : m];
            const CUtensorMap* ts = dn_fused ? &p.tm_s_dn[ti.group] : &p.tm_s[ti.group][dn ? 0 : m];
            const int wr = wrow + (dn ? m * kMTile : 0) + (int)rank * kMTile;
            if constexpr (WT == WT_Q4_K) {
              tma_load_2d_hint(wt, tw, kc * 144, wr, &full[s], pol_w);
            } else if constexpr (WT == WT_Q8_0) {
              tma_load_2d_hint(wt, tw, kc * 128, wr, &full[s], pol_w);
              tma_load_2d_hint(wt + 128 * 128, ts, kc * 4, wr, &full[s], pol_w);
            } else {
              tma_load_2d_hint(wt, tw, kc * 128, wr, &full[s], pol_w);
              tma_load_2d_hint(wt + 128 * 128, tw, kc * 128 + 64, wr, &full[s], pol_w);
            }
          }
        }
        __syncwarp();
        ++stage_seq;
      }
      if (!ok) break;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp walks the schedule, waits included, and one elected lane issues each
    // k-block's MMAs as one straight-line block. Issued this way a kind::f16 M=128 MMA costs
    // 24 / 32 / 64 cycles at N = 32 / 64 / 128; issued from a lane-0-only branch it costs
    // 46 cycles or more even at N <= 64, and a run-time branch between two MMAs about 100.
    // PAIR: only the leader's warp issues; its MMAs read both CTAs' A (TMEM) and B (shared
    // memory) halves at the same addresses and write both CTAs' accumulators, and its commits
    // arrive on the barriers of both CTAs.
    constexpr uint32_t idesc = idesc_f16_f32(C::PAIR ? 256 : 128, NT);
    uint32_t stage_seq = 0, tile_seq = 0, unit_seq = 0;
    for (int t = t_first; t < total && !warp_abort(abort_flag) && (!C::PAIR || rank == 0); t += t_step) {
      const TileInfo ti = decode(t);
      if (ti.skip) continue;
      const int ab = tile_seq % C::ACC_BUFS;
      const uint32_t aph = (tile_seq / C::ACC_BUFS) & 1u;
      if (!wbwait(&accempty[ab], aph ^ 1u, ERRBIT_TIMEOUT_TMEM)) break;
      if (C::BRES && ti.bfirst) {
        if (!wbwait(bfull, unit_seq & 1u, ERRBIT_TIMEOUT_FULL)) break;
        ++unit_seq;
      }
      tc_fence_after();
      const uint32_t dbase = tbase + ab * C::ACC_COLS;
      bool first = true;
      bool ok = true;
      for (int kc = ti.k0; kc < ti.k1 && ok; ++kc) {
        const int s = stage_seq % C::STAGES;
        const uint32_t ph = (stage_seq / C::STAGES) & 1u;
        // a pair's stage carries only weights under BRES, which reach the MMA through the dequant
        // warps' afull arrivals: nothing to wait for here
        if constexpr (!(C::PAIR && C::BRES)) {
          if (!wbwait(C::PAIR ? &full_b[s] : &full[s], ph, ERRBIT_TIMEOUT_FULL)) { ok = false; break; }
        }
        tc_fence_after();
        // Shared-memory descriptors are built once per stage; each (k-block, k-step) slice adds
        // a compile-time offset to the 14-bit start-address field (no carry: smem < 256 KB).
        // BRES: the stage's K range of the resident tile (boxes of 64 K, B_ROWS rows each).
        const uint64_t bdesc0 = sdesc_sw128(
            C::BRES ? smem_u32(bres + kc * (C::STAGE_K / 64) * C::B_ROWS * 128) : smem_u32(stage_ptr(s)), 1024);
        const uint32_t acc_first = first ? 0u : 1u;
        if constexpr (C::QUANT) {
#pragma unroll
          for (int kb = 0; kb < C::KB_PER_STAGE; ++kb) {
            const uint32_t kbs = stage_seq * C::KB_PER_STAGE + kb;
            const int a = kbs % C::NA;
            const uint32_t u = kbs / C::NA;
            if (!wbwait(&afull[a], u & 1u, ERRBIT_TIMEOUT_TMEM)) { ok = false; break; }
            tc_fence_after();
            const uint32_t abuf = tbase + C::ACC_BUFS * C::ACC_COLS + a * C::A_COLS;
            constexpr int JS = C::ABK / 8;  // 16-K steps per A block
            static_assert(JS == 8 || JS == 4, "A block steps");
            if (elect_one()) {
#pragma unroll
              for (int j = 0; j < JS; ++j) {
                // K offset kb AK + 16 j: its 64-K box, then 32 bytes per 16-K step inside it
                const int kofs = kb * C::AK + 16 * j;
                const uint64_t bdesc = bdesc0 + (uint64_t)(((kofs / 64) * (C::B_ROWS * 128) + (kofs % 64) * 2) >> 4);
                const uint32_t acc = (kb == 0 && j == 0) ? acc_first : 1u;
#pragma unroll
                for (int m = 0; m < C::MATS; ++m) {
                  if constexpr (C::PAIR)
                    mma_f16_ts_pair(dbase + m * NT, abuf + m * C::ABK + 8 * j, bdesc, idesc, acc);
                  else
                    mma_f16_ts(dbase + m * NT, abuf + m * C::ABK + 8 * j, bdesc, idesc, acc);
                }
              }
              if constexpr (C::PAIR) mma_commit_pair(&aempty[a]);
              else mma_commit(&aempty[a]);
            }
            __syncwarp();
          }
          if (!ok) break;
        } else {
          uint64_t adesc0[C::MATS];
#pragma unroll
          for (int m = 0; m < C::MATS; ++m) adesc0[m] = sdesc_sw128(smem_u32(wtile_ptr(s, m)), 1024);
          if (elect_one()) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint64_t bdesc = bdesc0 + (uint64_t)(((j / 4) * (NT * 128) + (j % 4) * 32) >> 4);
              const uint32_t acc = j == 0 ? acc_first : 1u;
#pragma unroll
              for (int m = 0; m < C::MATS; ++m) {
                const uint64_t adesc = adesc0[m] + (uint64_t)(((j / 4) * (128 * 128) + (j % 4) * 32) >> 4);
                mma_f16_ss(dbase + m * NT, adesc, bdesc, idesc, acc);
              }
            }
          }
          __syncwarp();
        }
        first = false;
        if (elect_one()) {
          if constexpr (C::PAIR) mma_commit_pair(&empty[s]);
          else mma_commit(&empty[s]);
        }
        __syncwarp();
        ++stage_seq;
      }
      if (!ok) break;
      if (elect_one()) {
        if constexpr (C::PAIR) mma_commit_pair(&accfull[ab]);
        else mma_commit(&accfull[ab]);
        // BRES: after the unit's last m-tile the resident tile may be overwritten
        if (C::BRES && ti.blast) {
          if constexpr (C::PAIR) mma_commit_pair(bempty);  // both CTAs' halves are free
          else mma_commit(bempty);
        }
      }
      __syncwarp();
      ++tile_seq;
    }
  } else if (warp < C::DQ_WARP0) {
    // ------------------------------------------------------------------ epilogue
    // Warp w reads TMEM lane quarter w % 4 (the hardware's rule) and column half (w - 2) / 4.
    // Lane = output feature, so every store below covers one contiguous 64 / 128-byte segment
    // of a token's row; the down tile's gate weights and token ids sit in registers, loaded
    // before the accumulator wait.
    constexpr int HC = C::EPI_COLS, NCH = HC / 16, NWR = (HC + 31) / 32;
    const int quarter = warp & 3;
    const int cb = ((warp - C::EPI_WARP0) >> 2) * HC;  // first accumulator column of this warp
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint32_t tile_seq = 0;
    for (int t = t_first; t < total && !*abort_flag; t += t_step) {
      const TileInfo ti = decode(t);
      if (ti.skip) continue;
      const int ab = tile_seq % C::ACC_BUFS;
      const uint32_t aph = (tile_seq / C::ACC_BUFS) & 1u;
      float wv[NWR];
      int tv[NWR];
#pragma unroll
      for (int j = 0; j < NWR; ++j) {
        const int c = cb + 32 * j + lane;
        const bool routed = ti.mode == MODE_DOWN && ti.group != 0 && c < ti.nrows && 32 * j + lane < HC;
        wv[j] = routed ? p.pair_w[ti.row0 + c] : 1.0f;
        tv[j] = (routed && p.y == nullptr) ? p.pair_tok[ti.row0 + c] : ti.row0 + c;
      }
      if (!bwait(&accfull[ab], aph, ERRBIT_TIMEOUT_MMA)) break;
      tc_fence_after();
      const uint32_t dbase = tbase + lane_off + ab * C::ACC_COLS;
      // first output feature of this warp (a pair's CTA r holds rows [128 r, 128 r + 128) of the tile)
      const int obase = ti.mt * C::out_rows(ti.mode) + (int)rank * kMTile + quarter * 32;
      bool released = false;
      if (ti.mode == MODE_GATEUP && p.gu_acc == nullptr) {
        // h = silu(g) * u for this warp's columns, kept as packed halves: the accumulator is
        // released before the stores, so the next tile's MMAs (single-buffered accumulators at
        // NT = 128) overlap them
        uint32_t hv[NCH][8];
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          const int c0 = cb + 16 * ch;
          if (c0 < ti.nrows) {  // warp-uniform
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {  // 8 columns at a time keeps g and u in 16 registers
              uint32_t g[8], u[8];
              tmem_ld8(dbase + c0 + 8 * hh, g);
              tmem_ld8(dbase + NT + c0 + 8 * hh, u);
              tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 8; c += 2) {
                const float h0 = silu_f(__uint_as_float(g[c])) * __uint_as_float(u[c]);
                const float h1 = silu_f(__uint_as_float(g[c + 1])) * __uint_as_float(u[c + 1]);
                hv[ch][4 * hh + c / 2] = as_u32(__floats2half2_rn(h0, h1));
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (C::PAIR) mbar_arrive_cluster(leader(&accempty[ab]));
          else mbar_arrive(&accempty[ab]);
        }
        released = true;
        // into the (possibly quad-swapped) h row: one 64-byte segment of a token's row per store
        const int pl = ((p.h_quad_swap >> ti.group) & 1) ? quad_swap(lane) : lane;
        __half* hcol = p.hbuf + (int64_t)(ti.row0 + cb) * p.h_ld + obase + pl;
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) {
          if (cb + 16 * ch >= ti.nrows) break;
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (cb + 16 * ch + c < ti.nrows)
              hcol[(int64_t)(16 * ch + c) * p.h_ld] =
                  __ushort_as_half((unsigned short)((c & 1) ? (hv[ch][c / 2] >> 16) : (hv[ch][c / 2] & 0xffffu)));
        }
      }
#pragma unroll
      for (int ch = 0; ch < NCH && !released; ++ch) {
        const int c0 = cb + 16 * ch;
        if (c0 >= ti.nrows) break;  // warp-uniform
        if (ti.mode == MODE_GATEUP) {
          uint32_t acc0[16];
          tmem_ld16(dbase + c0, acc0);
          uint32_t acc1[16];
          tmem_ld16(dbase + NT + c0, acc1);
          tmem_wait_ld();
          // split-K: fp32 partial sums of g and u
          const int64_t r0 = ti.row0 + c0;
          float* gcol = p.gu_acc + r0 * (2 * p.gu_half) + obase + lane;
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (c0 + c < ti.nrows) {
              atomicAdd(gcol + (int64_t)c * (2 * p.gu_half), __uint_as_float(acc0[c]));
              atomicAdd(gcol + (int64_t)c * (2 * p.gu_half) + p.gu_half, __uint_as_float(acc1[c]));
            }
        } else {
#pragma unroll 1
         for (int m = 0; m < C::MATS; ++m) {  // row block m: accumulator columns [m NT, (m + 1) NT)
          uint32_t acc0[16];
          tmem_ld16(dbase + m * NT + c0, acc0);
          const int ob = obase + m * kMTile;
          tmem_wait_ld();
          if (p.y != nullptr) {
            // shared rows into out, routed rows weighted into y
            if (ti.group == 0) {
              float* ocol = p.out + (int64_t)(ti.row0 + c0) * p.out_ld + ob + lane;
#pragma unroll
              for (int c = 0; c < 16; ++c)
                if (c0 + c < ti.nrows) ocol[(int64_t)c * p.out_ld] = __uint_as_float(acc0[c]);
            } else {
              float* ycol = p.y + (int64_t)(ti.row0 + c0 - p.n_tokens) * p.y_ld + ob + lane;
#pragma unroll
              for (int c = 0; c < 16; ++c) {
                const int k = 16 * ch + c;
                const float wgt = __shfl_sync(0xffffffffu, wv[k >> 5], k & 31);
                if (c0 + c < ti.nrows) ycol[(int64_t)c * p.y_ld] = __uint_as_float(acc0[c]) * wgt;
              }
            }
          } else {
            // out[tok] += w * y, fp32 reductions of one 128-byte segment per token
#pragma unroll
            for (int c = 0; c < 16; ++c) {
              const int k = 16 * ch + c;
              const float wgt = __shfl_sync(0xffffffffu, wv[k >> 5], k & 31);
              const int tok = __shfl_sync(0xffffffffu, tv[k >> 5], k & 31);
              float* dst = ti.group == 0 ? p.out : p.out_routed;
              if (c0 + c < ti.nrows) atomicAdd(dst + (int64_t)tok * p.out_ld + ob + lane, __uint_as_float(acc0[c]) * wgt);
            }
          }
         }
        }
      }
      if (C::FUSED && ti.mode == MODE_GATEUP) {
        // publish this warp's h rows of the token tile to the down tiles that wait for them
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(p.tt_done + ti.ttx, 1);
      }
      if (!released) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (C::PAIR) mbar_arrive_cluster(leader(&accempty[ab]));
          else mbar_arrive(&accempty[ab]);
        }
      }
      ++tile_seq;
    }
  } else if constexpr (C::QUANT) {
    // ------------------------------------------------------------------ dequant warpgroups
    const int wg = (warp - C::DQ_WARP0) >> 2;  // 0 .. NDQ-1
    const int quarter = warp & 3;              // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;       // weight row inside the 128-row tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint32_t stage_seq = 0;
    bool ok = true;
    for (int t = t_first; t < total && ok && !*abort_flag; t += t_step) {
      const TileInfo ti = decode(t);
      if (ti.skip) continue;
      for (int kc = ti.k0; kc < ti.k1; ++kc) {
        const int s = stage_seq % C::STAGES;
        const uint32_t ph = (stage_seq / C::STAGES) & 1u;
        if (!bwait(&full[s], ph, ERRBIT_TIMEOUT_FULL)) { ok = false; break; }
#pragma unroll
        for (int kb = 0; kb < C::KB_PER_STAGE; ++kb) {
          const uint32_t kbs = stage_seq * C::KB_PER_STAGE + kb;
          if ((int)(kbs % C::NDQ) != wg) continue;
          const int a = kbs % C::NA;
          const uint32_t u = kbs / C::NA;
          // the first matrix is converted while the A buffer may still be in use (PRECONVERT),
          // so only its TMEM store waits for the buffer
          uint32_t v[C::ABK];
          if constexpr (C::PRECONVERT) convert_ablock<WT, C::ABK>(smem_u32(wtile_ptr(s, 0)), row, kb, v);
          if (!bwait(&aempty[a], (u & 1u) ^ 1u, ERRBIT_TIMEOUT_TMEM)) { ok = false; break; }
          tc_fence_after();
          const uint32_t abuf = tbase + lane_off + C::ACC_BUFS * C::ACC_COLS + a * C::A_COLS;
#pragma unroll
          for (int m = 0; m < C::MATS; ++m) {
            if (!C::PRECONVERT || m > 0) convert_ablock<WT, C::ABK>(smem_u32(wtile_ptr(s, m)), row, kb, v);
            tmem_st_cols<C::ABK>(abuf + m * C::ABK, v);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (C::PAIR) mbar_arrive_cluster(leader(&afull[a]));  // the leader's MMAs read it
            else mbar_arrive(&afull[a]);
          }
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        ++stage_seq;
      }
    }
  }

  // ---------------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  // PAIR: the leader's MMAs write the peer's TMEM and arrive on its barriers, and the peer's
  // copies count on the leader's barriers: neither CTA releases TMEM or exits before both are done
  if constexpr (C::PAIR) cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (C::PAIR) tmem_dealloc_pair(tbase, 512);
    else tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------------------------------------
// launcher
// ------------------------------------------------------------------------------------------
template <int WT, int MODE, int NT, int NDQ, bool PAIR, bool BRES = false>
static cudaError_t launch_one(const GemmParams& p, int grid, cudaStream_t st) {
  using C = GemmCfg<WT, MODE, NT, NDQ, PAIR, BRES>;
  auto kern = moe_gemm_kernel<WT, MODE, NT, NDQ, PAIR, BRES>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  if constexpr (!PAIR) {
    return launch_pdl(kern, dim3(grid), dim3(C::THREADS), C::SMEM_BYTES, st, p);
  } else {
    // clusters of two CTAs; as many pairs as can be resident at once (the tile walk assumes a
    // persistent grid), counted once per instantiation (the library runs on B200s only, so every
    // device of the process gives the same count; concurrent first calls store the same value)
    static std::atomic<int> max_pairs{0};
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    if (max_pairs.load(std::memory_order_relaxed) == 0) {
      cfg.gridDim = dim3(grid & ~1);
      cfg.numAttrs = 1;
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      if (e != cudaSuccess) return e;
      if (n < 1) return cudaErrorInvalidConfiguration;
      max_pairs.store(n, std::memory_order_relaxed);
    }
    cfg.gridDim = dim3(2 * std::min(grid / 2, max_pairs.load(std::memory_order_relaxed)));
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
  }
}

// Launches with `ndq` dequant warpgroups when that configuration keeps NA >= NDQ, otherwise
// with the largest smaller one that does (2 always does).
template <int WT, int MODE, int NT, bool PAIR = false>
static cudaError_t launch_ndq(const GemmParams& p, int ndq, int grid, cudaStream_t st) {
  if constexpr (WT == WT_F16) {
    return launch_one<WT, MODE, NT, 2, false>(p, grid, st);
  } else {
    if constexpr (GemmCfg<WT, MODE, NT, 4, PAIR>::RING_OK) {
      if (ndq >= 4) return launch_one<WT, MODE, NT, 4, PAIR>(p, grid, st);
    }
    if constexpr (GemmCfg<WT, MODE, NT, 3, PAIR>::RING_OK) {
      if (ndq >= 3) return launch_one<WT, MODE, NT, 3, PAIR>(p, grid, st);
    }
    return launch_one<WT, MODE, NT, 2, PAIR>(p, grid, st);
  }
}

template <int WT, int MODE>
static cudaError_t launch_nt(const GemmParams& p, int nt, int ndq, bool pair, int grid, cudaStream_t st) {
  switch (nt) {
    case 32: return launch_ndq<WT, MODE, 32>(p, ndq, grid, st);
    case 64: return launch_ndq<WT, MODE, 64>(p, ndq, grid, st);
    case 128:
      if constexpr (MODE != MODE_FUSED) {
        if constexpr (WT != WT_F16) {
          if (pair) return launch_ndq<WT, MODE, 128, true>(p, ndq, grid, st);
        }
        return launch_ndq<WT, MODE, 128>(p, ndq, grid, st);
      }
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_moe_gemm(int wtype, int mode, int nt, int ndq, bool pair, const GemmParams& p, int grid,
                            cudaStream_t st) {
  if (pair && !gemm_pair_ok(wtype, mode, nt)) return cudaErrorInvalidValue;
  if (mode == MODE_GATEUP) {
    switch (wtype) {
      case WT_Q4_K: return launch_nt<WT_Q4_K, MODE_GATEUP>(p, nt, ndq, pair, grid, st);
      case WT_Q8_0: return launch_nt<WT_Q8_0, MODE_GATEUP>(p, nt, ndq, pair, grid, st);
      case WT_F16: return launch_nt<WT_F16, MODE_GATEUP>(p, nt, ndq, pair, grid, st);
    }
  } else if (mode == MODE_FUSED) {
    switch (wtype) {
      case WT_Q4_K: return launch_nt<WT_Q4_K, MODE_FUSED>(p, nt, ndq, pair, grid, st);
      case WT_Q8_0: return launch_nt<WT_Q8_0, MODE_FUSED>(p, nt, ndq, pair, grid, st);
      case WT_F16: return launch_nt<WT_F16, MODE_FUSED>(p, nt, ndq, pair, grid, st);
    }
  } else {
    switch (wtype) {
      case WT_Q4_K: return launch_nt<WT_Q4_K, MODE_DOWN>(p, nt, ndq, pair, grid, st);
      case WT_Q8_0: return launch_nt<WT_Q8_0, MODE_DOWN>(p, nt, ndq, pair, grid, st);
      case WT_F16: return launch_nt<WT_F16, MODE_DOWN>(p, nt, ndq, pair, grid, st);
    }
  }
  return cudaErrorInvalidValue;
}

bool gemm_pair_ok(int wtype, int mode, int nt) { return wtype != WT_F16 && mode != MODE_FUSED && nt == 128; }

cudaError_t launch_moe_gemm_bres(int wtype, bool pair, int ndq, const GemmParams& p, int grid, cudaStream_t st) {
  if (p.ksplit != 1 || p.tile_div < 1 || p.bres_chunks < 1) return cudaErrorInvalidValue;
  if (pair) {
    // NT = 128 split over the pair, one 128-row block per CTA: the A ring has room for 4 dequant
    // warpgroups
    switch (wtype) {
      case WT_Q4_K:
        return ndq >= 4 ? launch_one<WT_Q4_K, MODE_DOWN, 2 * kBresNT, 4, true, true>(p, grid, st)
                        : launch_one<WT_Q4_K, MODE_DOWN, 2 * kBresNT, 2, true, true>(p, grid, st);
      case WT_Q8_0:
        return ndq >= 4 ? launch_one<WT_Q8_0, MODE_DOWN, 2 * kBresNT, 4, true, true>(p, grid, st)
                        : launch_one<WT_Q8_0, MODE_DOWN, 2 * kBresNT, 2, true, true>(p, grid, st);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (wtype) {
    case WT_Q4_K: return launch_one<WT_Q4_K, MODE_DOWN, kBresNT, 2, false, true>(p, grid, st);
    case WT_Q8_0: return launch_one<WT_Q8_0, MODE_DOWN, kBresNT, 2, false, true>(p, grid, st);
    default: return cudaErrorInvalidValue;
  }
}

int gemm_stage_k(int wtype) { return wtype == WT_Q4_K ? 256 : 128; }

int gemm_out_rows(int mode, int nt, bool pair) {
  if (pair) return 2 * kMTile;
  return mode == MODE_GATEUP ? kMTile : (nt <= 64 ? 2 * kMTile : kMTile);
}

}  // namespace dmoe
