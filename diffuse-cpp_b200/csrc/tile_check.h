// tile_check.h — bounds of the routed token-tile list that the GEMM kernels walk.
//
// The list is built on the device (scan_tiles_kernel), so the GEMM kernel checks every tile it
// decodes, and the number of tiles, against the buffers it indexes. A tile outside them is
// decoded as an empty tile (no rows, expert 0, first row n_tokens), which every role of the
// kernel skips in the same way, and the kernel reports it through its error word. Plain C++:
// compiled by nvcc for the kernels and by the host compiler for the CPU unit tests.
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define DMOE_HD __host__ __device__ __forceinline__
#else
#define DMOE_HD inline
#endif

namespace dmoe {

// One token tile of one routed expert: rows [row0, row0 + nrows) of the gathered activation
// buffer all belong to `expert`.
struct TokTile {
  int32_t expert;
  int32_t row0;
  int32_t nrows;
  int32_t pad;
};

// A tile is usable iff its expert is one of the layer's, it holds at most nt rows, and its rows
// lie in the routed part [n_tokens, rows_total) of the gathered buffer.
DMOE_HD bool tile_out_of_bounds(const TokTile& tk, int32_t n_experts, int32_t nt, int64_t n_tokens,
                                int64_t rows_total) {
  return tk.expert < 0 || tk.expert >= n_experts || tk.nrows < 0 || tk.nrows > nt || (int64_t)tk.row0 < n_tokens ||
         (int64_t)tk.row0 + tk.nrows > rows_total;
}

// The tile itself, or the empty tile that stands in for one out of bounds (*bad set to 1).
DMOE_HD TokTile tile_checked(const TokTile& tk, int32_t n_experts, int32_t nt, int64_t n_tokens, int64_t rows_total,
                             int* bad) {
  *bad = tile_out_of_bounds(tk, n_experts, nt, n_tokens, rows_total) ? 1 : 0;
  if (!*bad) return tk;
  TokTile e;
  e.expert = 0;
  e.row0 = (int32_t)n_tokens;
  e.nrows = 0;
  e.pad = 0;
  return e;
}

// Number of routed tiles the kernel walks: the device-built count clamped to [0, cap], the
// capacity of the tile list and of the per-tile counters (*over set to 1 when it had to clamp).
DMOE_HD int32_t tile_count_checked(int32_t n_tiles, int32_t cap, int* over) {
  *over = (n_tiles < 0 || n_tiles > cap) ? 1 : 0;
  return n_tiles < 0 ? 0 : (n_tiles > cap ? cap : n_tiles);
}

}  // namespace dmoe
