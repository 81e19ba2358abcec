// Host build of the GEMM kernel's token-tile bounds checks (diffuse-cpp_b200/csrc/tile_check.h)
// for the CPU unit test tests/test_tile_check.py, which compiles this file with g++.
#include "tile_check.h"

extern "C" int tc_tile(int expert, int row0, int nrows, int n_experts, int nt, long long n_tokens, long long rows_total,
                       int* out4) {
  dmoe::TokTile t{expert, row0, nrows, 0};
  int bad = 0;
  const dmoe::TokTile r = dmoe::tile_checked(t, n_experts, nt, n_tokens, rows_total, &bad);
  out4[0] = r.expert;
  out4[1] = r.row0;
  out4[2] = r.nrows;
  out4[3] = r.pad;
  return bad;
}

extern "C" int tc_count(int n_tiles, int cap, int* over) { return dmoe::tile_count_checked(n_tiles, cap, over); }
