"""CPU unit test of the token-tile bounds checks the expert GEMM kernel applies to the device-built
tile list (diffuse-cpp_b200/csrc/tile_check.h, compiled here for the host with g++).

A tile outside the buffers must become the empty tile (expert 0, first row n_tokens, no rows)
and be flagged; the tile count must be clamped to the list's capacity and flagged. No GPU run
with a corrupted list is needed: the kernel calls these same functions.
"""
import ctypes
import os
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "diffuse-cpp_b200", "csrc")


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    out = tmp_path_factory.mktemp("tile_check") / "libtc.so"
    subprocess.run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-I", CSRC, os.path.join(HERE, "tile_check_host.cpp"),
                    "-o", str(out)], check=True)
    L = ctypes.CDLL(str(out))
    L.tc_tile.argtypes = [ctypes.c_int] * 5 + [ctypes.c_longlong, ctypes.c_longlong, ctypes.POINTER(ctypes.c_int)]
    L.tc_tile.restype = ctypes.c_int
    L.tc_count.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    L.tc_count.restype = ctypes.c_int
    return L


# layer of E = 16 experts, NT = 32, 100 tokens, gathered rows [0, 100) shared + [100, 900) routed
E, NT, NTOK, ROWS = 16, 32, 100, 900


def check(lib, expert, row0, nrows):
    out = (ctypes.c_int * 4)()
    bad = lib.tc_tile(expert, row0, nrows, E, NT, NTOK, ROWS, out)
    return bad, tuple(out)


@pytest.mark.parametrize("tile", [(0, 100, 32), (15, 868, 32), (3, 500, 0), (7, 899, 1), (0, 100, 1)])
def test_tiles_in_bounds_pass_unchanged(lib, tile):
    bad, out = check(lib, *tile)
    assert bad == 0
    assert out[:3] == tile


@pytest.mark.parametrize("tile", [
    (16, 100, 32),   # expert == E
    (-1, 100, 32),   # negative expert
    (0, 99, 32),     # row0 inside the shared rows (row0 < n_tokens)
    (0, 869, 32),    # row0 + nrows == rows_total + 1
    (0, 100, 33),    # nrows == NT + 1
    (0, 100, -1),    # negative row count
    (2, -5, 3),      # negative row0
])
def test_tiles_out_of_bounds_become_empty(lib, tile):
    bad, out = check(lib, *tile)
    assert bad == 1
    assert out == (0, NTOK, 0, 0)


@pytest.mark.parametrize("n,cap,want,over", [(0, 10, 0, 0), (10, 10, 10, 0), (11, 10, 10, 1), (-3, 10, 0, 1),
                                             (5, 0, 0, 1)])
def test_tile_count_clamped_to_capacity(lib, n, cap, want, over):
    o = ctypes.c_int(-1)
    assert lib.tc_count(n, cap, ctypes.byref(o)) == want
    assert o.value == over
