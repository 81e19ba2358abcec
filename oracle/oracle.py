"""ctypes wrapper of the CPU oracle (oracle/libdmoe_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline, as the checker. The product never imports it.

The oracle restates Akicou/diffuse-cpp src/diffuse-moe-graph.cpp:195-287 (see dmoe_oracle.h
for the per-function citations). Its GGUF codecs are pinned against gguf-py golden vectors;
its layer maths is unpinned against the reference itself (ggml is absent from the reference
checkout), so it is the definition the CUDA path is checked against.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdmoe_oracle.so")

F32, F16, Q8_0, Q4_K = 0, 1, 8, 12


class OrcLayer(ctypes.Structure):
    _fields_ = [
        ("H", ctypes.c_int64),
        ("I", ctypes.c_int64),
        ("Is", ctypes.c_int64),
        ("E", ctypes.c_int64),
        ("top_k", ctypes.c_int64),
        ("expert_type", ctypes.c_int),
        ("shared_type", ctypes.c_int),
        ("w_gate", ctypes.c_void_p),
        ("w_up", ctypes.c_void_p),
        ("w_down", ctypes.c_void_p),
        ("sw_gate", ctypes.c_void_p),
        ("sw_up", ctypes.c_void_p),
        ("sw_down", ctypes.c_void_p),
    ]


_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    lib = ctypes.CDLL(LIB_PATH)
    P = ctypes.c_void_p
    lib.dmoe_oracle_row_size.argtypes = [ctypes.c_int, ctypes.c_int64]
    lib.dmoe_oracle_row_size.restype = ctypes.c_size_t
    lib.dmoe_oracle_f32_to_f16.argtypes = [ctypes.c_float]
    lib.dmoe_oracle_f32_to_f16.restype = ctypes.c_uint16
    lib.dmoe_oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
    lib.dmoe_oracle_f16_to_f32.restype = ctypes.c_float
    lib.dmoe_oracle_dequant.argtypes = [ctypes.c_int, P, ctypes.c_int64, ctypes.c_int64, P]
    lib.dmoe_oracle_dequant.restype = ctypes.c_int
    lib.dmoe_oracle_exp_neg.argtypes = [ctypes.c_float]
    lib.dmoe_oracle_exp_neg.restype = ctypes.c_float
    lib.dmoe_oracle_sigmoid.argtypes = [ctypes.c_float]
    lib.dmoe_oracle_sigmoid.restype = ctypes.c_float
    lib.dmoe_oracle_logits.argtypes = [P, ctypes.c_int64, ctypes.c_int64, P, ctypes.c_int64, P, ctypes.c_int]
    lib.dmoe_oracle_logits.restype = None
    lib.dmoe_oracle_route.argtypes = [P, ctypes.c_int64, ctypes.c_int64, P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_float, P, P, P, P]
    lib.dmoe_oracle_route.restype = ctypes.c_int
    lib.dmoe_oracle_experts.argtypes = [ctypes.POINTER(OrcLayer), P, ctypes.c_int64, P, P, P, ctypes.c_int,
                                        ctypes.c_int]
    lib.dmoe_oracle_experts.restype = ctypes.c_int
    lib.dmoe_oracle_ggml_dot.argtypes = [ctypes.c_int, P, ctypes.c_int64, ctypes.c_int64, P, P, ctypes.c_int]
    lib.dmoe_oracle_ggml_dot.restype = ctypes.c_int
    lib.dmoe_oracle_ggml_round_act.argtypes = [ctypes.c_int, P, ctypes.c_int64, P]
    lib.dmoe_oracle_ggml_round_act.restype = ctypes.c_int
    lib.dmoe_oracle_sample_step.argtypes = [P, ctypes.c_int64, ctypes.c_int64, P, ctypes.c_int32, ctypes.c_int32,
                                            ctypes.c_float, P, P]
    lib.dmoe_oracle_sample_step.restype = ctypes.c_int32
    _lib = lib
    return lib


def _p(a):
    return None if a is None else a.ctypes.data


def dequant(qtype: int, data: np.ndarray, nrows: int, k: int) -> np.ndarray:
    data = np.ascontiguousarray(data)
    out = np.empty((nrows, k), dtype=np.float32)
    if load().dmoe_oracle_dequant(qtype, data.ctypes.data, nrows, k, out.ctypes.data) != 0:
        raise ValueError("dequant failed")
    return out


def exp_neg(l: float) -> float:
    return load().dmoe_oracle_exp_neg(l)


def sigmoid(l: float) -> float:
    return load().dmoe_oracle_sigmoid(l)


def logits(x: np.ndarray, w_router: np.ndarray, nthreads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    wr = np.ascontiguousarray(w_router, dtype=np.float32)
    n, h = x.shape
    e = wr.shape[0]
    out = np.empty((n, e), dtype=np.float32)
    load().dmoe_oracle_logits(x.ctypes.data, n, h, wr.ctypes.data, e, out.ctypes.data, nthreads)
    return out


def route(lg: np.ndarray, bias, top_k: int, cap: int, blk: int, norm_topk: int = 1, scale: float = 1.0):
    """Returns (idx [n,k] int32, w [n,k] f32, probs [n,e] f32, allowed [n/blk,e] u8 or None, used_block)."""
    lg = np.ascontiguousarray(lg, dtype=np.float32)
    n, e = lg.shape
    idx = np.empty((n, top_k), dtype=np.int32)
    w = np.empty((n, top_k), dtype=np.float32)
    probs = np.empty((n, e), dtype=np.float32)
    nb = n // blk if blk > 0 else 0
    allowed = np.zeros((max(nb, 1), e), dtype=np.uint8)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    used = load().dmoe_oracle_route(lg.ctypes.data, n, e, _p(b), top_k, cap, blk, norm_topk, scale, idx.ctypes.data,
                                    w.ctypes.data, probs.ctypes.data, allowed.ctypes.data)
    return idx, w, probs, (allowed[:nb] if used else None), bool(used)


MODE_EXACT, MODE_F32, MODE_GGML = 0, 1, 2


def ggml_dot(qtype: int, w: np.ndarray, k: int, x: np.ndarray, simd: bool = True) -> np.ndarray:
    """Weight rows (GGUF bytes [rows, row_bytes]) . x rounded to the vec-dot type, as the
    ggml-faithful mode computes them (SIMD or scalar kernel)."""
    w = np.ascontiguousarray(w)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(w.shape[0], np.float32)
    if load().dmoe_oracle_ggml_dot(qtype, w.ctypes.data, w.shape[0], k, x.ctypes.data, out.ctypes.data,
                                   1 if simd else 0) != 0:
        raise ValueError("ggml_dot failed")
    return out


def ggml_round_act(qtype: int, x: np.ndarray) -> np.ndarray:
    """x rounded to the vec-dot type of weight type qtype (Q8_K / Q8_0 / F16), widened to float."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    if load().dmoe_oracle_ggml_round_act(qtype, x.ctypes.data, x.size, out.ctypes.data) != 0:
        raise ValueError("ggml_round_act failed")
    return out


def experts(hp: dict, t: dict, x: np.ndarray, idx: np.ndarray, w: np.ndarray, mode: int = 0,
            nthreads: int = 0) -> np.ndarray:
    """Routed experts + slot sum + shared expert for the given routing. mode 0: double
    accumulation (the reference answer); 1: float accumulation; 2: ggml-faithful (activations
    rounded to the weight type's vec-dot type, integer block dot products)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    L = OrcLayer()
    L.H, L.I, L.Is, L.E, L.top_k = hp["n_embd"], hp["n_ff_exp"], hp.get("n_ff_shexp", 0), hp["n_expert"], hp[
        "n_expert_used"]
    L.expert_type = hp["expert_type"]
    L.shared_type = hp.get("shared_type", hp["expert_type"])
    keep = []
    for name in ("w_gate", "w_up", "w_down", "sw_gate", "sw_up", "sw_down"):
        a = t.get(name)
        if a is not None and L.Is == 0 and name.startswith("sw"):
            a = None
        if a is not None:
            a = np.ascontiguousarray(a)
            keep.append(a)
        setattr(L, name, None if a is None else a.ctypes.data)
    n = x.shape[0]
    out = np.empty((n, L.H), dtype=np.float32)
    rc = load().dmoe_oracle_experts(ctypes.byref(L), x.ctypes.data, n, idx.ctypes.data, w.ctypes.data,
                                    out.ctypes.data, mode, nthreads)
    if rc != 0:
        raise ValueError(f"oracle experts failed ({rc})")
    return out


def layer(hp: dict, t: dict, x: np.ndarray, mode: int = 0, nthreads: int = 0):
    """Full layer: returns (out, idx, w, allowed, used_block)."""
    lg = logits(x, t["w_router"], nthreads)
    idx, w, _, allowed, used = route(lg, t.get("b_router"), hp["n_expert_used"], hp.get("expert_capacity", 48),
                                     hp.get("moe_block_size", 32), hp.get("norm_topk_prob", 1),
                                     hp.get("routed_scaling", 1.0))
    out = experts(hp, t, x, idx, w, mode, nthreads)
    return out, idx, w, allowed, used


def sample_step(logits: np.ndarray, seq, mask_id: int, n_transfer: int, threshold: float):
    """Greedy sampler step (src/diffuse-sampler.cpp:29-49,183-237). logits [n_pos][n_vocab] f32;
    seq [n_pos] int32 or None. Returns (token, prob, seq_after, n_committed)."""
    lib = load()
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    n_pos, n_vocab = lg.shape
    tok = np.empty(n_pos, np.int32)
    pr = np.empty(n_pos, np.float32)
    s = None if seq is None else np.array(seq, dtype=np.int32, copy=True)
    nc = lib.dmoe_oracle_sample_step(_p(lg), n_pos, n_vocab, None if s is None else _p(s), mask_id, n_transfer,
                                     threshold, _p(tok), _p(pr))
    return tok, pr, s, int(nc)
