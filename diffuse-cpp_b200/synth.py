"""Seeded synthetic MoE layers with the shapes and value distributions of the benchmark configs.

There are no public checkpoints or datasets on this path: every config is synthetic.
  weights  ~ N(0, 0.02), rounded to F16, then quantised (Q8_0 / Q4_K) with the library's own
           quantiser (dmoe_quantize), in the GGUF layouts of the reference converter
           (tools/convert-llada2-fast.py: experts stacked [E][I][H] / [E][H][I]).
  router   ~ N(0, 0.02) f32 [E][H];  expert_bias ~ U(-0.05, 0.05), or for the skewed config
           0.5 * log(zipf_w[perm]) with zipf_w_k proportional to k^-1.1 over a random permutation.
  input    ~ N(0, 1) per element, RMS-normalised per token (x / sqrt(mean x^2 + 1e-6)).
Random streams: router and bias from numpy default_rng([seed, 0]); expert matrix m of expert e
from the counter-based generator of libdmoe_synth.so, stream 3 e + m (gate, up, down), the
shared expert's streams 3 E + m; inputs from default_rng([seed, 1]).
"""
from __future__ import annotations

import ctypes
import dataclasses
import os
from typing import Optional

import numpy as np

import diffuse_moe as dm


@dataclasses.dataclass
class LayerSpec:
    H: int
    I: int
    Is: int
    E: int
    top_k: int = 8
    cap: int = 48
    blk: int = 32
    scale: float = 2.5
    norm_topk: int = 1
    expert_type: int = dm.TYPE_Q4_K
    shared_type: Optional[int] = None
    bias: str = "uniform"  # "uniform" | "zipf" | "none"
    seed: int = 0
    std: float = 0.02

    @property
    def stype(self) -> int:
        return self.expert_type if self.shared_type is None else self.shared_type

    def hparams(self) -> dict:
        return dict(n_embd=self.H, n_ff_exp=self.I, n_ff_shexp=self.Is, n_expert=self.E, n_expert_used=self.top_k,
                    expert_capacity=self.cap, moe_block_size=self.blk, routed_scaling=self.scale,
                    norm_topk_prob=self.norm_topk, expert_type=self.expert_type, shared_type=self.stype)


# The benchmark configs (shapes of the small LLaDA2-style layer and the LLaDA2.2-flash layer)
def config(name: str) -> LayerSpec:
    if name == "c1":  # small layer, F16, 1 block
        return LayerSpec(H=2048, I=512, Is=512, E=256, expert_type=dm.TYPE_F16, seed=0)
    if name == "c2":  # small layer, q8_0, 64 blocks
        return LayerSpec(H=2048, I=512, Is=512, E=256, expert_type=dm.TYPE_Q8_0, seed=1)
    if name == "c3":  # flash layer, q4_K
        return LayerSpec(H=4096, I=1024, Is=1024, E=256, expert_type=dm.TYPE_Q4_K, seed=2)
    if name == "c4":  # flash layer, q4_K, Zipf-skewed expert bias
        return LayerSpec(H=4096, I=1024, Is=1024, E=256, expert_type=dm.TYPE_Q4_K, bias="zipf", seed=3)
    if name == "tiny":
        return LayerSpec(H=256, I=256, Is=256, E=16, top_k=4, cap=6, blk=32, expert_type=dm.TYPE_Q4_K, seed=7)
    raise KeyError(name)


_synth_lib = None


def _synth():
    global _synth_lib
    if _synth_lib is None:
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libdmoe_synth.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with `make -C diffuse-cpp_b200`")
        lib = ctypes.CDLL(path)
        lib.dmoe_synth_normal_f16.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, ctypes.c_float,
                                              ctypes.c_void_p]
        lib.dmoe_synth_normal_f16.restype = None
        _synth_lib = lib
    return _synth_lib


def normal_f16(seed: int, stream: int, shape, std: float) -> np.ndarray:
    """N(0, std^2) rounded to F16 from the counter-based generator (thread-count independent)."""
    out = np.empty(shape, dtype=np.float16)
    _synth().dmoe_synth_normal_f16(seed, stream, out.size, std, out.ctypes.data)
    return out


def _weights(seed: int, stream: int, rows: int, k: int, std: float, qtype: int) -> np.ndarray:
    w = normal_f16(seed, stream, (rows, k), std)
    if qtype == dm.TYPE_F16:
        return w.view(np.uint8).reshape(rows, 2 * k)
    return dm.quantize(w.astype(np.float32), qtype)


def make_layer(spec: LayerSpec) -> dict:
    """Returns the layer's GGUF tensors (numpy) for MoELayer / the oracle."""
    rng = np.random.default_rng([spec.seed, 0])
    E, H, I, Is = spec.E, spec.H, spec.I, spec.Is
    t = {}
    t["w_router"] = rng.standard_normal((E, H), dtype=np.float32) * np.float32(spec.std)
    if spec.bias == "uniform":
        t["b_router"] = rng.uniform(-0.05, 0.05, size=E).astype(np.float32)
    elif spec.bias == "zipf":
        k = np.arange(1, E + 1, dtype=np.float64)
        zw = k ** -1.1
        zw /= zw.sum()
        perm = rng.permutation(E)
        b = np.empty(E, dtype=np.float64)
        b[perm] = 0.5 * np.log(zw)
        t["b_router"] = b.astype(np.float32)
    else:
        t["b_router"] = None
    rs_h = dm.quantized_size(spec.expert_type, 1, H)
    rs_i = dm.quantized_size(spec.expert_type, 1, I)
    t["w_gate"] = np.empty((E * I, rs_h), dtype=np.uint8)
    t["w_up"] = np.empty((E * I, rs_h), dtype=np.uint8)
    t["w_down"] = np.empty((E * H, rs_i), dtype=np.uint8)
    sd = spec.seed
    for e in range(E):
        t["w_gate"][e * I:(e + 1) * I] = _weights(sd, 3 * e, I, H, spec.std, spec.expert_type)
        t["w_up"][e * I:(e + 1) * I] = _weights(sd, 3 * e + 1, I, H, spec.std, spec.expert_type)
        t["w_down"][e * H:(e + 1) * H] = _weights(sd, 3 * e + 2, H, I, spec.std, spec.expert_type)
    if Is > 0:
        t["sw_gate"] = _weights(sd, 3 * E, Is, H, spec.std, spec.stype)
        t["sw_up"] = _weights(sd, 3 * E + 1, Is, H, spec.std, spec.stype)
        t["sw_down"] = _weights(sd, 3 * E + 2, H, Is, spec.std, spec.stype)
    else:
        t["sw_gate"] = t["sw_up"] = t["sw_down"] = None
    return t


_named_cache: dict = {}


def cached_layer(name: str) -> dict:
    """make_layer(config(name)), built once per process (the flash-shaped layers take ~30 s)."""
    if name not in _named_cache:
        _named_cache[name] = make_layer(config(name))
    return _named_cache[name]


def make_input(n: int, H: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng([seed, 1])
    x = rng.standard_normal((n, H), dtype=np.float32)
    ms = np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True)
    return (x / np.sqrt(ms + 1e-6)).astype(np.float32)


def expert_bytes(spec: LayerSpec) -> int:
    """Bytes of one routed expert (gate + up + down)."""
    return 2 * spec.I * dm.quantized_size(spec.expert_type, 1, spec.H) + spec.H * dm.quantized_size(
        spec.expert_type, 1, spec.I)


def shared_bytes(spec: LayerSpec) -> int:
    if spec.Is == 0:
        return 0
    return 2 * spec.Is * dm.quantized_size(spec.stype, 1, spec.H) + spec.H * dm.quantized_size(spec.stype, 1, spec.Is)


def flops_per_token(spec: LayerSpec) -> int:
    return 2 * spec.H * spec.E + spec.top_k * 6 * spec.H * spec.I + 6 * spec.H * spec.Is
