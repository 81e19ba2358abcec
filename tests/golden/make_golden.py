"""Generates tests/golden/quant_golden.npz from gguf-py (the reference's Python dependency for GGUF
I/O and quantisation, used by tools/convert-llada2-fast.py and tools/quantize_streaming.py).

gguf-py restates ggml's block formats bit-exactly (its Q8_0 quantiser is documented as matching
ggml-quants.c). The fixtures pin the library's Q8_0 quantiser and the oracle's F16 / Q8_0 / Q4_K
dequantisers without needing gguf-py at test time. Run from the repository root:
    python tests/golden/make_golden.py
"""
import os

import numpy as np
from gguf import quants
from gguf.constants import GGMLQuantizationType as QT

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    rng = np.random.default_rng(20260101)
    out = {}
    # Q8_0: quantise + dequantise 64 blocks of 32 (normal data, a zero block, tiny and huge values)
    x = rng.standard_normal((4, 512)).astype(np.float32) * 0.02
    x[0, :32] = 0.0
    x[1, 32:64] *= 1e-6
    x[2, 64:96] *= 1e4
    out["q80_in"] = x
    q = quants.quantize(x, QT.Q8_0)
    out["q80_bytes"] = np.ascontiguousarray(q).view(np.uint8).reshape(4, -1)
    out["q80_deq"] = quants.dequantize(q, QT.Q8_0).astype(np.float32)
    # Q4_K: dequantise random super-blocks whose d / dmin are finite halves
    nb = 48
    blk = rng.integers(0, 256, size=(nb, 144), dtype=np.uint8)
    d = (rng.standard_normal(nb) * 1e-3).astype(np.float16).view(np.uint8).reshape(nb, 2)
    dm = (np.abs(rng.standard_normal(nb)) * 1e-3).astype(np.float16).view(np.uint8).reshape(nb, 2)
    blk[:, 0:2] = d
    blk[:, 2:4] = dm
    out["q4k_bytes"] = blk.reshape(6, 8 * 144)  # 6 rows of K = 2048
    out["q4k_deq"] = quants.dequantize(out["q4k_bytes"], QT.Q4_K).astype(np.float32)
    # F16: every finite half -> f32, and f32 -> f16 rounding on random and edge values
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    hv = h.view(np.float16)
    fin = np.isfinite(hv)
    out["f16_bits"] = h[fin]
    out["f16_vals"] = hv[fin].astype(np.float32)
    f = np.concatenate([rng.standard_normal(4096).astype(np.float32) * 10.0 ** rng.integers(-8, 5, 4096),
                        np.array([65504.0, 65519.0, 65520.0, 6.1035156e-05, 5.9604645e-08, 2.9802322e-08, -0.0],
                                 dtype=np.float32)]).astype(np.float32)
    out["f32_in"] = f
    out["f32_to_f16"] = f.astype(np.float16).view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
