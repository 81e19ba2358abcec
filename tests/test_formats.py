"""GGUF block formats against gguf-py golden vectors (tests/golden/make_golden.py).

Pins the library's Q8_0 quantiser (bit-identical to ggml's rule) and the oracle's F16 / Q8_0 / Q4_K
dequantisers, bit for bit, plus quantiser round-trip quality for Q4_K (the library's own search).
"""
import os

import numpy as np
import pytest

import diffuse_moe as dm
import oracle

GOLD = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "quant_golden.npz"))


def test_f16_decode_all_halves():
    bits, vals = GOLD["f16_bits"], GOLD["f16_vals"]
    lib = oracle.load()
    got = np.array([lib.dmoe_oracle_f16_to_f32(int(b)) for b in bits[::7]], dtype=np.float32)
    assert np.array_equal(got.view(np.uint32), vals[::7].view(np.uint32))


def test_f16_encode_rounding():
    lib = oracle.load()
    f, ref = GOLD["f32_in"], GOLD["f32_to_f16"]
    got = np.array([lib.dmoe_oracle_f32_to_f16(float(v)) for v in f], dtype=np.uint16)
    assert np.array_equal(got, ref)
    # the library's own F16 quantiser agrees
    q = dm.quantize(f[None, : (len(f) // 32) * 32], dm.TYPE_F16).view(np.uint16)[0]
    assert np.array_equal(q, ref[: len(q)])


def test_q8_0_quantiser_matches_gguf_bytes():
    x, ref = GOLD["q80_in"], GOLD["q80_bytes"]
    assert np.array_equal(dm.quantize(x, dm.TYPE_Q8_0), ref)


def test_q8_0_dequant_matches_gguf():
    q, ref = GOLD["q80_bytes"], GOLD["q80_deq"]
    got = oracle.dequant(oracle.Q8_0, q, q.shape[0], ref.shape[1])
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_q4_k_dequant_matches_gguf():
    q, ref = GOLD["q4k_bytes"], GOLD["q4k_deq"]
    got = oracle.dequant(oracle.Q4_K, q, q.shape[0], ref.shape[1])
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_q4_k_quantiser_round_trip():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((16, 4096)) * 0.02).astype(np.float16).astype(np.float32)
    q = dm.quantize(x, dm.TYPE_Q4_K)
    assert q.shape == (16, 16 * 144)
    y = oracle.dequant(oracle.Q4_K, q, 16, 4096)
    rel = np.linalg.norm(y - x) / np.linalg.norm(x)
    assert rel < 0.12, rel  # 4-bit affine quantisation of Gaussian data: ~8-10 % RMS error


def test_quantized_sizes():
    assert dm.quantized_size(dm.TYPE_Q4_K, 3, 4096) == 3 * 16 * 144
    assert dm.quantized_size(dm.TYPE_Q8_0, 2, 2048) == 2 * 64 * 34
    assert dm.quantized_size(dm.TYPE_F16, 5, 128) == 5 * 256
    assert dm.quantized_size(dm.TYPE_Q4_K, 1, 100) == 0


def test_live_against_gguf_if_installed():
    quants = pytest.importorskip("gguf.quants")
    from gguf.constants import GGMLQuantizationType as QT

    rng = np.random.default_rng(11)
    x = (rng.standard_normal((8, 1024)) * 0.05).astype(np.float32)
    assert np.array_equal(dm.quantize(x, dm.TYPE_Q8_0), np.asarray(quants.quantize(x, QT.Q8_0)).view(np.uint8))
    q = dm.quantize(x, dm.TYPE_Q4_K)
    ref = quants.dequantize(q, QT.Q4_K).astype(np.float32)
    got = oracle.dequant(oracle.Q4_K, q, 8, 1024)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
