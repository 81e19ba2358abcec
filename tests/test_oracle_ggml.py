"""CPU tests of the oracle's ggml-faithful mode (oracle/dmoe_oracle_ggml.c, mode 2).

That mode restates what the reference's ggml CPU backend computes for the experts
(src/diffuse-moe-graph.cpp:265-270): weights stay in their GGUF blocks, each activation row is
rounded to the weight type's vec-dot type (Q8_K for Q4_K, Q8_0 for Q8_0, F16 for F16), and every
product is an integer block dot product scaled by the two block scales. It is the timed CPU
baseline and the estimate of what ggml would output. Pinned here:
  - Q8_0 activation rounding bit-for-bit against gguf-py's Q8_0 quantiser (golden vectors);
  - Q8_K and F16 rounding by their defining properties;
  - the AVX2 dot kernels against the scalar ones, and both against a float64 product of the
    dequantised weights and the rounded activations;
  - the layer output against the exact (float64) mode.
"""
import os

import numpy as np
import pytest

import diffuse_moe as dm
import oracle
import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "quant_golden.npz")


def test_q8_0_activation_rounding_matches_gguf_py():
    g = np.load(GOLDEN)
    x = g["q80_in"]
    r = oracle.ggml_round_act(dm.TYPE_Q8_0, x.ravel()).reshape(x.shape)
    assert np.array_equal(r.view(np.uint32), g["q80_deq"].view(np.uint32))


def test_q8_k_activation_rounding_rule():
    rng = np.random.default_rng(3)
    x = rng.standard_normal(4096).astype(np.float32)
    x[256:512] = 0.0                     # an all-zero block stays zero
    x[600] = -9.0                        # a negative extreme sets the scale's sign
    r = oracle.ggml_round_act(dm.TYPE_Q4_K, x)
    for b in range(16):
        xb, rb = x[256 * b:256 * (b + 1)], r[256 * b:256 * (b + 1)]
        if not np.any(xb):
            assert not np.any(rb)
            continue
        mx = xb[np.argmax(np.abs(xb))]
        d = 1.0 / np.float32(-127.0 / mx)
        q = rb / d
        assert np.allclose(q, np.round(q), atol=1e-3), "values are integer multiples of d"
        assert np.max(np.abs(q)) <= 127.0 + 1e-3
        assert np.isclose(rb[np.argmax(np.abs(xb))], mx, rtol=1e-6), "the extreme value is kept"
        assert np.max(np.abs(rb - xb)) <= abs(d) * 0.5 * (1 + 1e-5)


def test_f16_activation_rounding():
    x = np.random.default_rng(4).standard_normal(1024).astype(np.float32) * 10
    r = oracle.ggml_round_act(dm.TYPE_F16, x)
    assert np.array_equal(r, x.astype(np.float16).astype(np.float32))


@pytest.mark.parametrize("qtype,k", [(dm.TYPE_Q4_K, 4096), (dm.TYPE_Q4_K, 1024), (dm.TYPE_Q8_0, 2048),
                                     (dm.TYPE_F16, 512)])
def test_dot_kernels(qtype, k):
    rng = np.random.default_rng(k + qtype)
    wf = (rng.standard_normal((48, k)) * 0.02).astype(np.float32)
    if qtype == dm.TYPE_F16:
        wq = wf.astype(np.float16).view(np.uint8).reshape(48, -1)
    else:
        wq = dm.quantize(wf, qtype)
    x = rng.standard_normal(k).astype(np.float32)
    simd = oracle.ggml_dot(qtype, wq, k, x, simd=True)
    scal = oracle.ggml_dot(qtype, wq, k, x, simd=False)
    exact = oracle.dequant(qtype, wq, 48, k).astype(np.float64) @ oracle.ggml_round_act(qtype, x).astype(np.float64)
    scale = np.abs(exact).max()
    assert np.max(np.abs(simd - scal)) <= 2e-6 * scale
    assert np.max(np.abs(simd - exact)) <= 2e-6 * scale


@pytest.mark.parametrize("qtype,bound", [(dm.TYPE_F16, 1e-3), (dm.TYPE_Q8_0, 2e-2), (dm.TYPE_Q4_K, 2e-2)])
def test_layer_against_exact(qtype, bound):
    """ggml's activation rounding costs accuracy: about 1e-2 relative L2 for the 8-bit formats
    (more than the GPU path's fp16 activations), a few 1e-4 for F16."""
    spec = synth.LayerSpec(H=1024, I=512, Is=512, E=32, top_k=8, cap=12, blk=32, expert_type=qtype, seed=31)
    hp = spec.hparams()
    t = synth.make_layer(spec)
    x = synth.make_input(96, spec.H, spec.seed)
    exact, idx, w, _, _ = oracle.layer(hp, t, x, mode=oracle.MODE_EXACT)
    g = oracle.experts(hp, t, x, idx, w, mode=oracle.MODE_GGML)
    err = float(np.linalg.norm(g.astype(np.float64) - exact) / np.linalg.norm(exact.astype(np.float64)))
    assert err <= bound, err
    assert err > 0.0
