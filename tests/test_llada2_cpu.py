"""CPU checks of the full-model host code (diffuse-cpp_b200/llada2.py) that needs no GPU: RMSNorm,
partial NeoX RoPE and the transfer schedule against the float64 restatement and the reference's
formula (src/diffuse-sampler.cpp:16-25)."""
import numpy as np
import torch

import llada2
import llada2_ref


def test_rms_norm_and_rope_match_restatement():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 3, 64)).astype(np.float32)
    w = rng.standard_normal(64).astype(np.float32)
    got = llada2.rms_norm(torch.from_numpy(x), torch.from_numpy(w), 1e-6).numpy()
    assert np.allclose(got, llada2_ref.rms_norm(x, w, 1e-6), rtol=1e-5, atol=1e-6)
    pos = np.array([0, 1, 7, 100, 4095])
    got = llada2.rope_neox(torch.from_numpy(x), torch.from_numpy(pos), 32, 10000.0).numpy()
    ref = llada2_ref.rope_neox(x.astype(np.float64), pos, 32, 10000.0)
    assert np.allclose(got, ref, rtol=1e-4, atol=1e-4)
    assert np.array_equal(got[..., 32:], x[..., 32:])  # dims past rotary_dim pass through
    assert np.allclose(got[0], x[0])  # position 0 is the identity


def test_transfer_schedule():
    assert llada2.transfer_schedule(32, 8) == [4] * 8
    assert llada2.transfer_schedule(32, 5) == [7, 7, 6, 6, 6]
    assert llada2.transfer_schedule(32, 32) == [1] * 32
    assert llada2.transfer_schedule(32, 0) == []
    for L, s in ((32, 3), (32, 7), (30, 4)):
        assert sum(llada2.transfer_schedule(L, s)) == L
