"""The fused expert launch (GPU): gate/up and down GEMMs in one persistent kernel, where every
down tile waits for its token tile's h rows (per-token-tile counters). It is used at small N by
default; DMOE_FUSED=1 / 0 forces it on / off. Both must meet the oracle tolerance, and at a size
with many token tiles the two must agree (only the fp32 summation order differs).
"""
import os

import numpy as np
import pytest

import diffuse_moe as dm
import oracle
import synth
from test_gpu_parity import TOL, rel_l2, tiny


@pytest.fixture
def fused_env():
    old = os.environ.get("DMOE_FUSED")

    def set_(v):
        os.environ["DMOE_FUSED"] = str(v)

    yield set_
    if old is None:
        os.environ.pop("DMOE_FUSED", None)
    else:
        os.environ["DMOE_FUSED"] = old


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", [dm.TYPE_F16, dm.TYPE_Q8_0, dm.TYPE_Q4_K])
@pytest.mark.parametrize("Is", [256, 0])
def test_fused_and_split_match_oracle(qtype, Is, fused_env):
    spec = tiny(qtype, Is=Is)
    t = synth.make_layer(spec)
    x = synth.make_input(96, spec.H, spec.seed)
    ref = oracle.layer(spec.hparams(), t, x)[0]
    L = dm.MoELayer(spec.hparams(), t)
    for f in (1, 0):
        fused_env(f)
        out = L.forward(x, profile=True)
        L.sync()
        assert L.stats()["fused_gemm"] == f
        assert rel_l2(out, ref) <= TOL[qtype], (f, rel_l2(out, ref))
    L.close()


@pytest.mark.gpu
@pytest.mark.slow
def test_fused_agrees_with_split_many_tiles(fused_env):
    spec = synth.config("c2")  # S shape, q8_0, 2048 tokens: hundreds of token tiles
    L = dm.MoELayer(spec.hparams(), synth.make_layer(spec))
    x = synth.make_input(2048, spec.H, 9)
    fused_env(1)
    a = L.forward(x, profile=True)
    L.sync()
    assert L.stats()["fused_gemm"] == 1 and L.stats()["token_tile"] <= 64
    fused_env(0)
    b = L.forward(x)
    assert rel_l2(a, b) < 1e-5
    L.close()
