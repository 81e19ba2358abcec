"""CTA-pair expert GEMMs (GPU): clusters of two CTAs share each 256-row weight tile through
tcgen05 cta_group::2, each CTA dequantising 128 of the rows and loading half of the 128 token
rows. Quantised layers at a 128-token tile (DMOE_NT=128) use them for gate/up by default
(DMOE_PAIR=1); DMOE_PAIR=2 adds the down GEMM, 0 turns them off. Every setting must meet the
oracle tolerance, and on the same input they must agree to fp32 rounding.
"""
import os

import numpy as np
import pytest

import diffuse_moe as dm
import oracle
import synth
from test_gpu_parity import TOL, rel_l2, tiny


@pytest.fixture
def env():
    keys = ("DMOE_PAIR", "DMOE_NT")
    old = {k: os.environ.get(k) for k in keys}

    def set_(**kv):
        for k, v in kv.items():
            os.environ[k] = str(v)

    yield set_
    for k, v in old.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", [dm.TYPE_Q8_0, dm.TYPE_Q4_K])
@pytest.mark.parametrize("H,I,Is,n", [(256, 256, 256, 96), (512, 512, 0, 300), (512, 256, 512, 640)])
def test_pair_matches_oracle_and_single(qtype, H, I, Is, n, env):
    spec = tiny(qtype, H=H, I=I, Is=Is)
    t = synth.make_layer(spec)
    x = synth.make_input(n, spec.H, spec.seed)
    ref = oracle.layer(spec.hparams(), t, x)[0]
    L = dm.MoELayer(spec.hparams(), t)
    outs = {}
    for pair in (2, 1, 0):
        env(DMOE_PAIR=pair, DMOE_NT=128)
        out = L.forward(x)
        L.sync()
        assert L.stats()["token_tile"] == 128
        assert rel_l2(out, ref) <= TOL[qtype], (pair, rel_l2(out, ref))
        outs[pair] = out
    assert rel_l2(outs[1], outs[0]) < 1e-5 and rel_l2(outs[2], outs[0]) < 1e-5
    L.close()


@pytest.mark.gpu
@pytest.mark.slow
def test_pair_flash_shape_many_tiles(env):
    """c3's shape (hidden 4096, 256 experts of 1024, q4_K) at 64 blocks: 16 output tiles per
    expert matrix, hundreds of token tiles spread over every pair of the grid."""
    spec = synth.config("c3")
    L = dm.MoELayer(spec.hparams(), synth.make_layer(spec))
    x = synth.make_input(2048, spec.H, 5)
    env(DMOE_PAIR=0, DMOE_NT=128)
    a = L.forward(x)
    for pair in (1, 2):
        env(DMOE_PAIR=pair, DMOE_NT=128)
        b = L.forward(x)
        L.sync()
        assert np.isfinite(b).all()
        assert rel_l2(b, a) < 1e-5, pair
    L.close()
