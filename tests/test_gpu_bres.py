"""Down GEMM with resident activation tiles (moe_gemm_kernel BRES variant) against the oracle.

The variant keeps one 64-token tile of the SwiGLU output in shared memory and runs every 256-row
m-tile of the down matrix against it; the CTA walks whole units (group, token tile, m-chunk).
It is off by default (measured slower: the down GEMM is bound by its dequant issue rate, not by
L2); these tests force it (and its unit chunking, and 128-row list tiles taken as two halves) on
small layers, check the oracle bar, and check that in the deterministic mode (every output row
stored once) it gives the same bits as the per-m-tile launch at the same token tile.
"""
import numpy as np
import pytest

import diffuse_moe as dm
import oracle
import synth

TOL = 2e-3


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b.astype(np.float64)) / np.linalg.norm(b.astype(np.float64)))


@pytest.fixture(autouse=True)
def _need_gpu():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


def small(qtype, **kw):
    base = dict(H=1024, I=512, Is=512, E=16, top_k=4, cap=6, blk=32, expert_type=qtype, seed=41)
    base.update(kw)
    return synth.LayerSpec(**base)


def run(spec, n, monkeypatch, env, deterministic=False):
    for k, v in env.items():
        monkeypatch.setenv(k, str(v))
    t = synth.make_layer(spec)
    x = synth.make_input(n, spec.H, spec.seed)
    L = dm.MoELayer(spec.hparams(), t)
    try:
        out = L.forward(x, deterministic=deterministic)
        L.forward(x, profile=True)
        L.sync()
        st = L.stats()
    finally:
        L.close()
    return out, st, t, x


# (token tile, env): pair variant (DMOE_BRES=1, NT = 128) with 1 / 2 / 4 m-chunks per unit;
# single-CTA variant (DMOE_BRES=2) on 64-token tiles, and on 128-row list tiles taken as halves
CASES = [
    (128, dict(DMOE_BRES=1, DMOE_BRES_CHUNKS=1)),
    (128, dict(DMOE_BRES=1, DMOE_BRES_CHUNKS=2)),
    (128, dict(DMOE_BRES=1, DMOE_BRES_CHUNKS=4)),
    (64, dict(DMOE_BRES=2, DMOE_BRES_CHUNKS=1)),
    (64, dict(DMOE_BRES=2, DMOE_BRES_CHUNKS=4)),
    (128, dict(DMOE_BRES=2, DMOE_PAIR=0)),
]


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", [dm.TYPE_Q4_K, dm.TYPE_Q8_0])
@pytest.mark.parametrize("nt,env", CASES)
def test_bres_against_oracle(qtype, nt, env, monkeypatch):
    spec = small(qtype)
    out, st, t, x = run(spec, 320, monkeypatch, dict(env, DMOE_NT=nt, DMOE_FUSED=0))
    assert st["token_tile"] == nt and st["fused_gemm"] == 0
    r_out, *_ = oracle.layer(spec.hparams(), t, x)
    err = rel_l2(out, r_out)
    assert err <= TOL, err


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", [dm.TYPE_Q4_K, dm.TYPE_Q8_0])
@pytest.mark.parametrize("nt,env", [(128, dict(DMOE_BRES=1)), (64, dict(DMOE_BRES=2))])
def test_bres_shared_expert_of_another_width(qtype, nt, env, monkeypatch):
    """The shared group's K (its width I_s) differs from the routed experts': each unit loads its
    own group's K of activations."""
    spec = small(qtype, Is=256, I=1024)
    out, _, t, x = run(spec, 192, monkeypatch, dict(env, DMOE_NT=nt, DMOE_FUSED=0))
    r_out, *_ = oracle.layer(spec.hparams(), t, x)
    assert rel_l2(out, r_out) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", [dm.TYPE_Q4_K, dm.TYPE_Q8_0])
@pytest.mark.parametrize("nt,on,off", [(128, dict(DMOE_PAIR=2, DMOE_BRES=1), dict(DMOE_PAIR=2, DMOE_BRES=0)),
                                       (64, dict(DMOE_BRES=2), dict(DMOE_BRES=0))])
def test_bres_bitwise_equal_to_per_mtile_launch(qtype, nt, on, off, monkeypatch):
    """Deterministic mode (every output row stored once): the same MMAs over the same K order as
    the launch that reloads the activation tile per m-tile (pairs at NT = 128, single CTAs at
    NT = 64), so the outputs are bit for bit the same."""
    spec = small(qtype)
    env = dict(DMOE_NT=nt, DMOE_FUSED=0)
    a, *_ = run(spec, 256, monkeypatch, dict(env, **on), deterministic=True)
    for k in on:
        monkeypatch.delenv(k, raising=False)
    b, *_ = run(spec, 256, monkeypatch, dict(env, **off), deterministic=True)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
