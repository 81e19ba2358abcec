"""CUDA path vs the CPU oracle on the same seeded inputs (through the C ABI).

Bar: routing bit-exact (selected experts in slot order, applied gate weights bitwise, the
per-block capacity mask); layer output relative L2 error <= 1e-3 for F16 weights and
<= 2e-3 for Q8_0 / Q4_K weights, against the oracle's double-accumulation answer.
"""
import numpy as np
import pytest

import diffuse_moe as dm
import oracle
import synth

TOL = {dm.TYPE_F16: 1e-3, dm.TYPE_Q8_0: 2e-3, dm.TYPE_Q4_K: 2e-3}


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b.astype(np.float64)) / np.linalg.norm(b.astype(np.float64)))


def check_layer(spec: synth.LayerSpec, n: int, t=None, x=None, layer=None):
    hp = spec.hparams()
    t = synth.make_layer(spec) if t is None else t
    x = synth.make_input(n, spec.H, spec.seed) if x is None else x
    L = dm.MoELayer(hp, t) if layer is None else layer
    out, (idx, w, allowed) = L.forward(x, route=True)
    r_out, r_idx, r_w, r_allowed, used = oracle.layer(hp, t, x)
    assert np.array_equal(idx, r_idx), f"routing differs at {np.argwhere(idx != r_idx)[:5]}"
    assert np.array_equal(w.view(np.uint32), r_w.view(np.uint32)), "gate weights differ"
    if used:
        assert np.array_equal(allowed[: n // spec.blk], r_allowed), "capacity mask differs"
    err = rel_l2(out, r_out)
    tol = max(TOL[spec.expert_type], TOL[spec.stype])
    assert err <= tol, f"rel L2 {err:.3e} > {tol:.1e}"
    return err, L


def tiny(qtype, **kw):
    base = dict(H=256, I=256, Is=256, E=16, top_k=4, cap=6, blk=32, expert_type=qtype, seed=11)
    base.update(kw)
    return synth.LayerSpec(**base)


@pytest.fixture(autouse=True)
def _need_gpu():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", [dm.TYPE_F16, dm.TYPE_Q8_0, dm.TYPE_Q4_K])
@pytest.mark.parametrize("n", [32, 64, 50, 1])
def test_tiny_layer(qtype, n):
    check_layer(tiny(qtype), n)


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", [dm.TYPE_Q8_0, dm.TYPE_Q4_K])
def test_tiny_variants(qtype):
    check_layer(tiny(qtype, Is=0), 64)                         # no shared expert
    check_layer(tiny(qtype, bias="none"), 64)                  # no expert bias
    check_layer(tiny(qtype, norm_topk=0, scale=1.0), 64)      # no renormalisation / scaling
    check_layer(tiny(qtype, shared_type=dm.TYPE_F16), 96)     # shared expert in another type
    check_layer(tiny(qtype, I=512, Is=256, E=32, top_k=8, cap=12), 128)


@pytest.mark.gpu
def test_c1_f16_one_block():
    err, _ = check_layer(synth.config("c1"), 32)
    print("c1 rel L2", err)


@pytest.mark.gpu
@pytest.mark.slow
def test_c2_q8_0_64_blocks():
    err, _ = check_layer(synth.config("c2"), 2048)
    print("c2 rel L2", err)


@pytest.mark.gpu
@pytest.mark.slow
def test_c3_q4k_1_and_8_blocks():
    spec = synth.config("c3")
    t = synth.make_layer(spec)
    L = dm.MoELayer(spec.hparams(), t)
    for n in (32, 256):
        err, _ = check_layer(spec, n, t=t, layer=L)
        print("c3", n, "rel L2", err)


@pytest.mark.gpu
@pytest.mark.parametrize("plan", [0, 1, 2, 3])
@pytest.mark.parametrize("E", [64, 160, 320])
def test_router_plans_bit_exact(plan, E, monkeypatch):
    """Each router logits plan (whole-K 128- or 112-token tiles of 128 experts; per-segment
    partials of 32- or 128-token tiles of 64 experts summed in segment order) gives the oracle's
    routing bit for bit, on a ragged last token tile; E = 64 leaves the upper half of a 128-expert
    tile empty, E = 160 fills the second tile a quarter; E = 320 takes the routing kernel's
    shared-memory top-k (more than 8 candidates per lane)."""
    monkeypatch.setenv("DMOE_ROUTER_SPLIT", str(plan))
    spec = tiny(dm.TYPE_Q8_0, H=1024, E=E, top_k=6, cap=20, seed=23)
    check_layer(spec, 608)  # 19 routing blocks: the last 128-token tile holds 96 tokens


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", [dm.TYPE_Q8_0, dm.TYPE_Q4_K])
def test_forced_split_k(qtype, monkeypatch):
    """Split-K (off by default, forced with DMOE_KSPLIT_GU / DMOE_KSPLIT_DN): gate/up partial sums
    in fp32 then the SwiGLU kernel, down partials reduced into the output; same oracle bar."""
    monkeypatch.setenv("DMOE_KSPLIT_GU", "2")
    monkeypatch.setenv("DMOE_KSPLIT_DN", "2")
    spec = tiny(qtype, H=1024, I=512, Is=512, E=16, seed=29)
    t = synth.make_layer(spec)
    L = dm.MoELayer(spec.hparams(), t)
    check_layer(spec, 96, t=t, layer=L)
    L.forward(synth.make_input(96, spec.H, spec.seed), profile=True)
    L.sync()
    assert L.stats()["ksplit_gateup"] == 2 and L.stats()["ksplit_down"] == 2
    L.close()
