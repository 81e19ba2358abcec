"""dmoe_route_static: routing for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc, for instance a process whose device memory is owned by
another allocator (a serving stack that reserves its whole budget up front, or a framework that
hands out every buffer itself). dmoe_route_static serves them: they pass their own device
buffers, and the library's working memory is a fixed array inside the library. These tests
check, through the C ABI, that it returns the same routing as the existing entry point
(dmoe_forward with DMOE_F_ROUTE_ONLY): selected experts equal and gate weights bitwise equal,
the bar every routing test here uses, on two calls in a row (the shared array keeps the previous
call's contents), and that sizes beyond its stated limits are refused.

This file is collected last so that a run stopping at the first failure has run every other test.
"""
import numpy as np
import pytest

import diffuse_moe as dm
import synth


def _spec():
    return synth.LayerSpec(H=1024, I=256, Is=256, E=64, top_k=8, cap=12, blk=32, expert_type=dm.TYPE_Q8_0, seed=21)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [96, 50])  # block routing (96 % 32 == 0) and plain per-token top-k
def test_route_static_matches_forward(n):
    import torch

    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    spec = _spec()
    hp = spec.hparams()
    t = synth.make_layer(spec)
    layer = dm.MoELayer(hp, t)
    x = torch.from_numpy(synth.make_input(n, spec.H, spec.seed + n)).cuda()
    ref_idx, ref_w, _ = layer.forward(x, route_only=True)
    layer.sync()
    wr = torch.from_numpy(t["w_router"]).cuda()
    br = torch.from_numpy(t["b_router"]).cuda()
    for call in range(2):
        idx = torch.full((n, spec.top_k), -1, dtype=torch.int32, device="cuda")
        w = torch.full((n, spec.top_k), float("nan"), dtype=torch.float32, device="cuda")
        dm.route_static(x, wr, br, hp, idx, w)
        torch.cuda.synchronize()
        assert torch.equal(idx, ref_idx), f"call {call}: experts differ"
        assert torch.equal(w.view(torch.int32), ref_w.view(torch.int32)), f"call {call}: gate weights differ"
    layer.close()


def test_route_static_refuses_sizes_beyond_its_scratch():
    lib = dm.load()
    n = 4097  # DMOE_STATIC_MAX_TOKENS + 1: refused before any device work
    st = lib.dmoe_route_static(None, n, 1024, None, None, 64, 8, 12, 32, 2.5, 1, None, None, None)
    assert st == 2, dm.STATUS_NAMES.get(st)  # DMOE_ERR_UNSUPPORTED
    assert "exceed the fixed scratch limits" in dm.last_error()


def test_route_static_refuses_misaligned_pointers():
    """x is read with 16-byte copies and the bias as float4: a pointer off that alignment (a tensor
    view offset by one float) is refused with a status before any device work, not faulted on."""
    lib = dm.load()
    base = 1 << 20  # never dereferenced: the call returns before any device work
    args = dict(n=64, h=1024, e=64)
    for x, b in ((base + 4, base), (base, base + 8)):
        st = lib.dmoe_route_static(x, args["n"], args["h"], base, b, args["e"], 8, 12, 32, 2.5, 1, base, base, None)
        assert st == 1, dm.STATUS_NAMES.get(st)  # DMOE_ERR_INVALID_ARG
        assert "16-byte aligned" in dm.last_error()
    # a large moe_block_size is fine when block routing is off (n % block != 0): the routing kernel
    # then runs 32-token CTAs, so the shared-memory check must not refuse it (it gets as far as the
    # alignment check here)
    st = lib.dmoe_route_static(base + 4, 96, 1024, base, None, 256, 8, 48, 4096, 2.5, 1, base, base, None)
    assert st == 1 and "16-byte aligned" in dm.last_error(), dm.last_error()


def test_route_static_python_checks_tensors():
    """The Python binding refuses CPU, strided or wrongly typed tensors before calling the library."""
    import torch

    hp = _spec().hparams()
    x = torch.zeros((4, hp["n_embd"]), dtype=torch.float32)
    with pytest.raises(ValueError):
        dm.route_static(x, x, None, hp, x, x)
