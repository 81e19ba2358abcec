"""The C ABI library (no GPU needed): it loads, exports every entry point include/*.h declares,
and rejects bad arguments with status codes (never an exit, never a CPU fallback)."""
import ctypes
import glob
import os
import re

import numpy as np
import pytest

import diffuse_moe as dm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(dmoe_[a-z_0-9]+)\s*\(", src):
            names.add(m.group(1))
    return sorted(names)


def test_every_declared_symbol_is_exported():
    lib = dm.load()
    names = declared_functions()
    assert "dmoe_forward" in names and "dmoe_create" in names
    for n in names:
        assert hasattr(lib, n), n


def test_abi_version():
    assert dm.load().dmoe_abi_version() == 5


def test_model_and_split_argument_errors(tmp_path):
    """dmoe_model_load / dmoe_create_split refuse null arguments and unreadable files with status
    codes; the model accessors tolerate a null model."""
    lib = dm.load()
    h = ctypes.c_void_p()
    assert lib.dmoe_model_load(None, None, ctypes.byref(h)) == 1
    assert lib.dmoe_model_load(os.fsencode(str(tmp_path / "missing.gguf")), None, ctypes.byref(h)) == 1
    assert "cannot open" in dm.last_error() and not h.value
    assert lib.dmoe_model_load(b"x", None, None) == 1
    assert lib.dmoe_model_get_info(None, None) == 1
    assert lib.dmoe_model_layer(None, 0) is None
    lib.dmoe_model_free(None)
    d = dm.LayerDesc()
    assert lib.dmoe_create_split(ctypes.byref(d), None, None, ctypes.byref(h)) == 1
    assert "null parent" in dm.last_error()
    # a valid descriptor but no expert-parallel config: refused before the parent is touched
    import synth

    sp = synth.LayerSpec(H=256, I=256, Is=256, E=16, top_k=4, cap=6, blk=32, expert_type=dm.TYPE_Q8_0, seed=1)
    t = synth.make_layer(sp)
    keep = {k: np.ascontiguousarray(v) for k, v in t.items() if v is not None}
    d = dm.LayerDesc(n_embd=256, n_ff_exp=256, n_ff_shexp=256, n_expert=16, n_expert_used=4, expert_capacity=6,
                     moe_block_size=32, routed_scaling=2.5, norm_topk_prob=1, expert_type=dm.TYPE_Q8_0,
                     shared_type=dm.TYPE_Q8_0)
    for k, v in keep.items():
        setattr(d, k, v.ctypes.data)
    assert lib.dmoe_create_split(ctypes.byref(d), None, ctypes.c_void_p(8), ctypes.byref(h)) == 1
    assert "needs an expert-parallel dist" in dm.last_error()


def test_replicate_experts_argument_errors():
    """dmoe_replicate_experts refuses a null layer and an n_hot outside [0, DMOE_MAX_HOT] before
    any device or NCCL work."""
    lib = dm.load()
    assert lib.dmoe_replicate_experts(None, None, 4) == 1  # DMOE_ERR_INVALID_ARG
    assert "null layer" in dm.last_error()


def test_argument_errors_are_status_codes():
    lib = dm.load()
    h = ctypes.c_void_p()
    assert lib.dmoe_create(None, None, ctypes.byref(h)) == 1  # DMOE_ERR_INVALID_ARG
    assert "null layer descriptor" in dm.last_error()
    d = dm.LayerDesc()
    d.n_embd, d.n_ff_exp, d.n_expert, d.n_expert_used = 256, 256, 16, 32  # top-k > 16
    assert lib.dmoe_create(ctypes.byref(d), None, ctypes.byref(h)) == 1
    assert lib.dmoe_forward(None, None, 0, None, None, None, 0) == 1
    assert lib.dmoe_sync(None) == 1


def test_no_device_is_reported_not_worked_around():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    import numpy as np
    import synth

    spec = synth.config("tiny")
    with pytest.raises(dm.DmoeError) as ei:
        dm.MoELayer(spec.hparams(), synth.make_layer(spec))
    assert ei.value.status == 3  # DMOE_ERR_NO_DEVICE


def test_sample_step_argument_errors():
    """dmoe_sample_step validates its arguments before touching the device."""
    lib = dm.load()
    assert lib.dmoe_sample_step(None, 4, 0, None, 0, 1, 0.5, None, None, None, None) == 1  # n_vocab <= 0
    assert "n_vocab" in dm.last_error()
    assert lib.dmoe_sample_step(None, 2000, 100, None, 0, 1, 0.5, None, None, None, None) == 2  # > max positions
    assert lib.dmoe_sample_step(None, 4, 100, None, 0, 1, 0.5, None, None, None, None) == 1  # null logits
    assert "null pointer" in dm.last_error()
    assert lib.dmoe_sample_step(None, 0, 100, None, 0, 1, 0.5, None, None, None, None) == 0  # nothing to do
