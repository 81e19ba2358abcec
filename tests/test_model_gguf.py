"""CPU tests of the GGUF model loader's reader and checks (dmoe_model_inspect: no device).

Files are written with gguf-py's GGUFWriter and the reference converter's names
(tools/convert-llada2-fast.py); the loader follows diffuse_model_load_impl
(src/diffuse-model.cpp:67-224). The device side (dmoe_model_load) is tested in
test_gpu_model.py.
"""
import os

import numpy as np
import pytest

import diffuse_moe as dm
from model_gguf import ModelSpec, write_model


def moe_bytes(layers: dict) -> int:
    n = 0
    for t in layers.values():
        for k in ("w_router", "b_router", "w_gate", "w_up", "w_down", "sw_gate", "sw_up", "sw_down"):
            if t.get(k) is not None:
                n += t[k].nbytes
    return n


@pytest.mark.parametrize("qtype,stype", [(dm.TYPE_Q4_K, None), (dm.TYPE_Q8_0, dm.TYPE_F16), (dm.TYPE_F16, None)])
def test_inspect_reads_hparams_and_tensors(tmp_path, qtype, stype):
    ms = ModelSpec(n_layer=4, first_k=1, expert_type=qtype, shared_type=stype)
    path = str(tmp_path / "m.gguf")
    layers = write_model(path, ms)
    info = dm.model_inspect(path)
    assert info["n_layer"] == 4 and info["first_k_dense"] == 1 and info["n_moe_layers"] == 3
    assert (info["n_embd"], info["n_ff_exp"], info["n_ff_shexp"], info["n_expert"]) == (ms.H, ms.I, ms.Is, ms.E)
    assert (info["n_expert_used"], info["expert_capacity"], info["moe_block_size"]) == (ms.top_k, ms.cap, ms.blk)
    assert info["routed_scaling"] == pytest.approx(ms.scale) and info["norm_topk_prob"] == 1
    assert info["expert_type"] == qtype and info["shared_type"] == (qtype if stype is None else stype)
    assert info["moe_bytes"] == moe_bytes(layers)


def test_defaults_and_no_shared_expert(tmp_path):
    """Keys the reference defaults (expert_capacity 48, moe_block_size from block_length,
    routed_scaling 1) and a model without shared experts."""
    ms = ModelSpec(n_layer=2, first_k=0, Is=0, blk=16)
    path = str(tmp_path / "m.gguf")
    write_model(path, ms, omit=("expert_capacity", "moe_block_size", "routed_scaling_factor"))
    info = dm.model_inspect(path)
    assert info["n_ff_shexp"] == 0 and info["n_moe_layers"] == 2 and info["first_k_dense"] == 0
    assert info["expert_capacity"] == 48 and info["moe_block_size"] == 16 and info["routed_scaling"] == 1.0
    path = str(tmp_path / "m2.gguf")
    write_model(path, ms, omit=("moe_block_size", "block_length"))
    assert dm.model_inspect(path)["moe_block_size"] == 32


def test_custom_alignment(tmp_path):
    path = str(tmp_path / "m.gguf")
    layers = write_model(path, ModelSpec(n_layer=2), alignment=64)
    assert dm.model_inspect(path)["moe_bytes"] == moe_bytes(layers)


def expect_error(path, status, text):
    with pytest.raises(dm.DmoeError) as e:
        dm.model_inspect(path)
    assert e.value.status == status, str(e.value)
    assert text in str(e.value), str(e.value)


def test_missing_and_malformed_tensors(tmp_path):
    ms = ModelSpec(n_layer=3)
    p = str(tmp_path / "a.gguf")
    write_model(p, ms, drop=("blk.2.moe_experts_down.weight",))
    expect_error(p, 1, "tensor not found: blk.2.moe_experts_down.weight")
    p = str(tmp_path / "b.gguf")
    bad = np.zeros((ms.E, ms.H + 32), np.float32)
    write_model(p, ms, override={"blk.1.moe_gate.weight": (bad, None)})
    expect_error(p, 1, "blk.1.moe_gate.weight: ne [288, 16], expected [256, 16]")
    p = str(tmp_path / "c.gguf")
    write_model(p, ms, override={"blk.1.moe_gate.weight": (np.zeros((ms.E, ms.H), np.float16), None)})
    expect_error(p, 2, "must be F32")
    p = str(tmp_path / "d.gguf")  # F32 expert stacks (the converter's --type f32) are not a kernel format
    f32 = np.zeros((ms.E, ms.I, ms.H), np.float32)
    write_model(p, ms, override={"blk.1.moe_experts_gate.weight": (f32, None),
                                 "blk.1.moe_experts_up.weight": (f32, None),
                                 "blk.1.moe_experts_down.weight": (np.zeros((ms.E, ms.H, ms.I), np.float32), None)})
    expect_error(p, 2, "expert stacks of ggml types 0 / 0 / 0")


def test_model_type_and_keys(tmp_path):
    ms = ModelSpec(n_layer=2)
    p = str(tmp_path / "dream.gguf")
    write_model(p, ms, model_type="dream")
    expect_error(p, 2, "model type dream has no MoE layers")
    p = str(tmp_path / "nokey.gguf")  # no diffuse.model_type: architecture "diffuse" means llada2_moe
    write_model(p, ms, model_type=None)
    assert dm.model_inspect(p)["n_moe_layers"] == 1
    p = str(tmp_path / "nodense.gguf")
    write_model(p, ms, keys={"first_k_dense_replace": 5})
    expect_error(p, 1, "first_k_dense_replace 5 > block_count 2")


def test_corrupt_files(tmp_path):
    p = str(tmp_path / "m.gguf")
    write_model(p, ModelSpec(n_layer=2))
    data = open(p, "rb").read()
    q = str(tmp_path / "magic.gguf")
    open(q, "wb").write(b"GGUX" + data[4:])
    expect_error(q, 1, "bad magic")
    q = str(tmp_path / "short.gguf")
    open(q, "wb").write(data[: len(data) // 2])  # tensor data cut off
    expect_error(q, 1, "past the end of the file")
    q = str(tmp_path / "hdr.gguf")
    open(q, "wb").write(data[:1000])  # header cut off among the tensor infos
    expect_error(q, 1, "truncated")
    q = str(tmp_path / "tiny.gguf")
    open(q, "wb").write(data[:200])  # counts that cannot fit in the file
    expect_error(q, 1, "implausible")
    expect_error(str(tmp_path / "none.gguf"), 1, "cannot open")
    assert not os.path.exists(str(tmp_path / "none.gguf"))


def test_implausible_block_count(tmp_path):
    """A block count the file's tensors cannot hold is refused before any table is sized from it."""
    p = str(tmp_path / "m.gguf")
    write_model(p, ModelSpec(n_layer=2), keys={"block_count": 4000000})
    expect_error(p, 1, "block_count 4000000 with")


def test_real_file_metadata(tmp_path):
    """A file carrying what the reference converter writes besides the layers
    (tools/convert-llada2-fast.py:144-173): string, bool, string-array and int-array keys (the
    tokenizer's token list, types and merges), plus u64 / f64 / i32 keys; the reader skips them."""
    p = str(tmp_path / "m.gguf")

    def tokenizer(w):
        w.add_string("tokenizer.ggml.model", "gpt2")
        w.add_token_list([f"tok{i}" for i in range(3000)] + ["", "éè", "x" * 300])
        w.add_token_types([1] * 3003)
        w.add_token_merges(["a b", "c d"])
        w.add_bool("tokenizer.ggml.add_bos_token", False)
        w.add_uint64("diffuse.some_u64", 1 << 40)
        w.add_float64("diffuse.some_f64", 0.5)
        w.add_int32("diffuse.some_i32", -7)
        w.add_string("tokenizer.chat_template", "{{ messages }}")

    layers = write_model(p, ModelSpec(n_layer=2), extra=tokenizer)
    info = dm.model_inspect(p)
    assert info["n_moe_layers"] == 1 and info["moe_bytes"] == moe_bytes(layers)
