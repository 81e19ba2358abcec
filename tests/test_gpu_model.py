"""Whole-model upload from GGUF on the GPU (dmoe_model_load through the C ABI).

A small LLaDA2-MoE file (gguf-py writer, the reference converter's names) is loaded once; every
MoE block's layer must give the oracle's routing bit for bit and its output within the oracle
bar, and its output must equal, bit for bit, that of a layer bound directly from the same
tensors (deterministic slot-order sum): the upload changes nothing. Dense blocks have no layer.
"""
import numpy as np
import pytest

import diffuse_moe as dm
import oracle
import synth
from model_gguf import ModelSpec, write_model

TOL = {dm.TYPE_F16: 1e-3, dm.TYPE_Q8_0: 2e-3, dm.TYPE_Q4_K: 2e-3}


@pytest.fixture(autouse=True)
def _need_gpu():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


@pytest.mark.gpu
@pytest.mark.parametrize("qtype,stype", [(dm.TYPE_Q4_K, None), (dm.TYPE_Q8_0, dm.TYPE_F16)])
def test_model_layers_match_oracle_and_direct_binding(tmp_path, qtype, stype):
    ms = ModelSpec(n_layer=4, first_k=1, expert_type=qtype, shared_type=stype)
    path = str(tmp_path / "m.gguf")
    layers = write_model(path, ms)
    model = dm.MoEModel(path)
    assert model.info["n_moe_layers"] == 3 and model.layer(0) is None and model.layer(4) is None
    x = synth.make_input(96, ms.H, 77)
    for il, t in layers.items():
        hp = ms.layer_spec(il).hparams()
        L = model.layer(il)
        out, (idx, w, _) = L.forward(x, route=True, deterministic=True)
        r_out, r_idx, r_w, _, _ = oracle.layer(hp, t, x)
        assert np.array_equal(idx, r_idx) and np.array_equal(w.view(np.uint32), r_w.view(np.uint32)), il
        err = float(np.linalg.norm(out.astype(np.float64) - r_out) / np.linalg.norm(r_out))
        assert err <= max(TOL[qtype], TOL[stype or qtype]), (il, err)
        D = dm.MoELayer(hp, t)
        d_out = D.forward(x, deterministic=True)
        D.close()
        assert np.array_equal(out.view(np.uint32), d_out.view(np.uint32)), f"block {il}: model layer differs"
    model.close()
