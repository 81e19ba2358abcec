"""The oracle's expert FFN (src/diffuse-moe-graph.cpp:264-286) against a numpy float64 restatement
on tiny shapes, for every weight type, with and without the shared expert (CPU)."""
import numpy as np
import pytest

import diffuse_moe as dm
import oracle
import synth


def ffn_ref(hp, t, x, idx, w):
    H, I, Is, E, K = hp["n_embd"], hp["n_ff_exp"], hp["n_ff_shexp"], hp["n_expert"], hp["n_expert_used"]
    et, st = hp["expert_type"], hp["shared_type"]
    Wg = oracle.dequant(et, t["w_gate"], E * I, H).astype(np.float64).reshape(E, I, H)
    Wu = oracle.dequant(et, t["w_up"], E * I, H).astype(np.float64).reshape(E, I, H)
    Wd = oracle.dequant(et, t["w_down"], E * H, I).astype(np.float64).reshape(E, H, I)
    x64 = x.astype(np.float64)
    out = np.zeros((x.shape[0], H))
    for n in range(x.shape[0]):
        for s in range(K):
            e = idx[n, s]
            g = Wg[e] @ x64[n]
            u = Wu[e] @ x64[n]
            out[n] += (Wd[e] @ (g / (1 + np.exp(-g)) * u)) * float(w[n, s])
    if Is > 0:
        Sg = oracle.dequant(st, t["sw_gate"], Is, H).astype(np.float64)
        Su = oracle.dequant(st, t["sw_up"], Is, H).astype(np.float64)
        Sd = oracle.dequant(st, t["sw_down"], H, Is).astype(np.float64)
        g = x64 @ Sg.T
        u = x64 @ Su.T
        out += (g / (1 + np.exp(-g)) * u) @ Sd.T
    return out


@pytest.mark.parametrize("qtype", [dm.TYPE_F16, dm.TYPE_Q8_0, dm.TYPE_Q4_K])
@pytest.mark.parametrize("Is", [256, 0])
def test_experts_match_float64(qtype, Is):
    spec = synth.LayerSpec(H=256, I=256, Is=Is, E=8, top_k=3, cap=4, blk=32, expert_type=qtype, seed=13)
    hp = spec.hparams()
    t = synth.make_layer(spec)
    x = synth.make_input(40, spec.H, 13)
    out, idx, w, _, _ = oracle.layer(hp, t, x, mode=0)
    ref = ffn_ref(hp, t, x, idx, w)
    assert np.max(np.abs(out - ref)) <= 1e-5 * np.max(np.abs(ref))
    out1 = oracle.experts(hp, t, x, idx, w, mode=1)  # the float-accumulation CPU baseline
    assert np.linalg.norm(out1 - ref) / np.linalg.norm(ref) < 1e-5
