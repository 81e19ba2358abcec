"""The full LLaDA2-MoE forward and block-diffusion loop (diffuse-cpp_b200/llada2.py) on the GPU.

A tiny model (3 blocks, the first dense, two MoE layers through the C ABI; F16 experts) in fp32:
  - one forward over a 2-block window against the float64 restatement of
    diffuse_build_graph_moe (oracle/llada2_ref.py): relative L2 of the logits <= 3e-3;
  - the key/value-cached forward of a block equals the whole-window forward the reference runs
    at every step (relative L2 <= 1e-5);
  - generation with the cache commits the same tokens as generation that recomputes the window
    at every step, and so does the cache with each step replayed from a CUDA graph.
"""
import numpy as np
import pytest
import torch

import diffuse_moe as dm
import llada2
import llada2_ref
import synth


@pytest.fixture(autouse=True)
def _need_gpu():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


def tiny_model(dtype=torch.float32):
    cfg = llada2.LLaDA2Config(n_layer=3, n_embd=256, n_head=4, n_head_kv=2, head_dim=64, rotary_dim=32, n_ff=512,
                              first_k_dense=1, n_vocab=1000, rope_base=10000.0, mask_token_id=999)
    w = llada2.LLaDA2Model.random_weights(cfg, seed=5)
    w["output"][cfg.mask_token_id] = 0.0  # the mask token is never the argmax (its logit is 0)
    moe, specs = {}, {}
    for il in range(cfg.first_k_dense, cfg.n_layer):
        sp = synth.LayerSpec(H=256, I=256, Is=256, E=16, top_k=4, cap=6, blk=32, expert_type=dm.TYPE_F16,
                             seed=60 + il)
        t = synth.make_layer(sp)
        moe[il] = dm.MoELayer(sp.hparams(), t)
        specs[il] = (sp.hparams(), t)
    return cfg, w, llada2.LLaDA2Model(cfg, w, moe, dtype=dtype), specs


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.gpu
def test_forward_matches_restatement():
    torch.backends.cuda.matmul.allow_tf32 = False
    cfg, w, model, specs = tiny_model()
    tokens = np.random.default_rng(1).integers(0, cfg.n_vocab - 1, size=64)
    got = model.forward(torch.as_tensor(tokens, device="cuda"), 0).cpu().numpy()
    wn = {k: v.float().cpu().numpy() for k, v in w.items()}
    ref = llada2_ref.forward(cfg, wn, specs, tokens)
    assert rel(got, ref) <= 3e-3, rel(got, ref)


@pytest.mark.gpu
def test_cached_block_equals_window():
    torch.backends.cuda.matmul.allow_tf32 = False
    cfg, w, model, _ = tiny_model()
    tokens = torch.as_tensor(np.random.default_rng(2).integers(0, cfg.n_vocab - 1, size=96), device="cuda")
    full = model.forward(tokens, 0)[64:]
    cache = model.new_cache(96)
    model.forward(tokens[:64], 0, cache, commit=64)
    assert cache["len"] == 64
    part = model.forward(tokens[64:], 64, cache)
    assert rel(part.cpu().numpy(), full.cpu().numpy()) <= 1e-5


@pytest.mark.gpu
def test_generation_with_cache_equals_recompute():
    torch.backends.cuda.matmul.allow_tf32 = False
    cfg, w, model, _ = tiny_model()
    prompt = np.random.default_rng(3).integers(0, cfg.n_vocab - 1, size=70)  # ends inside a block
    seq_c, nf_c = llada2.generate(model, prompt, 60, steps=8, threshold=0.95, use_cache=True)
    seq_r, nf_r = llada2.generate(model, prompt, 60, steps=8, threshold=0.95, use_cache=False)
    seq_g, nf_g = llada2.generate(model, prompt, 60, steps=8, threshold=0.95, use_cache=True, graphs=True)
    assert np.array_equal(seq_c, seq_r)
    assert np.array_equal(seq_g, seq_c) and nf_g == nf_c  # CUDA-graph replay of the same steps
    assert not np.any(seq_c == cfg.mask_token_id)  # every position committed
    assert np.array_equal(seq_c[:70], prompt)
    # 3 blocks of 26, 32, 32 masked positions, 4+ commits per step: at most 7 + 8 + 8 forwards;
    # the cached run adds one prefill of the prompt's first block
    assert 3 <= nf_r <= 23 and nf_c == nf_r + 1, (nf_c, nf_r)
