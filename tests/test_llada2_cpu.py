"""CPU checks of the full-model host code (diffuse-cpp_b200/llada2.py) that needs no GPU: RMSNorm,
partial NeoX RoPE and the transfer schedule against the float64 restatement and the reference's
formula (src/diffuse-sampler.cpp:16-25)."""
import numpy as np
import torch

import llada2
import llada2_ref


def test_rms_norm_and_rope_match_restatement():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 3, 64)).astype(np.float32)
    w = rng.standard_normal(64).astype(np.float32)
    got = llada2.rms_norm(torch.from_numpy(x), torch.from_numpy(w), 1e-6).numpy()
    assert np.allclose(got, llada2_ref.rms_norm(x, w, 1e-6), rtol=1e-5, atol=1e-6)
    pos = np.array([0, 1, 7, 100, 4095])
    got = llada2.rope_neox(torch.from_numpy(x), torch.from_numpy(pos), 32, 10000.0).numpy()
    ref = llada2_ref.rope_neox(x.astype(np.float64), pos, 32, 10000.0)
    assert np.allclose(got, ref, rtol=1e-4, atol=1e-4)
    assert np.array_equal(got[..., 32:], x[..., 32:])  # dims past rotary_dim pass through
    assert np.allclose(got[0], x[0])  # position 0 is the identity


def test_transfer_schedule():
    assert llada2.transfer_schedule(32, 8) == [4] * 8
    assert llada2.transfer_schedule(32, 5) == [7, 7, 6, 6, 6]
    assert llada2.transfer_schedule(32, 32) == [1] * 32
    assert llada2.transfer_schedule(32, 0) == []
    for L, s in ((32, 3), (32, 7), (30, 4)):
        assert sum(llada2.transfer_schedule(L, s)) == L


class OracleMoE:
    """Stand-in for a diffuse_moe.MoELayer on the CPU: the layer oracle (float64 accumulation) on
    the same tensors, written into `out` like dmoe_forward."""

    def __init__(self, hp, t):
        self.hp, self.t = hp, t

    def forward(self, h, out=None, stream=None):
        import oracle

        out.copy_(torch.from_numpy(oracle.layer(self.hp, self.t, h.numpy())[0].astype(np.float32)))
        return out


def cpu_model():
    import diffuse_moe as dm
    import synth

    cfg = llada2.LLaDA2Config(n_layer=3, n_embd=256, n_head=4, n_head_kv=2, head_dim=64, rotary_dim=32, n_ff=512,
                              first_k_dense=1, n_vocab=300, rope_base=10000.0, mask_token_id=299)
    w = llada2.LLaDA2Model.random_weights(cfg, seed=5, device="cpu")
    moe, specs = {}, {}
    for il in range(cfg.first_k_dense, cfg.n_layer):
        sp = synth.LayerSpec(H=256, I=256, Is=256, E=16, top_k=4, cap=6, blk=32, expert_type=dm.TYPE_Q8_0,
                             seed=60 + il)
        t = synth.make_layer(sp)
        moe[il] = OracleMoE(sp.hparams(), t)
        specs[il] = (sp.hparams(), t)
    return cfg, w, llada2.LLaDA2Model(cfg, w, moe, dtype=torch.float32, device="cpu"), specs


def test_model_forward_on_cpu_matches_restatement():
    """The model's host code (block-causal mask over the cache, GQA head mapping, RoPE positions,
    QK norm, residuals) on the CPU with the MoE layers replaced by the oracle: the logits of a
    3-block window match the float64 restatement; the last block's logits from the cache match
    the whole window."""
    cfg, w, model, specs = cpu_model()
    tokens = np.random.default_rng(1).integers(0, cfg.n_vocab - 1, size=96)
    got = model.forward(torch.as_tensor(tokens), 0).numpy()
    wn = {k: v.float().numpy() for k, v in w.items()}
    ref = llada2_ref.forward(cfg, wn, specs, tokens)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-4
    cache = model.new_cache(96)
    model.forward(torch.as_tensor(tokens[:64]), 0, cache, commit=64)
    part = model.forward(torch.as_tensor(tokens[64:]), 64, cache).numpy()
    assert np.linalg.norm(part - got[64:]) / np.linalg.norm(got[64:]) <= 1e-5


def oracle_sampler(logits, seq, mask_id, n_transfer, threshold, token, prob, n_committed):
    """diffuse_moe.sample_step's contract on CPU tensors, through the oracle's restatement."""
    import oracle

    tok, pr, s, nc = oracle.sample_step(logits.numpy(), seq.numpy(), mask_id, n_transfer, threshold)
    seq.copy_(torch.from_numpy(s))
    token.copy_(torch.from_numpy(tok))
    prob.copy_(torch.from_numpy(pr))
    n_committed.fill_(nc)


def test_generation_loop_on_cpu_cache_equals_recompute():
    """The block-diffusion loop (prefill, per-block steps, the previous block entering the cache in
    the next block's first step, the remaining-mask count) on the CPU with the oracle's MoE layers
    and sampler: the cached run commits the same tokens as the whole-window recompute, one forward
    more (the prefill)."""
    cfg, w, model, _ = cpu_model()
    w["output"][cfg.mask_token_id] = 0.0
    model.w["output"][cfg.mask_token_id] = 0.0
    prompt = np.random.default_rng(3).integers(0, cfg.n_vocab - 1, size=70)
    seq_c, nf_c = llada2.generate(model, prompt, 40, steps=4, threshold=0.95, use_cache=True, sampler=oracle_sampler)
    seq_r, nf_r = llada2.generate(model, prompt, 40, steps=4, threshold=0.95, use_cache=False, sampler=oracle_sampler)
    assert np.array_equal(seq_c, seq_r) and nf_c == nf_r + 1
    assert np.array_equal(seq_c[:70], prompt) and not np.any(seq_c == cfg.mask_token_id)
