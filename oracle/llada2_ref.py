"""CPU restatement of the full LLaDA2-MoE forward, for checking diffuse-cpp_b200/llada2.py.

TEST INFRASTRUCTURE ONLY: imported by tests/ as the checker; the product never imports it.

Follows diffuse_build_graph_moe (Akicou/diffuse-cpp src/diffuse-moe-graph.cpp) step by step, in
float64 numpy:
  - block-causal mask: query i sees key j iff i / block_length >= j / block_length (:38-52)
  - embedding rows (:109), per block: RMSNorm x / sqrt(mean x^2 + eps) * w (:123-124), fused
    QKV split as [Q heads; K heads; V heads] (:126-142), QK RMSNorm over head_dim (:145-150),
    partial NeoX RoPE over the first rotary_dim dims, theta_i = pos * base^(-2 i / rotary_dim)
    (:155-161), attention softmax(Q K^T / sqrt(head_dim) + mask) V with query head h reading
    KV head h / (n_head / n_head_kv) (:163-175), output projection and residual (:177-184),
    post-attention RMSNorm (:185-186), dense SwiGLU (:190-196) or the MoE layer (:197-288, the
    layer oracle in oracle.py), residual (:291); the output RMSNorm and lm_head (:295-299).
The MoE layer is oracle.layer (float64 accumulation). Weights are float32 arrays (the model's
parity runs keep the dense parts in fp32).
"""
from __future__ import annotations

import numpy as np

import oracle


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = x.astype(np.float64)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w.astype(np.float64)


def rope_neox(x: np.ndarray, pos: np.ndarray, rotary_dim: int, base: float) -> np.ndarray:
    half = rotary_dim // 2
    inv = base ** (-np.arange(half, dtype=np.float64) * 2.0 / rotary_dim)
    ang = pos.astype(np.float64)[:, None] * inv[None, :]
    cos, sin = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    x1, x2, rest = x[..., :half], x[..., half:rotary_dim], x[..., rotary_dim:]
    return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin, rest], axis=-1)


def forward(cfg, w: dict, moe: dict, tokens: np.ndarray) -> np.ndarray:
    """Logits [n, n_vocab] (float64) of the window `tokens` at positions 0 .. n - 1.
    w: name -> float32 array (the names of LLaDA2Model.random_weights); moe: block -> (hp, tensors)."""
    n = len(tokens)
    H, nh, nkv, hd = cfg.n_embd, cfg.n_head, cfg.n_head_kv, cfg.head_dim
    pos = np.arange(n)
    blk = pos // cfg.block_length
    mask = np.where(blk[:, None] >= blk[None, :], 0.0, -np.inf)
    x = w["tok_embd"][tokens].astype(np.float64)
    for il in range(cfg.n_layer):
        b = f"blk.{il}."
        residual = x
        h = rms_norm(x, w[b + "attn_norm"], cfg.rms_eps)
        qkv = h @ w[b + "attn_qkv"].astype(np.float64).T
        q = qkv[:, : nh * hd].reshape(n, nh, hd)
        k = qkv[:, nh * hd: (nh + nkv) * hd].reshape(n, nkv, hd)
        v = qkv[:, (nh + nkv) * hd:].reshape(n, nkv, hd)
        if cfg.use_qk_norm:
            q = rms_norm(q, w[b + "attn_q_norm"], cfg.rms_eps)
            k = rms_norm(k, w[b + "attn_k_norm"], cfg.rms_eps)
        q = rope_neox(q, pos, cfg.rotary_dim, cfg.rope_base)
        k = rope_neox(k, pos, cfg.rotary_dim, cfg.rope_base)
        o = np.empty((n, nh, hd))
        for hh in range(nh):
            kv = hh // (nh // nkv)
            s = q[:, hh, :] @ k[:, kv, :].T / np.sqrt(hd) + mask
            s = np.exp(s - s.max(axis=1, keepdims=True))
            o[:, hh, :] = (s / s.sum(axis=1, keepdims=True)) @ v[:, kv, :]
        x = o.reshape(n, nh * hd) @ w[b + "attn_output"].astype(np.float64).T + residual
        residual = x
        h = rms_norm(x, w[b + "post_attn_norm"], cfg.rms_eps)
        if il < cfg.first_k_dense:
            g = h @ w[b + "ffn_gate"].astype(np.float64).T
            u = h @ w[b + "ffn_up"].astype(np.float64).T
            y = ((g / (1.0 + np.exp(-g))) * u) @ w[b + "ffn_down"].astype(np.float64).T
        else:
            hp, t = moe[il]
            y = oracle.layer(hp, t, h.astype(np.float32))[0].astype(np.float64)
        x = y + residual
    x = rms_norm(x, w["output_norm"], cfg.rms_eps)
    return x @ w["output"].astype(np.float64).T
