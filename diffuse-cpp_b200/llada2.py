"""The full LLaDA2-MoE forward and its block-diffusion generation loop on one GPU, around
libdiffuse_moe's MoE layers and sampler step.

Reference: diffuse_build_graph_moe (src/diffuse-moe-graph.cpp:72-305, block-causal mask :19-55)
and generate_block_diffusion (src/diffuse-sampler.cpp:100-258). Per block: RMSNorm, fused QKV,
QK RMSNorm over head_dim, partial NeoX RoPE on the first rotary_dim dims, attention with the
block-causal mask (GQA: query head h reads KV head h / (n_head / n_head_kv)), output projection,
residual, post-attention RMSNorm, dense SwiGLU (blocks < first_k_dense) or the MoE layer, residual;
then the output RMSNorm and the lm_head.

The MoE layers and the sampler step are this library's CUDA kernels (dmoe_forward,
dmoe_sample_step); attention, the dense projections and the lm_head are PyTorch library calls
(cuBLAS GEMMs, scaled_dot_product_attention) on bf16 weights, or fp32 for parity checks.

Generation keeps a key/value cache of the committed blocks. This gives the reference's results
for the block being denoised: the mask is block-causal, so a committed block's keys and values
depend on no later block, and MoE routing couples only the tokens of one routing block. The
reference instead recomputes the whole window at every step. A block enters the cache in the
first step of the next block, whose forward covers both blocks (block-causal mask between them).
"""
from __future__ import annotations

import dataclasses
import math
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F

import diffuse_moe as dm


@dataclasses.dataclass
class LLaDA2Config:
    n_layer: int = 32
    n_embd: int = 4096
    n_head: int = 32
    n_head_kv: int = 4
    head_dim: int = 128
    rotary_dim: int = 64
    n_ff: int = 9216            # dense blocks (first_k_dense)
    first_k_dense: int = 1
    n_vocab: int = 157184
    rms_eps: float = 1e-6
    rope_base: float = 600000.0
    use_qk_norm: bool = True
    block_length: int = 32
    mask_token_id: int = 156895

    @property
    def qkv_dim(self) -> int:
        return (self.n_head + 2 * self.n_head_kv) * self.head_dim


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """ggml_rms_norm then ggml_mul (moe-graph.cpp:123-124): x / sqrt(mean x^2 + eps) * w, in fp32."""
    return F.rms_norm(x.float(), (x.shape[-1],), w, eps)


def rope_tables(pos: torch.Tensor, rotary_dim: int, base: float) -> tuple:
    """cos / sin [n, 1, rotary_dim / 2] of theta_i = pos * base^(-2 i / rotary_dim) (angles in fp64)."""
    half = rotary_dim // 2
    inv = base ** (-torch.arange(0, half, device=pos.device, dtype=torch.float64) * 2.0 / rotary_dim)
    ang = (pos.to(torch.float64)[:, None] * inv[None, :]).float()
    return ang.cos()[:, None, :], ang.sin()[:, None, :]


def rope_neox(x: torch.Tensor, pos: torch.Tensor, rotary_dim: int, base: float, tables=None) -> torch.Tensor:
    """Partial NeoX RoPE (ggml_rope_ext, GGML_ROPE_TYPE_NEOX, moe-graph.cpp:155-161): the first
    rotary_dim dims of each head rotate as two halves (x1, x2) -> (x1 cos - x2 sin, x2 cos + x1 sin)
    with theta_i = pos * base^(-2 i / rotary_dim); the rest pass through. x: [n, heads, head_dim]."""
    half = rotary_dim // 2
    cos, sin = tables if tables is not None else rope_tables(pos, rotary_dim, base)
    x1, x2, rest = x[..., :half], x[..., half:rotary_dim], x[..., rotary_dim:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin, rest], dim=-1)


class LLaDA2Model:
    """Weights on one GPU. `moe_layers[il]` is a diffuse_moe.MoELayer for every block
    il >= first_k_dense; the rest are torch tensors in `dtype` (bf16 for speed, fp32 for parity)."""

    def __init__(self, cfg: LLaDA2Config, weights: dict, moe_layers: dict, dtype=torch.bfloat16,
                 device: str = "cuda"):
        self.cfg = cfg
        self.dtype = dtype
        self.device = torch.device(device)
        self.w = {k: v.to(self.device, dtype if v.dim() == 2 else torch.float32) for k, v in weights.items()}
        self.moe = moe_layers
        # CUDA-graph state: a persistent cache the graphs read and write, the graphs by window
        # size, and the largest eager window so far. The MoE layers grow their workspaces only
        # for a window larger than any before, and a grown workspace would leave a captured graph
        # pointing at freed memory, so a larger eager window drops the graphs first.
        self._gcache = None
        self._graphs = {}
        self._max_n = 0
        self._graph_max_n = 0

    def reserve(self, max_len: int) -> dict:
        """The persistent cache of the CUDA-graph path, at least max_len positions (a larger one
        drops the graphs, which are bound to the old cache)."""
        if self._gcache is None or self._gcache["k"].shape[2] < max_len:
            self.drop_graphs()
            self._gcache = self.new_cache(max_len)
        return self._gcache

    def drop_graphs(self) -> None:
        if self._graphs:
            torch.cuda.synchronize(self.device)
            self._graphs.clear()

    def step_graph(self, n: int) -> "_StepGraph":
        if n not in self._graphs:
            self._graphs[n] = _StepGraph(self, n, self._gcache)
            self._graph_max_n = max(self._graph_max_n, self._max_n, n)
        return self._graphs[n]

    @staticmethod
    def random_weights(cfg: LLaDA2Config, seed: int, device: str = "cuda", std: float = 0.02) -> dict:
        """Random-init tensors of the non-MoE parts (norm weights 1 + small noise)."""
        g = torch.Generator(device=device).manual_seed(seed)
        H, hd = cfg.n_embd, cfg.head_dim

        def mat(rows, cols):
            return torch.randn(rows, cols, generator=g, device=device, dtype=torch.float32) * std

        def norm(n):
            return 1.0 + 0.1 * torch.randn(n, generator=g, device=device, dtype=torch.float32)

        w = {"tok_embd": mat(cfg.n_vocab, H) * 50.0, "output_norm": norm(H), "output": mat(cfg.n_vocab, H)}
        for il in range(cfg.n_layer):
            b = f"blk.{il}."
            w[b + "attn_norm"] = norm(H)
            w[b + "post_attn_norm"] = norm(H)
            w[b + "attn_qkv"] = mat(cfg.qkv_dim, H)
            w[b + "attn_output"] = mat(H, cfg.n_head * hd)
            if cfg.use_qk_norm:
                w[b + "attn_q_norm"] = norm(hd)
                w[b + "attn_k_norm"] = norm(hd)
            if il < cfg.first_k_dense:
                w[b + "ffn_gate"] = mat(cfg.n_ff, H)
                w[b + "ffn_up"] = mat(cfg.n_ff, H)
                w[b + "ffn_down"] = mat(H, cfg.n_ff)
        return w

    def _lin(self, x: torch.Tensor, name: str) -> torch.Tensor:
        return (x.to(self.dtype) @ self.w[name].t()).float()

    def new_cache(self, max_len: int) -> dict:
        """Keys / values of positions [0, max_len) for every block (zeroed: masked slots must hold
        finite values); `len` = how many leading positions are final."""
        c = self.cfg
        shape = (c.n_layer, c.n_head_kv, max_len, c.head_dim)
        return {"k": torch.zeros(shape, device=self.device, dtype=self.dtype),
                "v": torch.zeros(shape, device=self.device, dtype=self.dtype), "len": 0}

    def forward(self, tokens: torch.Tensor, pos0: int, cache: Optional[dict] = None, commit: int = 0,
                stream: Optional[int] = None) -> torch.Tensor:
        """Logits [n, n_vocab] f32 of `tokens` (int64 [n], a whole number of blocks) at positions
        pos0 .. pos0 + n - 1, attending to the cache's positions before pos0 (which must be final).
        The tokens' keys and values are written into the cache; the first `commit` of them are
        marked final. Without a cache (pos0 = 0) a temporary one covers the window."""
        n = int(tokens.shape[0])
        if n > self._max_n:
            if self._graphs and n > self._graph_max_n:
                self.drop_graphs()  # before the MoE layers grow under them
            self._max_n = n
        if cache is None:
            if pos0 != 0:
                raise ValueError("a window without a cache starts at position 0")
            cache = self.new_cache(n)
        elif cache["len"] < pos0:
            raise ValueError("the cache must hold the positions before pos0")
        pos = torch.arange(pos0, pos0 + n, device=self.device)
        logits = self.forward_static(tokens, pos, cache["k"], cache["v"], stream)
        cache["len"] = max(cache["len"], pos0 + commit)
        return logits

    def forward_static(self, tokens: torch.Tensor, pos: torch.Tensor, ck: torch.Tensor, cv: torch.Tensor,
                       stream: Optional[int] = None) -> torch.Tensor:
        """The forward with every shape fixed by (n, cache length), so that it can be captured in
        a CUDA graph: positions come as a device tensor, each block's keys and values are written
        into the cache at their positions, and attention runs over the whole cache under the
        block-causal mask (moe-graph.cpp:38-52: key j is visible to query i iff block(j) <= block(i);
        slots of later blocks are masked)."""
        c = self.cfg
        n = int(tokens.shape[0])
        lmax = ck.shape[2]
        bq = pos // c.block_length
        bk = torch.arange(lmax, device=self.device) // c.block_length
        mask = (bk[None, :] <= bq[:, None])[None, None]
        tables = rope_tables(pos, c.rotary_dim, c.rope_base)
        y = torch.empty((n, c.n_embd), device=self.device, dtype=torch.float32)  # MoE outputs
        x = self.w["tok_embd"][tokens].float()
        nq, nkv, hd = c.n_head, c.n_head_kv, c.head_dim
        for il in range(c.n_layer):
            b = f"blk.{il}."
            residual = x
            h = rms_norm(x, self.w[b + "attn_norm"], c.rms_eps)
            qkv = self._lin(h, b + "attn_qkv")
            q = qkv[:, : nq * hd].view(n, nq, hd)
            k = qkv[:, nq * hd: (nq + nkv) * hd].view(n, nkv, hd)
            v = qkv[:, (nq + nkv) * hd:].view(n, nkv, hd)
            if c.use_qk_norm:
                q = rms_norm(q, self.w[b + "attn_q_norm"], c.rms_eps)
                k = rms_norm(k, self.w[b + "attn_k_norm"], c.rms_eps)
            q = rope_neox(q, pos, c.rotary_dim, c.rope_base, tables)
            k = rope_neox(k, pos, c.rotary_dim, c.rope_base, tables)
            ck[il].index_copy_(1, pos, k.transpose(0, 1).to(self.dtype))
            cv[il].index_copy_(1, pos, v.transpose(0, 1).to(self.dtype))
            o = F.scaled_dot_product_attention(q.transpose(0, 1).to(self.dtype)[None], ck[il][None], cv[il][None],
                                               attn_mask=mask, scale=1.0 / math.sqrt(hd), enable_gqa=True)
            o = o[0].transpose(0, 1).reshape(n, nq * hd)
            x = self._lin(o, b + "attn_output") + residual
            residual = x
            h = rms_norm(x, self.w[b + "post_attn_norm"], c.rms_eps)
            if il < c.first_k_dense:
                g = self._lin(h, b + "ffn_gate")
                u = self._lin(h, b + "ffn_up")
                x = self._lin(F.silu(g) * u, b + "ffn_down") + residual
            else:
                self.moe[il].forward(h.contiguous(), out=y, stream=stream)
                x = y + residual
        x = rms_norm(x, self.w["output_norm"], c.rms_eps)
        return self._lin(x, "output")


class _StepGraph:
    """One CUDA graph of LLaDA2Model.forward_static for n tokens over a fixed cache: fill `tokens`
    and `pos`, replay, read `logits`. Captured on first use after two eager runs of the same
    inputs (the runs compute the same keys and values the replay writes)."""

    def __init__(self, model: LLaDA2Model, n: int, cache: dict):
        self.model, self.cache = model, cache
        self.tokens = torch.zeros(n, dtype=torch.int64, device=model.device)
        self.pos = torch.zeros(n, dtype=torch.int64, device=model.device)
        self.graph = None
        self.logits = None

    def __call__(self, tokens: torch.Tensor, pos0: int) -> torch.Tensor:
        self.tokens.copy_(tokens)
        torch.arange(pos0, pos0 + self.tokens.shape[0], device=self.tokens.device, out=self.pos)
        if self.graph is None:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(2):
                    self.model.forward_static(self.tokens, self.pos, self.cache["k"], self.cache["v"])
            torch.cuda.current_stream().wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.logits = self.model.forward_static(self.tokens, self.pos, self.cache["k"], self.cache["v"])
        self.graph.replay()
        return self.logits


def transfer_schedule(block_length: int, steps: int) -> list:
    """get_num_transfer_tokens (diffuse-sampler.cpp:16-25): block_length / steps per step, the
    remainder spread over the first steps."""
    if steps == 0:
        return []
    base, rem = divmod(block_length, steps)
    return [base + (1 if i < rem else 0) for i in range(steps)]


def generate(model: LLaDA2Model, prompt: np.ndarray, n_generate: int, steps: int = 8, threshold: float = 0.95,
             use_cache: bool = True, graphs: bool = False, sampler=None) -> tuple:
    """Greedy low-confidence block diffusion (generate_block_diffusion, diffuse-sampler.cpp:100-258):
    blocks tile from position 0; the prompt's whole blocks are prefilled; each later block runs up
    to `steps` denoising steps, each committing the schedule's count of its most confident masked
    positions plus any at or above `threshold` (at least one), until none is masked. Returns the
    sequence (int32 numpy) and the number of forwards. use_cache=False recomputes the whole window
    at every step, as the reference does. graphs=True (with the cache) replays each step's forward
    from a CUDA graph, one per window size, kept by the model over the cache of model.reserve()
    (captured at first use, after the prefill). sampler: the step function with the signature of
    diffuse_moe.sample_step (default: this library's GPU kernel)."""
    sample = dm.sample_step if sampler is None else sampler
    c = model.cfg
    L = c.block_length
    prompt_len = len(prompt)
    n_blocks = (prompt_len + n_generate + L - 1) // L
    total = n_blocks * L
    dev = model.device
    seq = torch.full((total,), c.mask_token_id, dtype=torch.int32, device=dev)
    seq[:prompt_len] = torch.as_tensor(prompt, dtype=torch.int32, device=dev)
    prefill = prompt_len // L
    sched = transfer_schedule(L, min(steps, L))
    if use_cache and graphs:
        cache = model.reserve(total)
        cache["len"] = 0
    else:
        cache = model.new_cache(total) if use_cache else None
    token = torch.empty(L, dtype=torch.int32, device=dev)
    prob = torch.empty(L, dtype=torch.float32, device=dev)
    ncom = torch.zeros(1, dtype=torch.int32, device=dev)
    forwards = 0
    if use_cache and prefill > 1:  # every whole prompt block but the last enters the cache
        model.forward(seq[: (prefill - 1) * L].long(), 0, cache, commit=(prefill - 1) * L)
        forwards += 1
    for blk in range(prefill, n_blocks):
        b0 = blk * L
        remaining = int((seq[b0: b0 + L] == c.mask_token_id).sum().item())
        for step in range(len(sched)):
            if remaining == 0:
                break
            if use_cache:
                p0 = cache["len"]  # the previous block (final) and this one
                if graphs:
                    logits = model.step_graph(b0 + L - p0)(seq[p0: b0 + L].long(), p0)[b0 - p0:]
                    cache["len"] = b0
                else:
                    logits = model.forward(seq[p0: b0 + L].long(), p0, cache, commit=b0 - p0)[b0 - p0:]
            else:
                logits = model.forward(seq[: b0 + L].long(), 0)[b0:]
            forwards += 1
            blk_seq = seq[b0: b0 + L]
            sample(logits.contiguous(), blk_seq, c.mask_token_id, sched[step], threshold, token, prob, ncom)
            remaining -= int(ncom.item())
    return seq.cpu().numpy(), forwards
