"""Writes small LLaDA2-MoE GGUF files for the model-loader tests, with gguf-py's GGUFWriter (the
writer the reference's converter uses) and the converter's key and tensor names
(tools/convert-llada2-fast.py:95-120,130-144): architecture "diffuse", keys "diffuse.<name>",
dense blocks [0, first_k) with ffn_{gate,up,down}, MoE blocks with moe_gate (+ moe_gate_bias),
the expert stacks moe_experts_{gate,up,down} ([E][I][H] / [E][H][I]) and moe_shared_*.
The MoE tensors come from synth.make_layer with one seed per block.
"""
from __future__ import annotations

import dataclasses

import numpy as np
from gguf import GGMLQuantizationType, GGUFWriter

import diffuse_moe as dm
import synth


@dataclasses.dataclass
class ModelSpec:
    n_layer: int = 3
    first_k: int = 1
    H: int = 256
    I: int = 256
    Is: int = 256
    E: int = 16
    top_k: int = 4
    cap: int = 6
    blk: int = 32
    scale: float = 2.5
    expert_type: int = dm.TYPE_Q4_K
    shared_type: int | None = None
    seed: int = 40

    def layer_spec(self, il: int) -> synth.LayerSpec:
        return synth.LayerSpec(H=self.H, I=self.I, Is=self.Is, E=self.E, top_k=self.top_k, cap=self.cap,
                               blk=self.blk, scale=self.scale, expert_type=self.expert_type,
                               shared_type=self.shared_type, seed=self.seed + il)


def _stack(t: np.ndarray, E: int) -> np.ndarray:
    """[E * rows, row_bytes] GGUF bytes -> [E, rows, row_bytes] (numpy order of ne [k, rows, E])."""
    return t.reshape(E, t.shape[0] // E, t.shape[1])


def write_model(path: str, ms: ModelSpec, *, drop=(), override=None, keys=None, model_type="llada2_moe",
                alignment=None, omit=(), extra=None) -> dict:
    """Writes the model; returns {il: tensors} of its MoE blocks. drop: tensor names to leave out;
    override: {tensor name: array (and raw type)} to replace; keys: extra / replaced u32 keys;
    omit: key names (without the prefix) to leave out; extra(writer): adds further metadata."""
    override = override or {}
    w = GGUFWriter(path, "diffuse")
    if alignment is not None:
        w.add_custom_alignment(alignment)
    u32 = {"block_count": ms.n_layer, "embedding_length": ms.H, "attention.head_count": 4,
           "attention.head_count_kv": 4, "feed_forward_length": 2 * ms.H, "expert_count": ms.E,
           "expert_used_count": ms.top_k, "expert_shared_count": 1 if ms.Is else 0,
           "expert_feed_forward_length": ms.I, "first_k_dense_replace": ms.first_k, "norm_topk_prob": 1,
           "block_length": ms.blk, "moe_block_size": ms.blk, "expert_capacity": ms.cap}
    u32.update(keys or {})
    for k, v in u32.items():
        if k not in omit:
            w.add_uint32(f"diffuse.{k}", v)
    if "routed_scaling_factor" not in omit:
        w.add_float32("diffuse.routed_scaling_factor", ms.scale)
    w.add_float32("diffuse.attention.layer_norm_rms_epsilon", 1e-6)
    if model_type is not None:
        w.add_string("diffuse.model_type", model_type)
    if extra is not None:
        extra(w)
    rng = np.random.default_rng(ms.seed)

    def put(name, arr, raw=None):
        if name in drop:
            return
        if name in override:
            arr, raw = override[name]
        w.add_tensor(name, arr, raw_dtype=None if raw is None else GGMLQuantizationType(raw))

    put("token_embd.weight", rng.standard_normal((64, ms.H)).astype(np.float16))
    layers = {}
    for il in range(ms.n_layer):
        b = f"blk.{il}."
        put(b + "attn_norm.weight", np.ones(ms.H, np.float32))
        if il < ms.first_k:
            put(b + "ffn_gate.weight", rng.standard_normal((2 * ms.H, ms.H)).astype(np.float16))
            put(b + "ffn_up.weight", rng.standard_normal((2 * ms.H, ms.H)).astype(np.float16))
            put(b + "ffn_down.weight", rng.standard_normal((ms.H, 2 * ms.H)).astype(np.float16))
            continue
        t = synth.make_layer(ms.layer_spec(il))
        layers[il] = t
        put(b + "moe_gate.weight", t["w_router"])
        if t["b_router"] is not None:
            put(b + "moe_gate_bias.weight", t["b_router"])
        put(b + "moe_experts_gate.weight", _stack(t["w_gate"], ms.E), ms.expert_type)
        put(b + "moe_experts_up.weight", _stack(t["w_up"], ms.E), ms.expert_type)
        put(b + "moe_experts_down.weight", _stack(t["w_down"], ms.E), ms.expert_type)
        if ms.Is:
            st = ms.expert_type if ms.shared_type is None else ms.shared_type
            put(b + "moe_shared_gate.weight", t["sw_gate"], st)
            put(b + "moe_shared_up.weight", t["sw_up"], st)
            put(b + "moe_shared_down.weight", t["sw_down"], st)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return layers
