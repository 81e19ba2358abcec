"""ctypes binding of libdiffuse_moe (C ABI: include/diffuse_moe.h).

This is the host-side mirror of the reference's MoE call site
(src/diffuse-moe-graph.cpp:195-287 inside diffuse_build_graph_moe): a layer is bound once from
its GGUF tensors (struct diffuse_moe_layer, src/diffuse-common.h:59-86) and called with
moe_in [n_tokens, n_embd] f32, returning moe_out (routed + shared, no residual).

There is no CPU fallback: if the shared library is missing, or the machine has no CUDA device,
the calls raise. Inputs may be numpy arrays (host memory; the call copies in and out and
returns when done) or torch CUDA tensors (device memory; work is enqueued on the current torch
stream and `sync()` waits for it).
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdiffuse_moe.so")

# ggml_type ids (ggml.h)
TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K = 0, 1, 8, 12
TYPE_NAMES = {TYPE_F32: "f32", TYPE_F16: "f16", TYPE_Q8_0: "q8_0", TYPE_Q4_K: "q4_K"}

F_HOST_PTRS, F_ROUTE_ONLY, F_PROFILE, F_DETERMINISTIC = 1, 2, 4, 8

STATUS_NAMES = {
    0: "DMOE_OK",
    1: "DMOE_ERR_INVALID_ARG",
    2: "DMOE_ERR_UNSUPPORTED",
    3: "DMOE_ERR_NO_DEVICE",
    4: "DMOE_ERR_CUDA",
    5: "DMOE_ERR_NCCL",
    6: "DMOE_ERR_TIMEOUT",
    7: "DMOE_ERR_OOM",
}


class LayerDesc(ctypes.Structure):
    _fields_ = [
        ("n_embd", ctypes.c_int64),
        ("n_ff_exp", ctypes.c_int64),
        ("n_ff_shexp", ctypes.c_int64),
        ("n_expert", ctypes.c_int64),
        ("n_expert_used", ctypes.c_int64),
        ("expert_capacity", ctypes.c_int64),
        ("moe_block_size", ctypes.c_int64),
        ("routed_scaling", ctypes.c_float),
        ("norm_topk_prob", ctypes.c_int32),
        ("expert_type", ctypes.c_int32),
        ("shared_type", ctypes.c_int32),
        ("w_gate", ctypes.c_void_p),
        ("w_up", ctypes.c_void_p),
        ("w_down", ctypes.c_void_p),
        ("sw_gate", ctypes.c_void_p),
        ("sw_up", ctypes.c_void_p),
        ("sw_down", ctypes.c_void_p),
        ("w_router", ctypes.c_void_p),
        ("b_router", ctypes.c_void_p),
    ]


class DistCfg(ctypes.Structure):
    _fields_ = [
        ("rank", ctypes.c_int32),
        ("world_size", ctypes.c_int32),
        ("device", ctypes.c_int32),
        ("timeout_ms", ctypes.c_int32),
        ("nccl_id", ctypes.c_void_p),
    ]


class RouteOut(ctypes.Structure):
    _fields_ = [
        ("idx", ctypes.c_void_p),
        ("weights", ctypes.c_void_p),
        ("allowed", ctypes.c_void_p),
    ]


class Stats(ctypes.Structure):
    _fields_ = [
        ("n_active", ctypes.c_int32),
        ("n_routed_tiles", ctypes.c_int32),
        ("token_tile", ctypes.c_int32),
        ("ksplit_gateup", ctypes.c_int32),
        ("ksplit_down", ctypes.c_int32),
        ("router_parts", ctypes.c_int32),
        ("kernels", ctypes.c_int32),
        ("used_block_routing", ctypes.c_int32),
        ("ms_router", ctypes.c_float),
        ("ms_dispatch", ctypes.c_float),
        ("ms_gateup", ctypes.c_float),
        ("ms_down", ctypes.c_float),
        ("ms_total", ctypes.c_float),
        ("ep_rows_sent", ctypes.c_int64),
        ("ep_rows_received", ctypes.c_int64),
        ("fused_gemm", ctypes.c_int32),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class ModelInfo(ctypes.Structure):
    _fields_ = [
        ("n_layer", ctypes.c_int32),
        ("first_k_dense", ctypes.c_int32),
        ("n_moe_layers", ctypes.c_int32),
        ("expert_type", ctypes.c_int32),
        ("shared_type", ctypes.c_int32),
        ("norm_topk_prob", ctypes.c_int32),
        ("routed_scaling", ctypes.c_float),
        ("n_embd", ctypes.c_int64),
        ("n_ff_exp", ctypes.c_int64),
        ("n_ff_shexp", ctypes.c_int64),
        ("n_expert", ctypes.c_int64),
        ("n_expert_used", ctypes.c_int64),
        ("expert_capacity", ctypes.c_int64),
        ("moe_block_size", ctypes.c_int64),
        ("moe_bytes", ctypes.c_int64),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class DmoeError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads libdiffuse_moe.so. Raises if it has not been built (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `make -C diffuse-cpp_b200` (no CPU fallback)")
    lib = ctypes.CDLL(path)
    P = ctypes.c_void_p
    lib.dmoe_create.argtypes = [ctypes.POINTER(LayerDesc), ctypes.POINTER(DistCfg), ctypes.POINTER(P)]
    lib.dmoe_create.restype = ctypes.c_int
    lib.dmoe_forward.argtypes = [P, P, ctypes.c_int64, P, ctypes.POINTER(RouteOut), P, ctypes.c_uint32]
    lib.dmoe_forward.restype = ctypes.c_int
    lib.dmoe_sync.argtypes = [P]
    lib.dmoe_sync.restype = ctypes.c_int
    lib.dmoe_get_stats.argtypes = [P, ctypes.POINTER(Stats)]
    lib.dmoe_get_stats.restype = ctypes.c_int
    lib.dmoe_destroy.argtypes = [P]
    lib.dmoe_destroy.restype = None
    lib.dmoe_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    lib.dmoe_last_error.restype = ctypes.c_size_t
    lib.dmoe_abi_version.argtypes = []
    lib.dmoe_abi_version.restype = ctypes.c_int32
    lib.dmoe_quantize.argtypes = [ctypes.c_int32, P, P, ctypes.c_int64, ctypes.c_int64]
    lib.dmoe_quantize.restype = ctypes.c_size_t
    lib.dmoe_quantized_size.argtypes = [ctypes.c_int32, ctypes.c_int64, ctypes.c_int64]
    lib.dmoe_quantized_size.restype = ctypes.c_size_t
    lib.dmoe_route_static.argtypes = [P, ctypes.c_int64, ctypes.c_int64, P, P, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_int32, P, P, P]
    lib.dmoe_route_static.restype = ctypes.c_int
    lib.dmoe_nccl_unique_id.argtypes = [P]
    lib.dmoe_nccl_unique_id.restype = ctypes.c_int
    lib.dmoe_replicate_experts.argtypes = [P, P, ctypes.c_int32]
    lib.dmoe_replicate_experts.restype = ctypes.c_int
    lib.dmoe_sample_step.argtypes = [P, ctypes.c_int64, ctypes.c_int64, P, ctypes.c_int32, ctypes.c_int32,
                                     ctypes.c_float, P, P, P, P]
    lib.dmoe_sample_step.restype = ctypes.c_int
    lib.dmoe_create_split.argtypes = [ctypes.POINTER(LayerDesc), ctypes.POINTER(DistCfg), P, ctypes.POINTER(P)]
    lib.dmoe_create_split.restype = ctypes.c_int
    lib.dmoe_model_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(DistCfg), ctypes.POINTER(P)]
    lib.dmoe_model_load.restype = ctypes.c_int
    lib.dmoe_model_inspect.argtypes = [ctypes.c_char_p, ctypes.POINTER(ModelInfo)]
    lib.dmoe_model_inspect.restype = ctypes.c_int
    lib.dmoe_model_get_info.argtypes = [P, ctypes.POINTER(ModelInfo)]
    lib.dmoe_model_get_info.restype = ctypes.c_int
    lib.dmoe_model_layer.argtypes = [P, ctypes.c_int32]
    lib.dmoe_model_layer.restype = P
    lib.dmoe_model_free.argtypes = [P]
    lib.dmoe_model_free.restype = None
    _lib = lib
    return lib


def nccl_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id (dmoe_nccl_unique_id): make it on one rank, share it."""
    buf = ctypes.create_string_buffer(128)
    _check(load().dmoe_nccl_unique_id(buf))
    return buf.raw


def dist_cfg(rank: int, world_size: int, device: int, nccl_id: Optional[bytes] = None, timeout_ms: int = 0):
    """dmoe_dist_cfg for one rank; the returned object keeps the id buffer alive."""
    cfg = DistCfg(rank, world_size, device, timeout_ms, None)
    if nccl_id is not None:
        if len(nccl_id) != 128:
            raise ValueError("nccl_id must be 128 bytes")
        cfg._id = ctypes.create_string_buffer(nccl_id, 128)
        cfg.nccl_id = ctypes.cast(cfg._id, ctypes.c_void_p)
    return cfg


def last_error() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(2048)
    lib.dmoe_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def _check(status: int) -> None:
    if status != 0:
        raise DmoeError(status, last_error())


def quantized_size(qtype: int, nrows: int, n_per_row: int) -> int:
    return int(load().dmoe_quantized_size(qtype, nrows, n_per_row))


def quantize(values: np.ndarray, qtype: int) -> np.ndarray:
    """Quantises a [rows, n_per_row] float32 array to GGUF block bytes (uint8 [rows, row_bytes])."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    if v.ndim == 1:
        v = v[None, :]
    rows, k = v.shape
    rs = quantized_size(qtype, 1, k)
    if rs == 0:
        raise ValueError(f"row length {k} is not a whole number of blocks of type {qtype}")
    out = np.empty((rows, rs), dtype=np.uint8)
    n = load().dmoe_quantize(qtype, v.ctypes.data, out.ctypes.data, rows, k)
    if n != rows * rs:
        raise RuntimeError("dmoe_quantize failed")
    return out


def _ptr(a) -> int:
    if a is None:
        return 0
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()  # torch tensor


class MoELayer:
    """One bound MoE layer (dmoe_create). `tensors` holds the GGUF tensors:
    w_gate/w_up/w_down (uint8 bytes or float16 arrays), sw_*, w_router [E, H] f32, b_router [E] f32 or None."""

    def __init__(self, hp: dict, tensors: dict, dist: Optional[DistCfg] = None, parent: Optional["MoELayer"] = None):
        """parent: an expert-parallel layer of the same ranks whose communicator this layer's is
        split from (dmoe_create_split); dist.nccl_id is then not needed."""
        lib = load()
        self._owner = None
        self._keep = {}
        d = LayerDesc()
        d.n_embd = hp["n_embd"]
        d.n_ff_exp = hp["n_ff_exp"]
        d.n_ff_shexp = hp.get("n_ff_shexp", 0)
        d.n_expert = hp["n_expert"]
        d.n_expert_used = hp["n_expert_used"]
        d.expert_capacity = hp.get("expert_capacity", 48)
        d.moe_block_size = hp.get("moe_block_size", 32)
        d.routed_scaling = hp.get("routed_scaling", 1.0)
        d.norm_topk_prob = hp.get("norm_topk_prob", 1)
        d.expert_type = hp["expert_type"]
        d.shared_type = hp.get("shared_type", hp["expert_type"])
        for name in ("w_gate", "w_up", "w_down", "sw_gate", "sw_up", "sw_down", "w_router", "b_router"):
            t = tensors.get(name)
            if t is not None:
                t = np.ascontiguousarray(t)
                self._keep[name] = t
                setattr(d, name, t.ctypes.data)
            else:
                setattr(d, name, None)
        self.hp = dict(hp)
        self.desc = d
        h = ctypes.c_void_p()
        dp = ctypes.byref(dist) if dist is not None else None
        if parent is not None:
            _check(lib.dmoe_create_split(ctypes.byref(d), dp, parent._h, ctypes.byref(h)))
        else:
            _check(lib.dmoe_create(ctypes.byref(d), dp, ctypes.byref(h)))
        self._h = h
        self._keep.clear()  # weights are on the device now

    @classmethod
    def _borrowed(cls, handle: int, hp: dict, owner) -> "MoELayer":
        """A view of a layer owned by a MoEModel (freed with the model, not by close())."""
        self = cls.__new__(cls)
        self._h = ctypes.c_void_p(handle)
        self.hp = dict(hp)
        self._keep = {}
        self._owner = owner
        return self

    def forward(self, x, out=None, route: bool = False, route_only: bool = False, profile: bool = False,
                stream: Optional[int] = None, deterministic: bool = False):
        """x: numpy [n, H] float32 (host mode) or torch CUDA float32 tensor (device mode).
        Returns out (and (idx, weights, allowed) when route=True). deterministic=True selects the
        bitwise-reproducible slot-order sum (DMOE_F_DETERMINISTIC)."""
        lib = load()
        H = self.hp["n_embd"]
        K = self.hp["n_expert_used"]
        E = self.hp["n_expert"]
        blk = self.hp.get("moe_block_size", 32)
        is_np = isinstance(x, np.ndarray)
        n = int(x.shape[0])
        flags = ((F_HOST_PTRS if is_np else 0) | (F_ROUTE_ONLY if route_only else 0) | (F_PROFILE if profile else 0)
                 | (F_DETERMINISTIC if deterministic else 0))
        if is_np:
            x = np.ascontiguousarray(x, dtype=np.float32)
            if out is None and not route_only:
                out = np.empty((n, H), dtype=np.float32)
            mk = lambda shape, dt: np.empty(shape, dtype=dt)  # noqa: E731
        else:
            import torch

            if out is None and not route_only:
                out = torch.empty((n, H), dtype=torch.float32, device=x.device)
            mk = lambda shape, dt: torch.empty(shape, dtype={np.int32: torch.int32, np.float32: torch.float32,  # noqa: E731
                                                             np.uint8: torch.uint8}[dt], device=x.device)
            if stream is None:
                stream = torch.cuda.current_stream(x.device).cuda_stream
        ro = None
        routes = None
        if route or route_only:
            idx = mk((n, K), np.int32)
            w = mk((n, K), np.float32)
            allowed = mk((max(n // blk, 1), E), np.uint8) if blk > 0 else None
            ro = RouteOut(_ptr(idx), _ptr(w), _ptr(allowed))
            routes = (idx, w, allowed)
        _check(lib.dmoe_forward(self._h, _ptr(x), n, _ptr(out), ctypes.byref(ro) if ro is not None else None,
                                stream if stream else None, flags))
        if route or route_only:
            return (out, routes) if not route_only else routes
        return out

    def sync(self) -> None:
        _check(load().dmoe_sync(self._h))

    def replicate_experts(self, n_hot: int, ids=None) -> None:
        """dmoe_replicate_experts (collective on every rank of an expert-parallel layer): hold the
        weights of n_hot experts on every rank, the given ids or (None) the busiest of the last
        forward summed over the ranks; their (token, slot) pairs are then computed locally."""
        arr = None
        if ids is not None:
            arr = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
            if arr.size != n_hot:
                raise ValueError("len(ids) must equal n_hot")
        _check(load().dmoe_replicate_experts(self._h, None if arr is None else arr.ctypes.data, n_hot))

    def stats(self) -> dict:
        s = Stats()
        _check(load().dmoe_get_stats(self._h, ctypes.byref(s)))
        return s.as_dict()

    def close(self) -> None:
        if getattr(self, "_owner", None) is not None:  # borrowed from a model
            self._h = None
            return
        if getattr(self, "_h", None):
            load().dmoe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def model_inspect(path: str) -> dict:
    """dmoe_model_inspect: the hyper-parameters and MoE tensor checks of a GGUF model, no device."""
    info = ModelInfo()
    _check(load().dmoe_model_inspect(os.fsencode(path), ctypes.byref(info)))
    return info.as_dict()


class MoEModel:
    """Every MoE layer of a GGUF model bound once (dmoe_model_load; replaces
    diffuse_model_load_impl, src/diffuse-model.cpp:67-224, for the MoE blocks). `layer(il)` is the
    MoELayer of block il (None for a dense block); the layers live as long as the model."""

    def __init__(self, path: str, dist: Optional[DistCfg] = None):
        lib = load()
        h = ctypes.c_void_p()
        _check(lib.dmoe_model_load(os.fsencode(path), ctypes.byref(dist) if dist is not None else None,
                                   ctypes.byref(h)))
        self._h = h
        info = ModelInfo()
        _check(lib.dmoe_model_get_info(self._h, ctypes.byref(info)))
        self.info = info.as_dict()
        hp = {k: self.info[k] for k in ("n_embd", "n_ff_exp", "n_ff_shexp", "n_expert", "n_expert_used",
                                        "expert_capacity", "moe_block_size", "routed_scaling", "norm_topk_prob",
                                        "expert_type", "shared_type")}
        self._layers = {}
        for il in range(self.info["first_k_dense"], self.info["n_layer"]):
            lh = lib.dmoe_model_layer(self._h, il)
            if not lh:
                raise DmoeError(1, f"dmoe_model_layer({il}) returned NULL")
            self._layers[il] = MoELayer._borrowed(lh, hp, self)

    def layer(self, il: int) -> Optional[MoELayer]:
        return self._layers.get(il)

    def close(self) -> None:
        if getattr(self, "_h", None):
            for L in self._layers.values():
                L._h = None
            self._layers = {}
            load().dmoe_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def route_static(x, w_router, b_router, hp: dict, idx, weights, stream: Optional[int] = None) -> None:
    """dmoe_route_static: routing with the library's fixed scratch array, for callers that cannot
    allocate device memory. Every argument is a torch CUDA tensor (device memory) owned by the
    caller: x [n, H] f32, w_router [E, H] f32, b_router [E] f32 or None, and the outputs
    idx [n, top_k] int32 and weights [n, top_k] f32. Enqueued on the current torch stream."""
    import torch

    dev = None
    for name, t, dt in (("x", x, torch.float32), ("w_router", w_router, torch.float32),
                        ("b_router", b_router, torch.float32), ("idx", idx, torch.int32),
                        ("weights", weights, torch.float32)):
        if t is None and name == "b_router":
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError(f"route_static: {name} must be a CUDA tensor")
        if dev is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        if t.device != dev:
            raise ValueError(f"route_static: {name} must be a CUDA tensor on the current device {dev}")
        if t.dtype != dt or not t.is_contiguous():
            raise ValueError(f"route_static: {name} must be a contiguous {dt} tensor")
    n = int(x.shape[0])
    if (tuple(x.shape) != (n, hp["n_embd"]) or tuple(w_router.shape) != (hp["n_expert"], hp["n_embd"])
            or tuple(idx.shape) != (n, hp["n_expert_used"]) or tuple(weights.shape) != (n, hp["n_expert_used"])
            or (b_router is not None and tuple(b_router.shape) != (hp["n_expert"],))):
        raise ValueError("route_static: tensor shapes do not match the layer's hyper-parameters")
    if stream is None:
        stream = torch.cuda.current_stream(x.device).cuda_stream
    _check(load().dmoe_route_static(_ptr(x), int(x.shape[0]), hp["n_embd"], _ptr(w_router), _ptr(b_router),
                                    hp["n_expert"], hp["n_expert_used"], hp.get("expert_capacity", 48),
                                    hp.get("moe_block_size", 32), hp.get("routed_scaling", 1.0),
                                    hp.get("norm_topk_prob", 1), _ptr(idx), _ptr(weights), stream if stream else None))


def sample_step(logits, seq, mask_id: int, n_transfer: int, threshold: float, token, prob, n_committed=None,
                stream: Optional[int] = None) -> None:
    """dmoe_sample_step: one greedy denoising step of the block sampler on the GPU
    (src/diffuse-sampler.cpp:29-49,183-237). torch CUDA tensors: logits [n_pos, n_vocab] f32,
    seq [n_pos] int32 (updated in place; None: argmax and probability only), token [n_pos] int32
    and prob [n_pos] f32 (outputs), n_committed [1] int32 or None. Enqueued on the current torch
    stream."""
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(logits.device).cuda_stream
    n_pos, n_vocab = int(logits.shape[0]), int(logits.shape[1])
    _check(load().dmoe_sample_step(_ptr(logits), n_pos, n_vocab, _ptr(seq), mask_id, n_transfer, threshold,
                                   _ptr(token), _ptr(prob), _ptr(n_committed), stream if stream else None))
