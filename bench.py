"""Benchmark of the block-routed MoE layer (the metric of BASELINE.json: MoE-layer tokens/s and
HBM GB/s, 256 experts, top-8, q4_K, at 1/2/4/8 B200).

Workload: the LLaDA2.2-flash-shaped layer (hidden 4096, 256 routed SwiGLU experts of width 1024,
one shared expert of width 1024, fp32 router, capacity 48 per 32-token block, top-8, x2.5) with
q4_K weights quantised from F16 ~N(0, 0.02), on 256 blocks x 32 tokens of RMS-normalised
N(0, 1) inputs per GPU (synthetic: no dataset exists for this path). The weights (1.8 GB) and
the per-step activations exceed the 126 MB L2, so no extra flush is needed between steps.

One step = one dmoe_forward over the GPU's 8192 tokens. `value` is device-resident throughput
(inputs already in HBM); `e2e` goes through the public C ABI with pinned host buffers (H2D of x,
D2H of out inside the timed region). With N > 1 (torchrun) the layer is expert-parallel: rank r
holds experts [256 r / N, 256 (r + 1) / N), routes its own 256 blocks and exchanges token rows and
partial outputs with the other ranks over NCCL inside every step (weak scaling: 8192 tokens per
GPU); the timing is the max over ranks. N > 1 also reports `c4`: the c4 workload of BASELINE.json
(16384 tokens in total, Zipf-skewed expert bias, expert-parallel over the N GPUs), as a strong-
scaling measurement with per-rank expert loads.

`--impl reference` times the reference's CPU algorithm on the host cores instead: the ggml CPU
path cannot be built (its ggml submodule is empty), so this is the oracle's ggml-faithful C
restatement (weights in their GGUF blocks, activations rounded to Q8_K, AVX2 integer dot products,
OpenMP on every host thread), each step a sample of the workload's blocks sized to fit a few
minutes (the whole step when it fits).

Besides the headline, the line carries `configs`: device-resident lines for the configs c1
(small layer, F16 weights, 1 block) and c2 (small layer, q8_0 weights, 64 blocks) of BASELINE.json,
each with its HBM GB/s and fraction of the layer roofline; and `c5`: the whole-model generation of
config 5 around these layers (bench_c5).
"""
from __future__ import annotations

import argparse
import json
import os
import signal
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "diffuse-cpp_b200"))

import numpy as np  # noqa: E402

METRIC = "moe_layer_tokens_per_s"
UNIT = "tokens/s"


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def load_traffic(key: str):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(key)
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.send_signal(signal.SIGTERM)
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [c.strip() for c in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def algorithmic(spec, n_tokens: int, n_active: int):
    import synth

    B = (n_active * synth.expert_bytes(spec) + synth.shared_bytes(spec) + 4 * spec.H * spec.E + 4 * spec.E
         + 8 * n_tokens * spec.H)
    F = n_tokens * synth.flops_per_token(spec)
    gateup_flops = n_tokens * (spec.top_k * 4 * spec.H * spec.I + 4 * spec.H * spec.Is)
    return B, F, gateup_flops


def run_cpu_reference(spec, t, n_tokens: int, steps: int, warmup: int, budget_s: float):
    """Times the reference's algorithm on the host cores: the oracle's ggml-faithful mode (the
    ggml CPU path itself cannot be built: its submodule is empty). Weights stay in their GGUF
    blocks, activations are rounded to the weight type's vec-dot type (Q8_K for q4_K) and every
    dot product is an AVX2 integer block product, on all host threads; the router and the
    routing run as in the reference. Each step is one call on a sample of the workload's routing
    blocks, sized from a 4-block calibration call so that warmup + steps fit in budget_s (the
    whole 256-block step when it fits). Returns (tokens_per_s, cores, sample, ms_per_step, blocks)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # CPU baseline leg only
    import synth

    cores = os.cpu_count() or 1
    hp = spec.hparams()
    x4 = synth.make_input(128, spec.H, spec.seed + 1000)
    oracle.layer(hp, t, x4, mode=oracle.MODE_GGML, nthreads=cores)  # page the weights in
    t0 = time.perf_counter()
    oracle.layer(hp, t, x4, mode=oracle.MODE_GGML, nthreads=cores)
    per_block = (time.perf_counter() - t0) / 4
    max_blocks = n_tokens // 32
    blocks = int(max(1, min(max_blocks, budget_s / max(1, steps + warmup) / per_block)))
    x = synth.make_input(32 * blocks, spec.H, spec.seed + 1001)
    for _ in range(warmup):
        oracle.layer(hp, t, x, mode=oracle.MODE_GGML, nthreads=cores)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        oracle.layer(hp, t, x, mode=oracle.MODE_GGML, nthreads=cores)
        times.append(time.perf_counter() - t0)
    mean_s = float(np.mean(times))
    tps = 32 * blocks / mean_s
    sample = (f"{steps} timed steps (+{warmup} warm-up) of {blocks} of the workload's {max_blocks} routing blocks "
              f"({32 * blocks} tokens) each, {mean_s:.2f} s per step; ggml-faithful CPU restatement "
              f"(q8_K activations, AVX2 integer dots), {cores} threads")
    return tps, cores, sample, mean_s * 1e3, blocks


def bench_sampler(dev, stream, peaks_hbm: float, no_cpu: bool) -> dict:
    """One block of 32 masked positions over the flash-model vocabulary (157,184): 8 logits
    buffers in rotation (160 MB > L2), a fresh all-masked seq per step, 40 steps captured in one
    CUDA graph and replayed (a host loop of ctypes calls, ~20 us each, would leave the GPU
    waiting between steps)."""
    import torch

    import diffuse_moe as dm

    V, P, NB, reps = 157184, 32, 8, 40
    gen = torch.Generator(device=dev).manual_seed(7)
    lbufs = [torch.randn((P, V), device=dev, generator=gen) * 3 for _ in range(NB)]
    seqs = torch.full((reps + 5, P), 156895, dtype=torch.int32, device=dev)  # every position masked
    tok = torch.empty(P, dtype=torch.int32, device=dev)
    prb = torch.empty(P, dtype=torch.float32, device=dev)
    for i in range(5):
        dm.sample_step(lbufs[i % NB], seqs[reps + i], 156895, 2, 0.95, tok, prb)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for i in range(reps):
                dm.sample_step(lbufs[i % NB], seqs[i], 156895, 2, 0.95, tok, prb)
    stream.wait_stream(side)
    seqs.fill_(156895)
    graph.replay()  # warm-up replay
    seqs.fill_(156895)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / reps * 1e3
    del graph
    sbytes = P * V * 4
    sampler = {"workload": "32 masked positions x 157184 logits (one LLaDA2 block), greedy, n_transfer 2, "
                           "threshold 0.95", "us_per_step": us, "bytes": sbytes,
               "hbm_gbs": sbytes / (us / 1e6) / 1e9, "frac": sbytes / (us / 1e6) / 1e9 / peaks_hbm,
               "kernels_per_step": 2, "timing": "CUDA-graph replay of 40 steps, CUDA events"}
    if not no_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle  # CPU baseline leg only

        lg = lbufs[0].cpu().numpy()
        t0 = time.perf_counter()
        for _ in range(3):
            oracle.sample_step(lg, np.full(P, 156895, np.int32), 156895, 2, 0.95)
        sampler["cpu_baseline"] = {"us_per_step": (time.perf_counter() - t0) / 3 * 1e6, "cores": os.cpu_count(),
                                   "kind": "port"}
    del lbufs
    return sampler


def bench_c5(layer_tensors: dict, spec, steps: int = 8) -> dict:
    """a LLaDA2.2-flash-shaped 32-block model (block 0 dense SwiGLU I = 9216,
    blocks 1-31 the c3 MoE layer, hidden 4096, 32 / 4 heads of 128, vocab 157184) with random
    weights generates 256 tokens after a 480-token random prompt in 32-token blocks, 8 denoising
    steps per block committing the 4 most confident positions (and any at >= 0.95). The MoE layers
    and the sampler step are this library's kernels; attention, dense projections and lm_head
    are torch library calls on bf16 weights. The 31 MoE layers are 31 device copies of one
    synthetic q4_K weight set. `value` = generated tokens / wall time of the generation (the
    model's forwards, sampler steps and the per-step host read of the commit count) with the
    key/value cache and each step's forward replayed from a CUDA graph; the cache without graphs
    and the reference's whole-window recompute at every step are timed beside it."""
    import torch

    import diffuse_moe as dm
    import llada2

    cfg = llada2.LLaDA2Config()
    moe = {il: dm.MoELayer(spec.hparams(), layer_tensors) for il in range(cfg.first_k_dense, cfg.n_layer)}
    w = llada2.LLaDA2Model.random_weights(cfg, seed=11)
    w["output"][cfg.mask_token_id] = 0.0
    model = llada2.LLaDA2Model(cfg, w, moe, dtype=torch.bfloat16)
    del w
    prompt = np.random.default_rng(5).integers(0, cfg.mask_token_id, size=480)
    out = {"workload": "config 5: 32 blocks (1 dense + 31 MoE c3 q4_K), 480-token prompt + 256 generated, "
                       "32-token blocks, 8 steps committing top-4 (threshold 0.95)", "generated": 256}
    model.reserve(480 + 256)
    for name, cache, graphs in (("kv_cache_graphs", True, True), ("kv_cache", True, False),
                                ("recompute_window", False, False)):
        # warm-up on the same prompt (the same prefill; the graphs are captured here)
        llada2.generate(model, prompt, 64, steps=steps, threshold=0.95, use_cache=cache, graphs=graphs)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        seq, nf = llada2.generate(model, prompt, 256, steps=steps, threshold=0.95, use_cache=cache, graphs=graphs)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        out[name] = {"seconds": dt, "tokens_per_s": 256 / dt, "forwards": nf, "ms_per_forward": dt / nf * 1e3,
                     "masked_left": int(np.sum(seq == cfg.mask_token_id))}
    out["value"] = out["kv_cache_graphs"]["tokens_per_s"]
    out["unit"] = "generated tokens/s"
    model.drop_graphs()
    for L in moe.values():
        L.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--blocks", type=int, default=256, help="32-token routing blocks per GPU")
    ap.add_argument("--config", default="c3")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-c5", action="store_true", help="skip the full-model (config 5) generation leg")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    import synth

    spec = synth.config(args.config)
    n_tok = 32 * args.blocks
    cfg = {"workload": f"{args.config}: flash-shaped MoE layer H4096 E256 I1024 Is1024 top8 cap48 q4_K, "
                       f"{args.blocks} blocks x 32 tokens per GPU",
           "tokens_per_gpu": n_tok, "global_tokens": n_tok * args.gpus, "weights": "q4_K (synthetic F16 N(0,0.02))",
           "l2": "working set > L2 (1.8 GB weights), no flush",
           "parallelism": "single GPU" if args.gpus == 1 else
           f"expert-parallel x{args.gpus} ({256 // args.gpus} experts per GPU, NCCL dispatch/combine), token blocks sharded"}

    if args.impl == "reference":
        if rank != 0:
            return
        t = synth.make_layer(spec)
        tps, cores, sample, ms_step, blocks = run_cpu_reference(spec, t, n_tok, args.steps, args.warmup,
                                                                budget_s=150.0)
        line = {"metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "q8_K x q4_K int8 dots, f32", "data": "synthetic",
                "config": dict(cfg, reference_step=f"{blocks} of {n_tok // 32} blocks per step ({32 * blocks} tokens)"),
                "impl": "reference",
                "cpu_baseline": {"value": tps, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
                "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "note": "ggml CPU path unbuildable here (empty ggml submodule); oracle/ ggml-faithful C "
                        "restatement (weights in GGUF blocks, activations rounded to the vec-dot type, AVX2 integer "
                        "dot products, OpenMP); ms_per_step is the time of one sampled step"}
        print(json.dumps(line))
        return

    import torch
    import torch.distributed as dist

    import diffuse_moe as dm

    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    peaks = load_peaks()
    hp = spec.hparams()
    t = synth.make_layer(spec)
    dev = torch.device("cuda", local_rank)
    nccl_id = None
    if world > 1:
        # one NCCL unique id from rank 0 for the layer's own communicator
        idt = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            idt.copy_(torch.frombuffer(bytearray(dm.nccl_unique_id()), dtype=torch.uint8).to(dev))
        dist.broadcast(idt, 0)
        nccl_id = bytes(idt.cpu().numpy().tobytes())

    def make(sp, tt):
        return dm.MoELayer(sp.hparams(), tt, dist=dm.dist_cfg(rank, world, local_rank, nccl_id, timeout_ms=120000))

    layer = make(spec, t)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        tt = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    def time_layer(L, sp, n: int, steps: int, warmup: int, profile_pass: bool = True):
        x = torch.from_numpy(synth.make_input(n, sp.H, sp.seed + 17 * rank)).to(dev)
        out = torch.empty((n, sp.H), dtype=torch.float32, device=dev)
        for _ in range(warmup):
            L.forward(x, out=out)
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(steps):
            L.forward(x, out=out)
        ev1.record(stream)
        barrier()
        ms = ev0.elapsed_time(ev1) / steps
        L.sync()
        st = L.stats()
        prof = None
        if profile_pass:  # per-stage CUDA events on the launching stream (separate, untimed pass)
            stages = []
            for _ in range(max(3, min(steps, 10))):
                L.forward(x, out=out, profile=True)
                L.sync()
                stages.append(L.stats())
            prof = {k: float(np.median([s[k] for s in stages])) for k in
                    ("ms_router", "ms_dispatch", "ms_gateup", "ms_down", "ms_total")}
        return max_over_ranks(ms), st, prof

    def time_device(n: int, steps: int, warmup: int, profile_pass: bool = True):
        return time_layer(layer, spec, n, steps, warmup, profile_pass)

    def roof_entry(sp, n, ms, st, prof):
        B, F, _ = algorithmic(sp, n, st["n_active"])
        t_roof = max(B / (peaks_hbm * 1e9), F / (peaks["bf16_tflops"] * 1e12))
        return {"tokens": n, "ms": ms, "tokens_per_s": n / (ms / 1e3), "hbm_gbs": B / (ms / 1e3) / 1e9,
                "tflops": F / (ms / 1e3) / 1e12, "n_active": st["n_active"], "roofline_frac": t_roof / (ms / 1e3),
                "bound": "hbm" if B / (peaks_hbm * 1e9) >= F / (peaks["bf16_tflops"] * 1e12) else "tensor",
                "bytes": B, "flops": F, "stages_ms": prof, "token_tile": st["token_tile"],
                "fused_gemm": st["fused_gemm"]}

    peaks_hbm = peaks["hbm_gbs"]
    sweep = []
    if not args.no_sweep and world == 1:
        for nb in (1, 8, 64):
            n = 32 * nb
            ms, st, prof = time_device(n, max(args.steps, 20), args.warmup)
            B, F, _ = algorithmic(spec, n, st["n_active"])
            t_roof = max(B / (peaks_hbm * 1e9), F / (peaks["bf16_tflops"] * 1e12))
            sweep.append({"blocks": nb, "tokens": n, "ms": ms, "tokens_per_s": n / (ms / 1e3),
                          "hbm_gbs": B / (ms / 1e3) / 1e9, "tflops": F / (ms / 1e3) / 1e12,
                          "n_active": st["n_active"], "roofline_frac": t_roof / (ms / 1e3),
                          "bound": "hbm" if B / (peaks_hbm * 1e9) >= F / (peaks["bf16_tflops"] * 1e12) else "tensor",
                          "stages_ms": prof, "token_tile": st["token_tile"], "ksplit": [st["ksplit_gateup"],
                                                                                        st["ksplit_down"]]})

    # ---- configs c1 (F16, 1 block) and c2 (q8_0, 64 blocks) of the small layer shape
    configs = None
    if not args.no_sweep and world == 1:
        configs = {}
        for cname, nb, what in (("c1", 1, "small layer H2048 E256 I512 Is512, F16 weights, 1 block x 32 tokens"),
                                ("c2", 64, "small layer H2048 E256 I512 Is512, q8_0 weights, 64 blocks x 32 tokens")):
            sp = synth.config(cname)
            Lc = dm.MoELayer(sp.hparams(), synth.make_layer(sp))
            ms_c, st_c, prof_c = time_layer(Lc, sp, 32 * nb, max(args.steps, 20), args.warmup)
            configs[cname] = dict(roof_entry(sp, 32 * nb, ms_c, st_c, prof_c), workload=what)
            Lc.close()
            del Lc

    # ---- headline: device-resident throughput on this GPU's token shard
    with ClockSampler(torch.cuda.current_device()) as cs:
        ms, st, prof = time_device(n_tok, args.steps, args.warmup)
    clocks = cs.summary()
    B, F, gu_flops = algorithmic(spec, n_tok, st["n_active"])
    value = n_tok * world / (ms / 1e3)

    # ---- e2e through the public API with pinned host buffers
    xh = torch.from_numpy(synth.make_input(n_tok, spec.H, spec.seed + 17 * rank)).pin_memory().numpy()
    oh = torch.empty((n_tok, spec.H), dtype=torch.float32).pin_memory().numpy()
    for _ in range(args.warmup):
        layer.forward(xh, out=oh)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        layer.forward(xh, out=oh)
    e2e_s = max_over_ranks((time.perf_counter() - t0) / args.steps)
    e2e = {"value": n_tok * world / e2e_s, "unit": UNIT, "h2d_bytes_per_step": int(xh.nbytes),
           "d2h_bytes_per_step": int(oh.nbytes), "ms_per_step": e2e_s * 1e3}

    # ---- roofline of the dominant kernel (gate/up grouped GEMM: 2/3 of the layer's flops); it is
    # timed inside steps of a few ms, so against the burst (not the seconds-long sustained) peak
    gu_ms = prof["ms_gateup"]
    achieved = gu_flops / (gu_ms / 1e3) / 1e12
    peak = peaks["bf16_tflops"]
    roofline = {"kernel": "moe_gemm_kernel<q4_K, gate/up>", "bound": "tensor", "achieved": achieved, "peak": peak,
                "unit": "TFLOP/s", "frac": achieved / peak, "traffic": load_traffic(f"gateup_{args.blocks}blk"),
                "peak_source": f"{peaks['source']} bf16 burst",
                "algorithmic_flops_per_launch": gu_flops, "launch_ms": gu_ms}
    t_roof = max(B / (peaks_hbm * 1e9), F / (peaks["bf16_tflops"] * 1e12))
    layer_roof = {"bytes": B, "flops": F, "hbm_gbs": B / (ms / 1e3) / 1e9, "tflops": F / (ms / 1e3) / 1e12,
                  "frac": t_roof / (ms / 1e3), "peak_source": peaks["source"],
                  # the same bound with the 8 TB/s HBM3e specification instead of the measured copy rate
                  "frac_hbm_spec_8tbs": max(B / 8.0e12, F / (peaks["bf16_tflops"] * 1e12)) / (ms / 1e3)}

    # ---- c4 (N > 1): 16384 tokens in total, Zipf-skewed bias, expert-parallel (strong scaling)
    c4 = None
    if world > 1:
        layer.close()
        del t
        sp4 = synth.config("c4")
        t4 = synth.make_layer(sp4)
        nid = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            nid.copy_(torch.frombuffer(bytearray(dm.nccl_unique_id()), dtype=torch.uint8).to(dev))
        dist.broadcast(nid, 0)
        nccl_id = bytes(nid.cpu().numpy().tobytes())
        layer = make(sp4, t4)
        n4 = 16384 // world
        x4 = torch.from_numpy(synth.make_input(n4, sp4.H, sp4.seed + 17 * rank)).to(dev)
        o4 = torch.empty((n4, sp4.H), dtype=torch.float32, device=dev)
        for _ in range(args.warmup):
            layer.forward(x4, out=o4)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            layer.forward(x4, out=o4)
        e1.record(stream)
        barrier()
        ms4 = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        layer.sync()
        st4 = layer.stats()

        def rows_per_rank(st_):
            loads = torch.tensor([float(st_["ep_rows_received"])], device=dev)
            allv = [torch.zeros_like(loads) for _ in range(world)]
            dist.all_gather(allv, loads)
            return [int(v.item()) for v in allv]

        rows4 = rows_per_rank(st4)
        # NVLink term of the expert-parallel roofline: every received row arrives as fp16 (2 B per
        # hidden unit) and returns as an fp32 partial (4 B), against the measured 770 GB/s peer copy
        # per direction (the busiest rank bounds the step; its own rows are included)
        nvl = max(rows4) * sp4.H * 6
        c4 = {"tokens": 16384, "ms_per_step": ms4, "tokens_per_s": 16384 / (ms4 / 1e3),
              "rows_received_per_rank": rows4, "scaling": "strong",
              "bias": "0.5 log Zipf(1.1) over a random expert permutation",
              "nvlink_bytes_busiest_rank": nvl, "nvlink_bound_ms": nvl / 770e9 * 1e3}
        # the same workload with the busiest experts of the last forward replicated on every rank
        # (dmoe_replicate_experts): their (token, slot) pairs stay on the token's rank
        n_hot = 16
        layer.replicate_experts(n_hot)
        for _ in range(args.warmup):
            layer.forward(x4, out=o4)
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            layer.forward(x4, out=o4)
        e1.record(stream)
        barrier()
        ms4r = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        layer.sync()
        c4["replicated"] = {"n_hot": n_hot, "ms_per_step": ms4r, "tokens_per_s": 16384 / (ms4r / 1e3),
                            "rows_received_per_rank": rows_per_rank(layer.stats())}

    # ---- sampler step (dmoe_sample_step): one block of 32 masked positions over the flash-model
    # vocabulary; a secondary measurement, so a failure there is reported in its object instead
    # of costing the layer's line
    sampler = None
    if rank == 0 and world == 1:
        try:
            sampler = bench_sampler(dev, stream, peaks_hbm, args.no_cpu)
        except Exception as ex:  # noqa: BLE001
            sampler = {"error": f"{type(ex).__name__}: {ex}"}

    # ---- config 5: the whole model's generation around these layers (secondary, like the sampler)
    c5 = None
    if rank == 0 and world == 1 and not args.no_c5 and args.config == "c3":
        try:
            c5 = bench_c5(t, spec)
        except Exception as ex:  # noqa: BLE001
            c5 = {"error": f"{type(ex).__name__}: {ex}"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        tps, cores, sample, _, _ = run_cpu_reference(spec, t, n_tok, 3, 1, budget_s=20.0)
        cpu = {"value": tps, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16",
                "precision": "q4_K weights dequantised to fp16, fp16 activations, fp32 accumulation",
                "data": "synthetic", "config": cfg, "e2e": e2e, "roofline": roofline, "layer_roofline": layer_roof,
                "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": int(st["kernels"]) * args.steps,
                "stages_ms": prof, "n_active": st["n_active"], "token_tile": st["token_tile"],
                "ksplit": [st["ksplit_gateup"], st["ksplit_down"]], "sweep": sweep}
        if c4 is not None:
            line["c4"] = c4
        if configs:
            line["configs"] = configs
        if sampler is not None:
            line["sampler"] = sampler
        if c5 is not None:
            line["c5"] = c5
        print(json.dumps(line))
    layer.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
