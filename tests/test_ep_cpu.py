"""Expert parallelism on CPU: the decomposition the library's EP path implements (ep.cu), run
with real collectives (torch.distributed gloo, world size 2 and 4) around the oracle.

Each rank routes its own whole token blocks, sends one row per (token, owning rank) with its
slot list (rank-local expert id or -1, gate weight), computes the weighted partial rows of its
own experts only (it is given only their weights), returns them, and the owner adds the
partials in rank order to its shared-expert rows. The result must equal the single-process
layer (oracle, double accumulation) on the same tokens, and routing needs no communication.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import diffuse_moe as dm
import oracle
import synth

def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def spec():
    return synth.LayerSpec(H=256, I=256, Is=256, E=8, top_k=3, cap=4, blk=32, expert_type=dm.TYPE_Q8_0, seed=21)


def local_tensors(t, hp, rank, world, hot=()):
    """This rank's expert slice of each [E][rows][k] GGUF tensor (what dmoe_create uploads),
    followed by the replicated hot experts (what dmoe_replicate_experts adds)."""
    el = hp["n_expert"] // world
    out = {}
    for name, rows in (("w_gate", hp["n_ff_exp"]), ("w_up", hp["n_ff_exp"]), ("w_down", hp["n_embd"])):
        a = np.asarray(t[name])
        per = a.shape[0] // hp["n_expert"]
        assert per == rows
        parts = [a[rank * el * per:(rank + 1) * el * per]] + [a[e * per:(e + 1) * per] for e in hot]
        out[name] = np.concatenate(parts)
    return out


def exchange(objs_by_dest):
    """all-to-all of python objects over gloo: returns the list received from each source."""
    world = dist.get_world_size()
    gathered = [None] * world
    dist.all_gather_object(gathered, objs_by_dest)
    me = dist.get_rank()
    return [gathered[src][me] for src in range(world)]


def worker(rank, world, port, ret, chunks=1, hot=()):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sp = spec()
        hp = sp.hparams()
        t = synth.make_layer(sp)
        E, K, el = hp["n_expert"], hp["n_expert_used"], hp["n_expert"] // world
        x = synth.make_input(64, sp.H, 100 + rank)  # this rank's 2 blocks
        # local routing (no communication)
        lg = oracle.logits(x, t["w_router"])
        idx, w, _, _, _ = oracle.route(lg, t["b_router"], K, hp["expert_capacity"], hp["moe_block_size"],
                                       hp["norm_topk_prob"], hp["routed_scaling"])
        # plan: one row per (token, computing rank), slot list with local ids (-1 elsewhere); a
        # slot whose expert is replicated on every rank (hot) is computed here, at local id
        # el + its replica index (the library's slot_dest)
        hot = list(hot)

        def dest(e):
            return (rank, el + hot.index(e)) if e in hot else (e // el, e - (e // el) * el)

        sends = [[] for _ in range(world)]
        for tok in range(x.shape[0]):
            ds = [dest(int(e)) for e in idx[tok]]
            for d in sorted({r for r, _ in ds}):
                slots = [(le if r == d else -1, float(w[tok, s])) for s, (r, le) in enumerate(ds)]
                sends[d].append((tok, x[tok], slots))
        # the exchange pipelined over chunks of this rank's tokens (the library's ep_chunks): every
        # chunk's dispatch, then every chunk's partials and combine, in chunk order on all ranks
        lt = local_tensors(t, hp, rank, world, hot)
        hp_l = dict(hp, n_expert=el + len(hot), n_ff_shexp=0)
        n = x.shape[0]
        bounds = [(n * c // chunks, n * (c + 1) // chunks) for c in range(chunks)]
        in_chunk = [[[(tok, xr_, sl) for tok, xr_, sl in sends[d] if lo <= tok < hi] for d in range(world)]
                    for lo, hi in bounds]
        recvs = [exchange([[(x_row, slots) for _, x_row, slots in cs[d]] for d in range(world)]) for cs in in_chunk]
        shared = oracle.experts(hp, t, x, np.zeros_like(idx), np.zeros_like(w), mode=0)
        acc = np.zeros_like(shared)
        for c, recv in enumerate(recvs):
            parts = []  # partial rows with only this rank's experts
            for src in range(world):
                rows = recv[src]
                if not rows:
                    parts.append(np.zeros((0, sp.H), np.float32))
                    continue
                xr = np.stack([r[0] for r in rows]).astype(np.float32)
                li = np.array([[max(e, 0) for e, _ in r[1]] for r in rows], dtype=np.int32)
                lw = np.array([[wv if e >= 0 else 0.0 for e, wv in r[1]] for r in rows], dtype=np.float32)
                parts.append(oracle.experts(hp_l, lt, xr, li, lw, mode=0))
            back = exchange(parts)
            # owner: partials of the chunk's tokens in rank order
            for d in range(world):
                for j, (tok, _, _) in enumerate(in_chunk[c][d]):
                    acc[tok] += back[d][j]
        out = acc + shared
        ref = oracle.layer(hp, t, x, mode=0)[0]
        err = float(np.linalg.norm(out - ref) / np.linalg.norm(ref))
        ret[rank] = err
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world,chunks,hot", [(2, 1, ()), (2, 3, ()), (2, 2, (0, 5, 6)), (4, 1, ()),
                                              (4, 2, (1, 2, 7))])
def test_expert_parallel_decomposition_gloo(world, chunks, hot):
    """chunks: the exchange pipelined over chunks of each rank's tokens; hot: experts replicated
    on every rank (owned by different ranks), whose slots are computed locally."""
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    mp.start_processes(worker, args=(world, free_port(), ret, chunks, hot), nprocs=world, start_method="spawn")
    assert sorted(ret.keys()) == list(range(world))
    for r in range(world):
        assert ret[r] < 1e-5, (r, ret[r])
