"""Expert parallelism through the C ABI on 2 GPUs (one process per GPU, NCCL).

Each rank binds its half of the experts, routes its own token blocks and runs dmoe_forward
collectively. Its output rows must meet the oracle tolerance for its tokens, and its routing
must stay bit-exact (routing is local). A rank that never joins must make the others' create
return DMOE_ERR_TIMEOUT within the deadline instead of hanging. Skipped with fewer than 2 GPUs.
NVLS is off for these child processes.
"""
import os

import numpy as np
import pytest

import diffuse_moe as dm
import oracle
import synth

WORLD = 2


def gpus() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


needs2 = pytest.mark.skipif(gpus() < WORLD, reason="expert parallelism needs 2 GPUs")


def layer_spec(kind: str) -> synth.LayerSpec:
    if kind == "tiny":
        return synth.LayerSpec(H=256, I=256, Is=256, E=16, top_k=4, cap=6, blk=32, expert_type=dm.TYPE_Q4_K, seed=31)
    # S shape with q8_0 (c2-like), 256 experts over 2 ranks
    return synth.LayerSpec(H=2048, I=512, Is=512, E=256, top_k=8, cap=48, blk=32, expert_type=dm.TYPE_Q8_0, seed=32)


def worker(rank, kind, ntok, nccl_id, ret, chunks=4):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["DMOE_EP_CHUNKS"] = str(chunks)  # read by dmoe_create; the same on every rank
    try:
        sp = layer_spec(kind)
        hp = sp.hparams()
        t = synth.make_layer(sp)
        x = synth.make_input(ntok, sp.H, 500 + rank)
        cfg = dm.dist_cfg(rank, WORLD, rank, nccl_id, timeout_ms=60000)
        L = dm.MoELayer(hp, t, dist=cfg)
        out, (idx, w, allowed) = L.forward(x, route=True)
        out2 = L.forward(x)  # a second call reuses the grown buffers and the communicator
        st = L.stats()
        L.close()
        r_out, r_idx, r_w, r_allowed, used = oracle.layer(hp, t, x)
        ok_route = bool(np.array_equal(idx, r_idx) and np.array_equal(w.view(np.uint32), r_w.view(np.uint32)))
        err = float(np.linalg.norm(out.astype(np.float64) - r_out) / np.linalg.norm(r_out))
        err2 = float(np.linalg.norm(out2.astype(np.float64) - r_out) / np.linalg.norm(r_out))
        ret[rank] = (ok_route, err, err2, int(st["ep_rows_sent"]), int(st["ep_rows_received"]))
    except Exception as e:  # reported to the parent
        ret[rank] = ("error", repr(e))


def run_world(kind, ntok, chunks=4):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    nccl_id = dm.nccl_unique_id()
    procs = [ctx.Process(target=worker, args=(r, kind, ntok, nccl_id, ret, chunks)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    return dict(ret)


@pytest.mark.gpu
@needs2
@pytest.mark.parametrize("kind,ntok,chunks", [("tiny", 64, 1), ("tiny", 64, 4), ("tiny", 32, 8), ("s_q8", 256, 1),
                                              ("s_q8", 256, 4)])
def test_ep_two_ranks_match_oracle(kind, ntok, chunks):
    """The exchange pipelined over `chunks` chunks of each rank's tokens (32 tokens in 8 chunks:
    every chunk's NCCL groups run, some with nothing to send) gives the oracle's answer."""
    ret = run_world(kind, ntok, chunks)
    for r in range(WORLD):
        v = ret[r]
        assert v[0] != "error", v
        ok_route, err, err2, sent, recvd = v
        assert ok_route, f"rank {r}: routing differs from the oracle"
        assert err <= 2e-3 and err2 <= 2e-3, (r, err, err2)
        assert sent > 0 and recvd > 0


def lonely_worker(nccl_id, ret):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import time

    sp = layer_spec("tiny")
    t = synth.make_layer(sp)
    cfg = dm.dist_cfg(0, WORLD, 0, nccl_id, timeout_ms=3000)
    t0 = time.time()
    try:
        dm.MoELayer(sp.hparams(), t, dist=cfg)
        ret["status"] = 0
    except dm.DmoeError as e:
        ret["status"] = e.status
        ret["msg"] = str(e)
    ret["seconds"] = time.time() - t0


@pytest.mark.gpu
@needs2
def test_ep_rank_that_never_joins_times_out():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    p = ctx.Process(target=lonely_worker, args=(dm.nccl_unique_id(), ret))  # rank 1 never starts
    p.start()
    p.join(120)
    assert p.exitcode == 0
    assert ret["status"] == 6, ret  # DMOE_ERR_TIMEOUT
    assert ret["seconds"] < 30, ret


def replica_worker(rank, nccl_id, ret):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        # small layer shape, q8_0, Zipf-skewed expert bias: a few experts take most of the slots
        sp = synth.LayerSpec(H=2048, I=512, Is=512, E=256, top_k=8, cap=48, blk=32, expert_type=dm.TYPE_Q8_0,
                             bias="zipf", seed=34)
        hp = sp.hparams()
        t = synth.make_layer(sp)
        x = synth.make_input(512, sp.H, 700 + rank)
        r_out, r_idx, r_w, _, _ = oracle.layer(hp, t, x)
        L = dm.MoELayer(hp, t, dist=dm.dist_cfg(rank, WORLD, rank, nccl_id, timeout_ms=60000))
        res = {}

        def run(tag):
            out, (idx, w, _) = L.forward(x, route=True)
            st = L.stats()
            err = float(np.linalg.norm(out.astype(np.float64) - r_out) / np.linalg.norm(r_out))
            res[tag] = (bool(np.array_equal(idx, r_idx)), err, int(st["ep_rows_sent"]), int(st["ep_rows_received"]))

        run("plain")
        L.replicate_experts(8)                      # the busiest 8 of that forward, over both ranks
        run("auto8")
        load = np.bincount(r_idx.ravel(), minlength=256)
        L.replicate_experts(3, ids=[int(np.argmax(load)), 5, 200])  # explicit ids (same on every rank)
        run("ids3")
        L.replicate_experts(0)                      # replicas dropped
        run("none")
        L.close()
        ret[rank] = res
    except Exception as e:  # reported to the parent
        ret[rank] = ("error", repr(e))


@pytest.mark.gpu
@needs2
def test_ep_hot_expert_replicas():
    """Replicated hot experts leave the results unchanged (oracle bar, routing exact) and take
    their (token, slot) pairs off the exchange: fewer rows cross to the other rank."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    nccl_id = dm.nccl_unique_id()
    procs = [ctx.Process(target=replica_worker, args=(r, nccl_id, ret)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
        assert p.exitcode == 0
    for r in range(WORLD):
        res = ret[r]
        assert isinstance(res, dict), res  # the worker reports ("error", message) on failure
        for tag, (ok, err, sent, recvd) in res.items():
            assert ok, (r, tag)
            assert err <= 2e-3, (r, tag, err)
        # rows sent to the other rank: with the busiest experts local, fewer (token, rank) rows
        assert res["auto8"][2] < res["plain"][2], res
        assert res["none"][2] == res["plain"][2], res


def empty_rank_worker(rank, nccl_id, ret):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        sp = layer_spec("tiny")
        hp = sp.hparams()
        t = synth.make_layer(sp)
        n = 64 if rank == 0 else 0  # rank 1 has no tokens this forward
        x = synth.make_input(max(n, 1), sp.H, 900)[:n]
        L = dm.MoELayer(hp, t, dist=dm.dist_cfg(rank, WORLD, rank, nccl_id, timeout_ms=30000))
        out = L.forward(x)
        out2 = L.forward(x)
        L.close()
        if n:
            r_out = oracle.layer(hp, t, x)[0]
            errs = [float(np.linalg.norm(o.astype(np.float64) - r_out) / np.linalg.norm(r_out)) for o in (out, out2)]
        else:
            errs = [0.0, 0.0] if out.shape == (0, sp.H) else [1.0, 1.0]
        ret[rank] = ("ok", errs)
    except Exception as e:  # reported to the parent
        ret[rank] = ("error", repr(e))


@pytest.mark.gpu
@needs2
def test_ep_rank_without_tokens():
    """A rank with no tokens still takes its part in the exchange (its experts receive the other
    rank's rows), so the forward completes on every rank and the other rank's output is right."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    nccl_id = dm.nccl_unique_id()
    procs = [ctx.Process(target=empty_rank_worker, args=(r, nccl_id, ret)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    for r in range(WORLD):
        status, errs = ret[r]
        assert status == "ok", (r, errs)
        assert max(errs) <= 2e-3, (r, errs)


def model_worker(rank, path, nccl_id, ret):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        from model_gguf import ModelSpec

        ms = ModelSpec(n_layer=3, first_k=1)
        model = dm.MoEModel(path, dist=dm.dist_cfg(rank, WORLD, rank, nccl_id, timeout_ms=60000))
        x = synth.make_input(64, ms.H, 600 + rank)
        res = {}
        for il in range(ms.first_k, ms.n_layer):
            hp = ms.layer_spec(il).hparams()
            t = synth.make_layer(ms.layer_spec(il))
            out, (idx, w, _) = model.layer(il).forward(x, route=True)
            r_out, r_idx, r_w, _, _ = oracle.layer(hp, t, x)
            err = float(np.linalg.norm(out.astype(np.float64) - r_out) / np.linalg.norm(r_out))
            res[il] = (bool(np.array_equal(idx, r_idx)), err, int(model.layer(il).stats()["ep_rows_sent"]))
        model.close()
        ret[rank] = res
    except Exception as e:  # reported to the parent
        ret[rank] = ("error", repr(e))


@pytest.mark.gpu
@needs2
def test_ep_model_load(tmp_path):
    """A GGUF model loaded on both ranks (dmoe_model_load with dist): the first MoE layer's
    communicator from the unique id, the next one's split from it; every layer exchanges rows
    and matches the oracle."""
    import torch.multiprocessing as mp

    from model_gguf import ModelSpec, write_model

    path = str(tmp_path / "m.gguf")
    write_model(path, ModelSpec(n_layer=3, first_k=1))
    ctx = mp.get_context("spawn")
    ret = ctx.Manager().dict()
    nccl_id = dm.nccl_unique_id()
    procs = [ctx.Process(target=model_worker, args=(r, path, nccl_id, ret)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
        assert p.exitcode == 0
    for r in range(WORLD):
        res = ret[r]
        assert isinstance(res, dict), res
        for il, (ok, err, sent) in res.items():
            assert ok, (r, il)
            assert err <= 2e-3, (r, il, err)
            assert sent > 0, (r, il)
