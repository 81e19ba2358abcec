"""CPU model of the grouped-GEMM kernel's mbarrier protocol (moe_gemm.cu, moe_gemm_kernel).

Every role is a step machine that waits for an absolute completion count of a barrier and
arrives on others, exactly as the kernel's producer, MMA issuer, epilogue and dequant warps do.
The hardware only compares parities, which is correct only while the barrier's phase is the
needed completion or the one before it; the model flags any wait evaluated outside that window
(aliasing) and any state where no role can move (deadlock), over randomised interleavings.
It covers every configuration the launcher can instantiate (the TMEM/smem budget formulas of
GemmCfg are restated below) and checks that an unsafe ring (fewer A buffers than dequant
warpgroups) is caught.
"""
import itertools
import random

import pytest

F16, Q8_0, Q4_K = 1, 8, 12
GATEUP, DOWN = 0, 1


def gemm_cfg(wt, mode, nt, ndq, pair=False):
    """Restates GemmCfg<WT, MODE, NT, NDQ, PAIR> (stage ring, TMEM ring) from moe_gemm.cu."""
    quant = wt != F16
    mats = 2 if (mode == GATEUP or nt <= 64) else 1  # down at NT <= 64: two 128-row blocks
    stage_k = 256 if wt == Q4_K else 128
    ak = 64 if (pair and quant) else 128  # K per A block (dequant hand-off): 64 for CTA pairs
    kb = stage_k // ak
    b_bytes = stage_k * (nt // 2 if pair else nt) * 2  # a pair's CTA loads half the token rows
    w_bytes = 128 * 144 if wt == Q4_K else (128 * 128 + 128 * 16 if wt == Q8_0 else 128 * 128 * 2)
    stage_bytes = b_bytes + mats * w_bytes
    stages = min(6, (227 * 1024 - 2048) // stage_bytes)
    acc_cols = mats * nt
    a_cols = mats * ak // 2
    acc_bufs = 2 if 2 * acc_cols + (2 * a_cols if quant else 0) <= 512 else 1
    na = min(4, (512 - acc_bufs * acc_cols) // a_cols) if quant else 0
    ndq = ndq if quant else 0
    return dict(stages=stages, na=na, ndq=ndq, kb=kb, acc_bufs=acc_bufs, quant=quant,
                ring_ok=(not quant) or na >= ndq)


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.phase = name, count, count, 0

    def arrive(self):
        self.pending -= 1
        assert self.pending >= 0, f"{self.name}: more arrivals than the count"
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count


def roles(cfg, tiles):
    S, NA, NDQ, KB, ACCB = cfg["stages"], max(cfg["na"], 1), cfg["ndq"], cfg["kb"], cfg["acc_bufs"]
    quant = cfg["quant"]
    full = [Bar(f"full{i}", 1) for i in range(S)]
    empty = [Bar(f"empty{i}", 1 + 4 * NDQ) for i in range(S)]
    afull = [Bar(f"afull{i}", 4) for i in range(NA)]
    aempty = [Bar(f"aempty{i}", 1) for i in range(NA)]
    accfull = [Bar(f"accfull{i}", 1) for i in range(ACCB)]
    accempty = [Bar(f"accempty{i}", 4) for i in range(ACCB)]

    def producer():
        seq = 0
        for t in tiles:
            for _ in range(t):
                s = seq % S
                yield empty[s], seq // S
                full[s].arrive()  # the stage's TMA transactions complete
                seq += 1

    def mma():
        seq = tseq = 0
        for t in tiles:
            ab = tseq % ACCB
            yield accempty[ab], tseq // ACCB
            for _ in range(t):
                s = seq % S
                yield full[s], seq // S + 1
                for kb in range(KB):
                    if quant:
                        kbs = seq * KB + kb
                        a, u = kbs % NA, kbs // NA
                        yield afull[a], u + 1
                        aempty[a].arrive()  # tcgen05.commit after the k-block's MMAs
                empty[s].arrive()
                seq += 1
            accfull[ab].arrive()
            tseq += 1

    def epilogue():
        tseq = 0
        for t in tiles:
            ab = tseq % ACCB
            yield accfull[ab], tseq // ACCB + 1
            accempty[ab].arrive()
            tseq += 1

    def dequant(g):
        seq = 0
        for t in tiles:
            for _ in range(t):
                s = seq % S
                yield full[s], seq // S + 1
                for kb in range(KB):
                    kbs = seq * KB + kb
                    if kbs % NDQ != g:
                        continue
                    a, u = kbs % NA, kbs // NA
                    yield aempty[a], u
                    afull[a].arrive()
                empty[s].arrive()
                seq += 1

    rs = [producer(), mma()] + [epilogue() for _ in range(4)]
    rs += [dequant(g) for g in range(NDQ) for _ in range(4)]
    return rs


def roles_pair(cfg, tiles):
    """The CTA pair (PAIR = true): each CTA runs a producer, its dequant warpgroups and its
    epilogue; the leader's MMA warp alone issues. Arrivals that cross the pair: both producers'
    activation halves on the leader's full_b, both CTAs' dequant warps on the leader's afull, both
    epilogues on the leader's accempty; the leader's commits arrive on aempty / empty / accfull
    of both CTAs."""
    S, NA, NDQ, KB, ACCB = cfg["stages"], max(cfg["na"], 1), cfg["ndq"], cfg["kb"], cfg["acc_bufs"]
    cta = []
    for r in range(2):
        cta.append(dict(
            full=[Bar(f"full{i}.{r}", 1) for i in range(S)],
            empty=[Bar(f"empty{i}.{r}", 1 + 4 * NDQ) for i in range(S)],
            aempty=[Bar(f"aempty{i}.{r}", 1) for i in range(NA)],
            accfull=[Bar(f"accfull{i}.{r}", 1) for i in range(ACCB)],
        ))
    full_b = [Bar(f"full_b{i}", 2) for i in range(S)]  # both halves' bytes (leader's barrier)
    afull = [Bar(f"afull{i}", 8) for i in range(NA)]
    accempty = [Bar(f"accempty{i}", 8) for i in range(ACCB)]

    def producer(r):
        seq = 0
        for t in tiles:
            for _ in range(t):
                s = seq % S
                yield cta[r]["empty"][s], seq // S
                cta[r]["full"][s].arrive()  # this CTA's weight tile
                full_b[s].arrive()          # this CTA's activation half, counted by the leader
                seq += 1

    def mma():
        seq = tseq = 0
        for t in tiles:
            ab = tseq % ACCB
            yield accempty[ab], tseq // ACCB
            for _ in range(t):
                s = seq % S
                yield full_b[s], seq // S + 1
                for kb in range(KB):
                    kbs = seq * KB + kb
                    a, u = kbs % NA, kbs // NA
                    yield afull[a], u + 1
                    for r in range(2):
                        cta[r]["aempty"][a].arrive()
                for r in range(2):
                    cta[r]["empty"][s].arrive()
                seq += 1
            for r in range(2):
                cta[r]["accfull"][ab].arrive()
            tseq += 1

    def epilogue(r):
        tseq = 0
        for t in tiles:
            ab = tseq % ACCB
            yield cta[r]["accfull"][ab], tseq // ACCB + 1
            accempty[ab].arrive()
            tseq += 1

    def dequant(r, g):
        seq = 0
        for t in tiles:
            for _ in range(t):
                s = seq % S
                yield cta[r]["full"][s], seq // S + 1
                for kb in range(KB):
                    kbs = seq * KB + kb
                    if kbs % NDQ != g:
                        continue
                    a, u = kbs % NA, kbs // NA
                    yield cta[r]["aempty"][a], u
                    afull[a].arrive()
                cta[r]["empty"][s].arrive()
                seq += 1

    rs = [mma()]
    for r in range(2):
        rs += [producer(r)] + [epilogue(r) for _ in range(4)]
        rs += [dequant(r, g) for g in range(NDQ) for _ in range(4)]
    return rs


def run(cfg, tiles, seed, pair=False):
    rng = random.Random(seed)
    rs = roles_pair(cfg, tiles) if pair else roles(cfg, tiles)
    cur = [None] * len(rs)
    alive = set(range(len(rs)))
    while alive:
        changed = True
        while changed:  # advance every role to its next wait (arrivals happen on the way)
            changed = False
            for i in list(alive):
                if cur[i] is None:
                    try:
                        cur[i] = next(rs[i])
                    except StopIteration:
                        alive.discard(i)
                    changed = True
        if not alive:
            return None
        ready = []
        for i in alive:
            bar, k = cur[i]
            if bar.phase < k - 1 or bar.phase > k:
                return f"parity alias on {bar.name}: needs completion {k}, at phase {bar.phase}"
            if bar.phase >= k:
                ready.append(i)
        if not ready:
            return "deadlock"
        cur[rng.choice(ready)] = None
    return None


LAUNCHABLE = []
for wt, mode, nt, ndq in itertools.product([F16, Q8_0, Q4_K], [GATEUP, DOWN], [32, 64, 128], [2, 3, 4]):
    c = gemm_cfg(wt, mode, nt, ndq)
    if c["ring_ok"] and (wt != F16 or ndq == 2):
        LAUNCHABLE.append((wt, mode, nt, ndq))


@pytest.mark.parametrize("wt,mode,nt,ndq", LAUNCHABLE)
def test_launchable_configs_are_safe(wt, mode, nt, ndq):
    cfg = gemm_cfg(wt, mode, nt, ndq)
    assert cfg["stages"] >= 2 and (not cfg["quant"] or cfg["na"] >= 2)
    for tiles in ([16, 16, 16], [3, 1, 2], [1, 1, 1, 1, 1]):
        for seed in range(12):
            assert run(cfg, tiles, seed) is None, (cfg, tiles, seed)


def test_model_catches_a_short_ring():
    # fewer A buffers than dequant warpgroups: a group can wait two completions ahead
    cfg = dict(stages=4, na=3, ndq=4, kb=2, acc_bufs=2, quant=True, ring_ok=False)
    results = [run(cfg, [16, 16, 16], seed) for seed in range(25)]
    assert any(r and "alias" in r for r in results)


PAIR_LAUNCHABLE = [(wt, mode, ndq) for wt, mode, ndq in itertools.product([Q8_0, Q4_K], [GATEUP, DOWN], [2, 3, 4])
                   if gemm_cfg(wt, mode, 128, ndq, pair=True)["ring_ok"]]


@pytest.mark.parametrize("wt,mode,ndq", PAIR_LAUNCHABLE)
def test_pair_configs_are_safe(wt, mode, ndq):
    cfg = gemm_cfg(wt, mode, 128, ndq, pair=True)
    assert cfg["stages"] >= 2 and cfg["na"] >= 2
    for tiles in ([16, 16, 16], [3, 1, 2], [1, 1, 1, 1, 1]):
        for seed in range(8):
            assert run(cfg, tiles, seed, pair=True) is None, (cfg, tiles, seed)


def test_pair_model_catches_a_short_ring():
    cfg = dict(stages=3, na=2, ndq=4, kb=2, acc_bufs=1, quant=True, ring_ok=False)
    results = [run(cfg, [16, 16], seed, pair=True) for seed in range(25)]
    assert any(r and "alias" in r for r in results)


def gemm_cfg_bres(wt):
    """GemmCfg<WT, MODE_DOWN, 64, 2, false, BRES = true>: the resident activation tile (64 rows x
    1024 K fp16 = 128 KB) comes off the shared-memory budget, the stages carry weights only."""
    stage_k = 256 if wt == Q4_K else 128
    w_bytes = 128 * 144 if wt == Q4_K else 128 * 128 + 128 * 16
    stages = min(6, (227 * 1024 - 2048 - 1024 * 64 * 2) // (2 * w_bytes))
    na = min(4, (512 - 2 * 128) // 128)
    return dict(stages=stages, na=na, ndq=2, kb=stage_k // 128, acc_bufs=2, quant=True, ring_ok=na >= 2)


def roles_bres(cfg, units):
    """The single-CTA roles plus the resident tile: `units` is a list of (m-tiles, k-stages per
    m-tile). The producer waits bempty before each unit's activation load and arrives (TMA bytes)
    on bfull; the MMA waits bfull before a unit's first m-tile and commits bempty after its last."""
    S, NA, NDQ, KB, ACCB = cfg["stages"], cfg["na"], cfg["ndq"], cfg["kb"], cfg["acc_bufs"]
    full = [Bar(f"full{i}", 1) for i in range(S)]
    empty = [Bar(f"empty{i}", 1 + 4 * NDQ) for i in range(S)]
    afull = [Bar(f"afull{i}", 4) for i in range(NA)]
    aempty = [Bar(f"aempty{i}", 1) for i in range(NA)]
    accfull = [Bar(f"accfull{i}", 1) for i in range(ACCB)]
    accempty = [Bar(f"accempty{i}", 4) for i in range(ACCB)]
    bfull, bempty = Bar("bfull", 1), Bar("bempty", 1)
    tiles = [(mt == 0, mt == m - 1, k) for m, k in units for mt in range(m)]

    def producer():
        seq = useq = 0
        for first, _, k in tiles:
            if first:
                yield bempty, useq  # parity (useq & 1) ^ 1: the previous unit's release
                bfull.arrive()
                useq += 1
            for _ in range(k):
                s = seq % S
                yield empty[s], seq // S
                full[s].arrive()
                seq += 1

    def mma():
        seq = tseq = useq = 0
        for first, last, k in tiles:
            ab = tseq % ACCB
            yield accempty[ab], tseq // ACCB
            if first:
                yield bfull, useq + 1
                useq += 1
            for _ in range(k):
                s = seq % S
                yield full[s], seq // S + 1
                for kb in range(KB):
                    kbs = seq * KB + kb
                    a, u = kbs % NA, kbs // NA
                    yield afull[a], u + 1
                    aempty[a].arrive()
                empty[s].arrive()
                seq += 1
            accfull[ab].arrive()
            if last:
                bempty.arrive()
            tseq += 1

    def epilogue():
        tseq = 0
        for _ in tiles:
            ab = tseq % ACCB
            yield accfull[ab], tseq // ACCB + 1
            accempty[ab].arrive()
            tseq += 1

    def dequant(g):
        seq = 0
        for _, _, k in tiles:
            for _ in range(k):
                s = seq % S
                yield full[s], seq // S + 1
                for kb in range(KB):
                    kbs = seq * KB + kb
                    if kbs % NDQ != g:
                        continue
                    a, u = kbs % NA, kbs // NA
                    yield aempty[a], u
                    afull[a].arrive()
                empty[s].arrive()
                seq += 1

    rs = [producer(), mma()] + [epilogue() for _ in range(4)]
    rs += [dequant(g) for g in range(NDQ) for _ in range(4)]
    return rs


def run_roles(rs, seed):
    rng = random.Random(seed)
    cur = [None] * len(rs)
    alive = set(range(len(rs)))
    while alive:
        changed = True
        while changed:
            changed = False
            for i in list(alive):
                if cur[i] is None:
                    try:
                        cur[i] = next(rs[i])
                    except StopIteration:
                        alive.discard(i)
                    changed = True
        if not alive:
            return None
        ready = []
        for i in alive:
            bar, k = cur[i]
            if bar.phase < k - 1 or bar.phase > k:
                return f"parity alias on {bar.name}: needs completion {k}, at phase {bar.phase}"
            if bar.phase >= k:
                ready.append(i)
        if not ready:
            return "deadlock"
        cur[rng.choice(ready)] = None
    return None


@pytest.mark.parametrize("wt", [Q8_0, Q4_K])
def test_resident_tile_configs_are_safe(wt):
    cfg = gemm_cfg_bres(wt)
    assert cfg["stages"] >= 2 and cfg["na"] >= 2 and cfg["ring_ok"]
    kst = 1024 // (256 if wt == Q4_K else 128)
    # whole token tiles (16 m-tiles), chunked ones, a shared group of another K, single m-tiles
    for units in ([(16, kst)] * 3, [(4, kst)] * 5, [(8, kst // 2), (8, kst), (8, kst)], [(1, kst)] * 4):
        for seed in range(10):
            assert run_roles(roles_bres(cfg, units), seed) is None, (cfg, units, seed)


def test_resident_tile_model_catches_an_early_reload():
    """The model is sharp: a producer that reloads the resident tile without waiting for the
    previous unit's release is caught (it runs ahead of the MMA's bfull waits)."""
    cfg = gemm_cfg_bres(Q4_K)

    def no_wait_roles(units):
        rs = roles_bres(cfg, units)
        prod = rs[0]

        def eager():
            for bar, k in prod:
                if bar.name == "bempty":
                    continue  # skip the wait: the arrival on bfull follows at once
                yield bar, k
        rs[0] = eager()
        return rs

    results = [run_roles(no_wait_roles([(1, 1)] * 8), seed) for seed in range(30)]
    assert any(r and "alias" in r for r in results)


def gemm_cfg_bres_pair(wt, ndq):
    """GemmCfg<WT, MODE_DOWN, 128, NDQ, PAIR = true, BRES = true>: each CTA keeps its 64 token rows
    resident (128 KB); one 128-row block per CTA, so the stages hold one weight tile each."""
    stage_k = 256 if wt == Q4_K else 128
    w_bytes = 128 * 144 if wt == Q4_K else 128 * 128 + 128 * 16
    stages = min(6, (227 * 1024 - 2048 - 1024 * 64 * 2) // w_bytes)
    na = min(4, (512 - 2 * 128) // 32)  # 64-K A blocks (pairs): 32 columns each
    return dict(stages=stages, na=na, ndq=ndq, kb=stage_k // 64, acc_bufs=2, quant=True, ring_ok=na >= ndq)


def roles_bres_pair(cfg, units):
    """The pair's roles with resident tiles: each CTA's producer waits its own bempty and its
    activation half counts on the leader's bfull; the leader's MMA waits bfull before a unit's
    first m-tile (and no per-stage activation barrier), and its commit after the unit's last
    m-tile arrives on both CTAs' bempty."""
    S, NA, NDQ, KB, ACCB = cfg["stages"], cfg["na"], cfg["ndq"], cfg["kb"], cfg["acc_bufs"]
    cta = []
    for r in range(2):
        cta.append(dict(
            full=[Bar(f"full{i}.{r}", 1) for i in range(S)],
            empty=[Bar(f"empty{i}.{r}", 1 + 4 * NDQ) for i in range(S)],
            aempty=[Bar(f"aempty{i}.{r}", 1) for i in range(NA)],
            accfull=[Bar(f"accfull{i}.{r}", 1) for i in range(ACCB)],
            bempty=Bar(f"bempty.{r}", 1),
        ))
    bfull = Bar("bfull", 2)  # both halves' bytes (leader's barrier)
    afull = [Bar(f"afull{i}", 8) for i in range(NA)]
    accempty = [Bar(f"accempty{i}", 8) for i in range(ACCB)]
    tiles = [(mt == 0, mt == m - 1, k) for m, k in units for mt in range(m)]

    def producer(r):
        seq = useq = 0
        for first, _, k in tiles:
            if first:
                yield cta[r]["bempty"], useq
                bfull.arrive()
                useq += 1
            for _ in range(k):
                s = seq % S
                yield cta[r]["empty"][s], seq // S
                cta[r]["full"][s].arrive()
                seq += 1

    def mma():
        seq = tseq = useq = 0
        for first, last, k in tiles:
            ab = tseq % ACCB
            yield accempty[ab], tseq // ACCB
            if first:
                yield bfull, useq + 1
                useq += 1
            for _ in range(k):
                s = seq % S
                for kb in range(KB):
                    kbs = seq * KB + kb
                    a, u = kbs % NA, kbs // NA
                    yield afull[a], u + 1
                    for r in range(2):
                        cta[r]["aempty"][a].arrive()
                for r in range(2):
                    cta[r]["empty"][s].arrive()
                seq += 1
            for r in range(2):
                cta[r]["accfull"][ab].arrive()
                if last:
                    cta[r]["bempty"].arrive()
            tseq += 1

    def epilogue(r):
        tseq = 0
        for _ in tiles:
            ab = tseq % ACCB
            yield cta[r]["accfull"][ab], tseq // ACCB + 1
            accempty[ab].arrive()
            tseq += 1

    def dequant(r, g):
        seq = 0
        for _, _, k in tiles:
            for _ in range(k):
                s = seq % S
                yield cta[r]["full"][s], seq // S + 1
                for kb in range(KB):
                    kbs = seq * KB + kb
                    if kbs % NDQ != g:
                        continue
                    a, u = kbs % NA, kbs // NA
                    yield cta[r]["aempty"][a], u
                    afull[a].arrive()
                cta[r]["empty"][s].arrive()
                seq += 1

    rs = [mma()]
    for r in range(2):
        rs += [producer(r)] + [epilogue(r) for _ in range(4)]
        rs += [dequant(r, g) for g in range(NDQ) for _ in range(4)]
    return rs


@pytest.mark.parametrize("wt,ndq", [(Q8_0, 2), (Q8_0, 4), (Q4_K, 2), (Q4_K, 4)])
def test_resident_tile_pair_configs_are_safe(wt, ndq):
    cfg = gemm_cfg_bres_pair(wt, ndq)
    assert cfg["stages"] >= 2 and cfg["ring_ok"]
    kst = 1024 // (256 if wt == Q4_K else 128)
    for units in ([(16, kst)] * 2, [(4, kst)] * 4, [(8, kst // 2), (8, kst)], [(1, kst)] * 4, [(1, 1)] * 6):
        for seed in range(8):
            assert run_roles(roles_bres_pair(cfg, units), seed) is None, (cfg, units, seed)
