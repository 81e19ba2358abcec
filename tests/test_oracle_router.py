"""The oracle's router against independent restatements (CPU).

1. Canonical logits: an exact rational emulation of the fmaf chains and float adds of the canonical
   order (correctly rounded to binary32) on a tiny shape, bit for bit.
2. Routing (src/diffuse-moe-graph.cpp:204-262): a second restatement of the ggml op sequence in
   numpy float32 (fold max, threshold at sorted position cap-1, `bmax - (thr - 1e-6) > 0`, -1e30
   mask, top-k with ties to the lower id, unbiased gates, double-summed renormalisation, scaling),
   on adversarial cases: ties, an exact capacity boundary, a near-tie inside 1e-6 that admits more
   than `cap` experts, n % 32 != 0, no bias, no renormalisation, capacity >= experts.
3. The oracle's double-precision exp against the correctly rounded exp (at most 1 ulp, mostly 0).
"""
import math
from fractions import Fraction

import numpy as np
import pytest

import oracle

f32 = np.float32


def round_f32(x: Fraction) -> float:
    """Correctly rounded (ties to even) binary32 value of a rational (normal range)."""
    if x == 0:
        return 0.0
    sign = -1 if x < 0 else 1
    a = abs(x)
    e = math.floor(math.log2(a.numerator) - math.log2(a.denominator))
    while Fraction(2) ** e > a:
        e -= 1
    while Fraction(2) ** (e + 1) <= a:
        e += 1
    scaled = a / (Fraction(2) ** (e - 23))  # in [2^23, 2^24)
    q, r = divmod(scaled.numerator, scaled.denominator)
    rem = Fraction(r, scaled.denominator)
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and q % 2 == 1):
        q += 1
    return sign * float(Fraction(q) * Fraction(2) ** (e - 23))


def canonical_logits(x, w, seg=256):
    n, h = x.shape
    e = w.shape[0]
    out = np.zeros((n, e), dtype=np.float32)
    for t in range(n):
        for j in range(e):
            tot = None
            for s0 in range(0, h, seg):
                acc = 0.0
                for k in range(s0, min(h, s0 + seg)):
                    acc = round_f32(Fraction(float(x[t, k])) * Fraction(float(w[j, k])) + Fraction(acc))
                tot = acc if tot is None else round_f32(Fraction(tot) + Fraction(acc))
            out[t, j] = tot
    return out


def test_canonical_logits_bit_exact():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, 512)).astype(np.float32)
    w = (rng.standard_normal((4, 512)) * 0.02).astype(np.float32)
    ref = canonical_logits(x, w)
    got = oracle.logits(x, w)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def route_ref(logits, bias, top_k, cap, blk, norm, scale):
    n, e = logits.shape
    p = np.array([[oracle.sigmoid(float(v)) for v in row] for row in logits], dtype=np.float32)
    sel = (p + bias.astype(np.float32)).astype(np.float32) if bias is not None else p.copy()
    use_block = blk > 1 and 0 < cap < e and n % blk == 0
    allowed = None
    if use_block:
        nb = n // blk
        allowed = np.zeros((nb, e), dtype=np.uint8)
        for b in range(nb):
            s0 = sel[b * blk:(b + 1) * blk].copy()
            m = s0[0].copy()
            for t in range(1, blk):
                d = (m - s0[t]).astype(f32)
                m = (s0[t] + np.where(d > 0, d, f32(0))).astype(f32)
            thr = np.sort(m)[::-1][cap - 1]
            thr_m = f32(f32(thr * f32(1.0)) + f32(-1e-6))
            keep = (m - thr_m).astype(f32) > 0
            allowed[b] = keep
            sel[b * blk:(b + 1) * blk] = (s0 + np.where(keep, f32(0), f32(-1e30))).astype(f32)
    idx = np.zeros((n, top_k), dtype=np.int32)
    w = np.zeros((n, top_k), dtype=np.float32)
    for t in range(n):
        order = sorted(range(e), key=lambda i: (-float(sel[t, i]), i))[:top_k]
        idx[t] = order
        wt = p[t, order].astype(np.float32)
        if norm:
            s = f32(sum(float(v) for v in wt))
            wt = (wt / s).astype(f32)
        if scale != 1.0:
            wt = (wt * f32(scale)).astype(f32)
        w[t] = wt
    return idx, w, allowed, use_block


def check(logits, bias, top_k, cap, blk, norm=1, scale=2.5):
    r_idx, r_w, r_allowed, r_used = route_ref(logits, bias, top_k, cap, blk, norm, scale)
    idx, w, _, allowed, used = oracle.route(logits, bias, top_k, cap, blk, norm, scale)
    assert used == r_used
    assert np.array_equal(idx, r_idx)
    assert np.array_equal(w.view(np.uint32), r_w.view(np.uint32))
    if used:
        assert np.array_equal(allowed, r_allowed)
    return allowed


def test_random_block_routing():
    rng = np.random.default_rng(1)
    lg = rng.standard_normal((64, 64)).astype(np.float32)
    bias = rng.uniform(-0.05, 0.05, 64).astype(np.float32)
    check(lg, bias, 8, 12, 32)


def test_ties_go_to_lower_expert():
    lg = np.zeros((32, 32), dtype=np.float32)  # every score equal: capacity and top-k all tie
    allowed = check(lg, None, 4, 6, 32)
    assert allowed.sum() == 32  # all bmax equal thr > thr - 1e-6: everyone admitted


def test_exact_boundary_and_near_tie_admission():
    e, cap = 32, 6
    lg = np.full((32, e), -4.0, dtype=np.float32)
    # distinct block maxima for experts 0..e-1, decreasing; token 0 carries them
    lg[0] = np.linspace(3.0, -3.0, e).astype(np.float32)
    allowed = check(lg.copy(), None, 4, cap, 32)
    assert allowed.sum() == cap  # strictly separated: exactly cap admitted
    # expert cap (7th) within 1e-6 below the threshold in probability space: admitted too
    p = np.array([oracle.sigmoid(float(v)) for v in lg[0]], dtype=np.float32)
    bias = np.zeros(e, dtype=np.float32)
    bias[cap] = f32(p[cap - 1] - p[cap] - f32(4e-7))
    allowed = check(lg.copy(), bias, 4, cap, 32)
    assert allowed.sum() == cap + 1


def test_plain_topk_when_not_block_multiple():
    rng = np.random.default_rng(2)
    lg = rng.standard_normal((50, 64)).astype(np.float32)
    check(lg, rng.uniform(-0.05, 0.05, 64).astype(np.float32), 8, 12, 32)


@pytest.mark.parametrize("norm,scale", [(0, 1.0), (1, 1.0), (0, 2.5)])
def test_no_bias_and_gate_options(norm, scale):
    rng = np.random.default_rng(3)
    lg = rng.standard_normal((32, 16)).astype(np.float32)
    check(lg, None, 4, 6, 32, norm, scale)


def test_capacity_not_below_experts_disables_block_routing():
    rng = np.random.default_rng(4)
    lg = rng.standard_normal((32, 16)).astype(np.float32)
    check(lg, None, 4, 16, 32)


def test_exp_within_one_ulp():
    rng = np.random.default_rng(6)
    vals = np.concatenate([rng.standard_normal(4000) * 8, np.array([0.0, -0.0, 87.0, -87.0, 103.0, -103.0])])
    exact = 0
    for v in vals.astype(np.float32):
        got = oracle.exp_neg(float(v))
        ref = f32(math.exp(-float(v))) if -float(v) < 88.7 else f32(np.inf)
        if got == ref:
            exact += 1
        else:
            assert abs(np.float32(got).view(np.int32) - ref.view(np.int32)) <= 1, (v, got, ref)
    assert exact >= 0.999 * len(vals)
