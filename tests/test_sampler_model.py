"""CPU model of the sampler kernels' two algorithmic choices (diffuse-cpp_b200/csrc/sampler.cu),
checked against the sequential rules of the reference (src/diffuse-sampler.cpp) as restated in
the oracle:

1. sample_commit_kernel decides each candidate independently from its rank (probability
   descending, position ascending on ties): committed iff rank < n_transfer or
   prob >= threshold, plus the rank-0 candidate when nothing else is. Fuzzed here against the
   oracle's sorted commit loop, including duplicated probabilities and thresholds placed exactly
   on candidate values.
2. sample_rows_kernel keeps a running (max, lowest index of the max, sum of exp(l - max)) per
   thread and merges the triples in a fixed tree. Restated in float32 with the kernel's slicing
   (8 CTAs, 512 threads, groups of 4 values, 10 groups per batch), checked for the lowest-index
   argmax on rows full of ties and for a probability within 2e-5 of the exact value.
"""
import numpy as np
import pytest

import oracle

MASK = 3


def commit_by_rank(tok, prob, n_transfer, threshold, seq):
    out = np.array(seq, np.int32)
    cand = tok >= 0
    n = 0
    top = -1
    for i in range(len(tok)):
        if not cand[i]:
            continue
        rank = sum(1 for j in range(len(tok)) if cand[j] and (prob[j] > prob[i] or (prob[j] == prob[i] and j < i)))
        if rank == 0:
            top = i
        if rank < n_transfer or prob[i] >= threshold:
            out[i] = tok[i]
            n += 1
    if n == 0 and top >= 0:
        out[top] = tok[top]
        n = 1
    return out, n


def commit_sequential(tok, prob, n_transfer, threshold, seq):
    out = np.array(seq, np.int32)
    c = [i for i in range(len(tok)) if tok[i] >= 0]
    c.sort(key=lambda i: -prob[i])  # stable
    n = 0
    for i in c:
        if n >= n_transfer and prob[i] < threshold:
            break
        out[i] = tok[i]
        n += 1
    if n == 0 and c:
        out[c[0]] = tok[c[0]]
        n = 1
    return out, n


@pytest.mark.parametrize("seed", range(40))
def test_rank_rule_equals_sorted_loop(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 40))
    levels = rng.random(int(rng.integers(1, 6))).astype(np.float32)  # few distinct values: ties
    prob = levels[rng.integers(0, len(levels), n)]
    tok = np.where(rng.random(n) < 0.75, rng.integers(0, 1000, n), -1).astype(np.int32)
    seq = np.where(tok >= 0, MASK, 77).astype(np.int32)
    n_transfer = int(rng.integers(-1, n + 2))
    threshold = float(levels[rng.integers(0, len(levels))]) if rng.random() < 0.5 else float(rng.random())
    a, na = commit_by_rank(tok, prob, n_transfer, threshold, seq)
    b, nb = commit_sequential(tok, prob, n_transfer, threshold, seq)
    assert na == nb and np.array_equal(a, b)


def test_rank_rule_equals_oracle_on_logits():
    rng = np.random.default_rng(11)
    logits = rng.normal(0, 2, (24, 3000)).astype(np.float32)
    logits[5] = logits[4]  # two equal rows: equal probabilities
    seq = np.where(rng.random(24) < 0.8, MASK, 9).astype(np.int32)
    t, p, s, n = oracle.sample_step(logits, seq, MASK, 3, 0.9)
    a, na = commit_by_rank(t, p, 3, 0.9, seq)
    assert na == n and np.array_equal(a, s)


# ---- the rows kernel's reduction, restated in float32 ----------------------------------------
F = np.float32


def visit(t, x, v):
    m, i, s = t
    if x > m:
        return (x, v, F(F(s * np.exp(F(m - x), dtype=F)) + F(1)))
    return (m, i, F(s + np.exp(F(x - m), dtype=F)))


def merge(a, b):
    if b[2] == 0:
        return a
    if a[2] == 0:
        return b
    if a[0] > b[0]:
        return (a[0], a[1], F(a[2] + F(b[2] * np.exp(F(b[0] - a[0]), dtype=F))))
    if b[0] > a[0]:
        return (b[0], b[1], F(b[2] + F(a[2] * np.exp(F(a[0] - b[0]), dtype=F))))
    return (a[0], min(a[1], b[1]), F(a[2] + b[2]))


def tree(parts):
    """The kernel's shuffle-down trees: offsets n/2, ..., 1 over a power-of-two list."""
    parts = list(parts)
    off = len(parts) // 2
    while off:
        parts = [merge(parts[k], parts[k + off]) if k + off < len(parts) else parts[k] for k in range(len(parts))]
        off //= 2
    return parts[0]


def model_row(row, ctas=8, threads=512, unroll=10):
    V = len(row)
    per = ((V + ctas - 1) // ctas + 3) & ~3
    empty = (F(-np.inf), 0, F(0))
    cta_best = []
    for c in range(ctas):
        v0, v1 = c * per, min(V, c * per + per)
        th = [empty] * threads
        if v0 < v1:
            n4 = (v1 - v0) // 4
            for tid in range(threads):
                t = empty
                for q0 in range(tid, n4, unroll * threads):
                    for u in range(unroll):
                        q = q0 + u * threads
                        if q >= n4:
                            break
                        b = v0 + 4 * q
                        for k in range(4):
                            t = visit(t, row[b + k], b + k)
                for q in range(v0 + 4 * n4 + tid, v1, threads):
                    t = visit(t, row[q], q)
                th[tid] = t
        warps = [tree(th[w * 32:(w + 1) * 32]) for w in range(threads // 32)]
        cta_best.append(tree(warps + [empty] * (32 - len(warps))))
    best = tree(cta_best)
    return best[1], F(1) / best[2]


@pytest.mark.parametrize("V,seed", [(4099, 0), (20000, 1), (7, 2)])
def test_rows_reduction_model(V, seed):
    rng = np.random.default_rng(seed)
    row = rng.integers(-4, 5, V).astype(F)  # integer logits: the maximum occurs many times
    tok, prob = model_row(row)
    assert tok == int(np.argmax(row))  # the lowest index of the maximum
    d = row.astype(np.float64)
    exact = 1.0 / np.exp(d - d.max()).sum()
    assert abs(prob - exact) <= 2e-5 * exact
