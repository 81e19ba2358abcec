"""The sampler oracle (no GPU): oracle/dmoe_oracle_sampler.c against an independent numpy
restatement of src/diffuse-sampler.cpp:29-49 (argmax by a strict `>` scan, probability
1 / sum expf(l - max) summed in float in index order) and :183-237 (commit the first n_transfer
candidates by probability, then every one at or above the threshold, at least one), on crafted
cases: threshold crossings, unmasked positions, none masked, ties in the logits and in the
probabilities (equal probabilities commit in position order)."""
import numpy as np
import pytest

import oracle

MASK = 7


def np_step(logits, seq, n_transfer, threshold):
    tok = np.full(len(logits), -1, np.int32)
    prob = np.zeros(len(logits), np.float32)
    for r, row in enumerate(logits):
        if seq is not None and seq[r] != MASK:
            continue
        tok[r] = int(np.argmax(row))  # first maximum = the strict-`>` scan's answer
        e = np.exp((row - row[tok[r]]).astype(np.float32)).astype(np.float32)
        prob[r] = np.float32(1.0) / np.add.accumulate(e, dtype=np.float32)[-1]  # float, index order
    if seq is None:
        return tok, prob, None, 0
    out = np.array(seq, np.int32)
    cands = [r for r in range(len(logits)) if tok[r] >= 0]
    cands.sort(key=lambda r: -prob[r])  # stable: equal probabilities stay in position order
    n = 0
    for r in cands:
        if n >= n_transfer and prob[r] < threshold:
            break
        out[r] = tok[r]
        n += 1
    if n == 0 and cands:
        out[cands[0]] = tok[cands[0]]
        n = 1
    return tok, prob, out, n


def peaked(V, peak_at, lift, seed):
    """A row of zeros but one logit `lift` at `peak_at`: prob = 1 / (1 + (V - 1) e^-lift)."""
    row = np.random.default_rng(seed).normal(0, 1e-3, V).astype(np.float32)
    row[peak_at] = lift
    return row


def check(logits, seq, n_transfer, threshold):
    t, p, s, n = oracle.sample_step(logits, seq, MASK, n_transfer, threshold)
    rt, rp, rs, rn = np_step(logits, seq, n_transfer, threshold)
    assert np.array_equal(t, rt)
    np.testing.assert_allclose(p, rp, rtol=2e-6)
    assert n == rn and (s is None or np.array_equal(s, rs))
    return t, p, s, n


def test_threshold_and_transfer_count():
    V = 1000
    lifts = [11.5, 7.0, 10.5, 5.0, 10.2, 3.0, 6.0, 9.8]  # probs ~0.99, 0.5, 0.97, .., 0.96, .., 0.94
    logits = np.stack([peaked(V, 10 * r + 3, l, r) for r, l in enumerate(lifts)])
    seq = np.full(8, MASK, np.int32)
    t, p, s, n = check(logits, seq, 2, 0.95)
    assert n == 3 and set(np.nonzero(s != MASK)[0]) == {0, 2, 4}
    assert all(s[r] == 10 * r + 3 for r in (0, 2, 4))


def test_unmasked_positions_are_not_candidates():
    V = 500
    logits = np.stack([peaked(V, r, 12.0 - r, r) for r in range(6)])
    seq = np.array([MASK, 42, MASK, 43, MASK, MASK], np.int32)
    t, p, s, n = check(logits, seq, 1, 0.999)
    assert t[1] == -1 and t[3] == -1 and s[1] == 42 and s[3] == 43
    assert n == 1 and s[0] == 0  # the most confident candidate only


def test_none_masked_and_at_least_one():
    V = 300
    logits = np.stack([peaked(V, r, 2.0, r) for r in range(4)])
    seq = np.arange(4, dtype=np.int32) + 100
    t, p, s, n = check(logits, seq, 3, 0.5)
    assert n == 0 and np.array_equal(s, seq)
    seq = np.full(4, MASK, np.int32)
    t, p, s, n = check(logits, seq, 0, 0.999)  # nothing required, nothing above threshold
    assert n == 1


def test_ties():
    V = 256
    row = np.random.default_rng(3).normal(0, 1, V).astype(np.float32)
    row[[17, 90, 200]] = 9.0  # equal maxima: the lowest index wins
    logits = np.stack([row, row, row])  # equal probabilities: position order
    seq = np.full(3, MASK, np.int32)
    t, p, s, n = check(logits, seq, 2, 1.5)
    assert (t == 17).all() and p[0] == p[1] == p[2]
    assert n == 2 and s[0] == 17 and s[1] == 17 and s[2] == MASK


def test_no_seq_means_every_row_and_no_commit():
    logits = np.random.default_rng(5).normal(0, 2, (5, 1001)).astype(np.float32)
    t, p, s, n = check(logits, None, 3, 0.5)
    assert s is None and n == 0 and (t >= 0).all()


@pytest.mark.parametrize("V", [1, 2, 157184])
def test_vocab_sizes(V):
    logits = np.random.default_rng(V).normal(0, 3, (3, V)).astype(np.float32)
    check(logits, np.full(3, MASK, np.int32), 1, 0.95)
