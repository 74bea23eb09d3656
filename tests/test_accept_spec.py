"""Properties of the acceptance spec on the CPU oracle (no GPU).

The reference has no rejection sampling; these tests check the restated
method (Leviathan et al. 2023, Chen et al. 2023) itself: the spec exponential
is accurate, and the first emitted token is distributed exactly as the
target's p, whatever the draft's q.
"""
import math

import numpy as np

import synthetic
import vo


def test_spec_exp_accuracy():
    ys = np.concatenate([np.linspace(-87, 88, 20001), -np.abs(np.random.default_rng(1).normal(0, 6, 20000))])
    err = max(abs(vo.spec_exp(float(y)) - math.exp(float(np.float32(y)))) / math.exp(float(np.float32(y)))
              for y in ys.astype(np.float32))
    assert err < 3e-7
    assert vo.spec_exp(0.0) == 1.0


def test_row_stats_normaliser():
    row = np.random.default_rng(2).normal(0, 2, 32000).astype(np.float32)
    M, Z = vo.row_stats(row, 1.0 / 0.8)
    s = row.astype(np.float64) / 0.8
    assert abs(M - s.max()) < 1e-5
    assert abs(Z - np.exp(s - M).sum()) / Z < 1e-5


def test_first_emitted_token_is_distributed_as_p():
    V, k, B, T = 12, 1, 60000, 1.0
    g = np.random.default_rng(3)
    t_row = g.normal(0, 1.5, V).astype(np.float32)
    d_row = (t_row + g.normal(0, 1.0, V)).astype(np.float32)
    tgt = np.broadcast_to(np.stack([t_row, t_row]), (B, 2, V)).copy()
    drf = np.broadcast_to(d_row, (B, 1, V)).copy()
    q = synthetic.softmax64(d_row / T)
    tok = g.choice(V, size=(B, 1), p=q).astype(np.uint32)
    u = g.random((B, 2)).astype(np.float32)
    acc, bonus = vo.accept(tgt, drf, tok, u, T)
    first = np.where(acc >= 1, tok[:, 0], bonus)
    p = synthetic.softmax64(t_row / T)
    freq = np.bincount(first, minlength=V) / B
    sigma = np.sqrt(p * (1 - p) / B)
    assert np.all(np.abs(freq - p) < 5 * sigma + 1e-4), (freq, p)
    # the acceptance rate is sum_x min(p(x), q(x))
    rate = np.minimum(p, q).sum()
    assert abs((acc >= 1).mean() - rate) < 5 * math.sqrt(rate * (1 - rate) / B)


def test_bonus_after_full_acceptance_is_distributed_as_p_k():
    V, k, B = 9, 2, 40000
    g = np.random.default_rng(4)
    rows = g.normal(0, 1, (k + 1, V)).astype(np.float32)
    tgt = np.broadcast_to(rows, (B, k + 1, V)).copy()
    drf = tgt[:, :k].copy()  # identical draft: always accepted
    tok = g.integers(0, V, (B, k)).astype(np.uint32)
    u = g.random((B, k + 1)).astype(np.float32)
    acc, bonus = vo.accept(tgt, drf, tok, u, 0.5)
    assert np.all(acc == k)
    p = synthetic.softmax64(rows[k] / 0.5)
    freq = np.bincount(bonus, minlength=V) / B
    assert np.all(np.abs(freq - p) < 5 * np.sqrt(p * (1 - p) / B) + 1e-4)


def test_greedy_matches_reference_prefix_rule():
    """speculative.rs:441-467 with GreedySampler rows: accept while the draft
    token equals the row argmax; the bonus is the argmax at the stop row."""
    g = np.random.default_rng(6)
    B, k, V = 32, 5, 50
    tgt = g.normal(0, 1, (B, k + 1, V)).astype(np.float32)
    am = tgt.argmax(-1)
    tok = am[:, :k].copy()
    cut = g.integers(0, k + 1, B)
    for b in range(B):
        if cut[b] < k:
            tok[b, cut[b]] = (am[b, cut[b]] + 1) % V
    acc, bonus = vo.accept(tgt, None, tok.astype(np.uint32), np.zeros((B, k + 1), np.float32), 0.0)
    assert np.array_equal(acc, cut)
    assert np.array_equal(bonus, am[np.arange(B), cut])
