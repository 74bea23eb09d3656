"""Rejection sampling over draft trees: the CPU spec (oracle vo_accept_tree,
multi-candidate speculative sampling as in SpecInfer, Miao et al. 2024).

- on chains it takes the decisions of the chain spec (vo_accept) bit for bit;
- it is a sampler of the target distribution: with a root whose children are
  drawn i.i.d. from q, the first emitted token (the accepted child, or the
  bonus) follows p, whatever q is;
- the walk descends only through accepted children and the path is a
  root-to-node path of the tree."""
import numpy as np

import synthetic
import vo


def test_tree_spec_on_chains_equals_chain_spec():
    B, k, V, T = 16, 6, 3000, 0.8
    tgt, drf, tok, u = synthetic.acceptance_inputs(B, k, V, T, seed=3)
    acc, bonus = vo.accept(tgt, drf, tok, u, T)
    N = k + 1
    ttok = np.zeros((B, N), np.uint32)
    ttok[:, 1:] = tok
    par = np.tile(np.arange(-1, N - 1, dtype=np.int32), (B, 1))
    path, plen, tb = vo.accept_tree(tgt, drf, ttok, par, u, T)
    assert np.array_equal(plen - 1, acc)
    assert np.array_equal(tb, bonus)
    for b in range(B):
        assert list(path[b, :plen[b]]) == list(range(plen[b]))
        assert (path[b, plen[b]:] == -1).all()


def test_tree_spec_samples_the_target_distribution():
    """Root with 3 children drawn i.i.d. from q: the first emitted token is
    distributed as p (SpecInfer's correctness theorem)."""
    V, T, n = 8, 1.0, 12000
    g = synthetic.rng(5, 80)
    t_log = g.normal(0, 1.0, V).astype(np.float32)
    d_log = g.normal(0, 1.0, V).astype(np.float32)
    p = synthetic.softmax64(t_log)
    q = synthetic.softmax64(d_log)
    N = 4
    par = np.array([[-1, 0, 0, 0]] * n, np.int32)
    tgt = np.tile(t_log, (n, N, 1))
    drf = np.tile(d_log, (n, N - 1, 1))
    tok = np.zeros((n, N), np.uint32)
    tok[:, 1:] = g.choice(V, size=(n, N - 1), p=q)
    u = g.random((n, N)).astype(np.float32)
    path, plen, bonus = vo.accept_tree(tgt, drf, tok, par, u, T)
    first = np.where(plen > 1, tok[np.arange(n), np.maximum(path[:, 1], 0)], bonus)
    freq = np.bincount(first, minlength=V) / n
    # 4.5 standard errors of a binomial proportion
    assert np.all(np.abs(freq - p) <= 4.5 * np.sqrt(p * (1 - p) / n) + 1e-3), (freq, p)


def test_tree_spec_paths_follow_the_tree():
    B, N, V, T = 24, 20, 500, 0.7
    g = synthetic.rng(6, 81)
    tgt = g.normal(0, 2, (B, N, V)).astype(np.float32)
    # drafts close to the target so that walks go deep
    drf = (tgt[:, :N - 1] + g.normal(0, 0.3, (B, N - 1, V))).astype(np.float32)
    par = np.stack([synthetic.random_tree(N, 5, g) for _ in range(B)])
    tok = np.zeros((B, N), np.uint32)
    for b in range(B):
        for n in range(1, N):
            q = synthetic.softmax64(drf[b, par[b, n]] / T)
            tok[b, n] = g.choice(V, p=q)
    u = g.random((B, N)).astype(np.float32)
    path, plen, bonus = vo.accept_tree(tgt, drf, tok, par, u, T)
    assert plen.max() >= 3
    for b in range(B):
        pth = path[b, :plen[b]]
        assert pth[0] == 0
        for i in range(1, len(pth)):
            assert par[b, pth[i]] == pth[i - 1]
        assert bonus[b] < V
