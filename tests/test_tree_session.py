"""SpeculativeTree / find_best_path / TopKSampler restated in speculative.py:
the reference's tree KAT (speculative.rs:797-825), agreement with the oracle's
find_best_path on random trees, and the top-k ordering rule (sampling.rs:105-131)."""
import numpy as np

import synthetic
import vo
from speculative import SpeculativeTree, top_k


def test_tree_best_path_kat():
    tree = SpeculativeTree(10)
    c1 = tree.add_child(0, 20)
    tree.add_child(0, 30)
    tree.add_child(c1, 40)
    assert tree.find_best_path([30, 99, 99, 99]) == ([10, 30], 99)
    assert tree.find_best_path([20, 40, 99, 99]) == ([10, 20, 40], 99)


def test_find_best_path_matches_oracle():
    g = synthetic.rng(3, 70)
    for _ in range(200):
        n = int(g.integers(1, 20))
        parents = [-1] + [int(g.integers(0, i)) for i in range(1, n)]
        tokens = g.integers(0, 4, n).astype(np.uint32)
        expected = g.integers(0, 4, n).astype(np.uint32)
        t = SpeculativeTree(tokens[0])
        for i in range(1, n):
            t.add_child(parents[i], tokens[i])
        path, bonus = t.find_best_path([int(e) for e in expected])
        rpath, rbonus = vo.find_best_path(np.array(parents, np.int32), tokens, expected)
        assert path == [int(tokens[i]) for i in rpath] and bonus == rbonus


def test_top_k_stable_descending():
    got = top_k([1.0, 3.0, 3.0, 2.0, 3.0], 4)
    assert [p.token for p in got] == [1, 2, 4, 3]
    assert top_k([0.5], 3)[0].token == 0 and len(top_k([0.5], 3)) == 1
