"""Rejection sampling over draft trees on the GPU (velo_cuda_accept_tree,
and velo_cuda_verify_step at temperature > 0 on trees) against the CPU spec
(oracle vo_accept_tree): accepted paths, path lengths and bonus tokens
bit-exact on the same logits and uniforms."""
import numpy as np
import pytest

import synthetic
import velo_cuda
import vo

pytestmark = pytest.mark.gpu

C3_TREE = [-1, 0, 0, 0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5, 6]


def _tree_inputs(B, parents, V, T, seed, draft_sigma=0.5, target_sigma=2.0):
    """Target rows ~ N(0, target_sigma^2), draft rows = target + noise, and
    children drawn from the draft distribution of their parent (i.i.d.)."""
    g = synthetic.rng(seed, 90)
    par = np.asarray(parents, np.int32)
    N = par.shape[-1]
    par = np.broadcast_to(par, (B, N)).copy()
    tgt = g.normal(0, target_sigma, (B, N, V)).astype(np.float32)
    drf = (tgt[:, :N - 1] + g.normal(0, draft_sigma, (B, N - 1, V))).astype(np.float32)
    tok = np.zeros((B, N), np.uint32)
    for b in range(B):
        q = synthetic.softmax64(drf[b] / T)
        c = np.cumsum(q, axis=-1)
        for n in range(1, N):
            tok[b, n] = min(int((c[par[b, n]] < g.random()).sum()), V - 1)
    u = g.random((B, N)).astype(np.float32)
    return tgt, drf, tok, par, u


@pytest.mark.parametrize("B,V,T,shape", [
    (32, 32000, 0.8, "c3"),          # the config-3 tree, config-3 vocabulary
    (8, 128256, 1.0, "c5"),          # 32-node trees at the config-5 vocabulary
    (12, 1000, 0.6, "random"),       # random trees, ragged last tile
    (5, 4097, 1.3, "random"),
])
def test_tree_acceptance_matches_spec(ctx, B, V, T, shape):
    g = synthetic.rng(B + V, 91)
    if shape == "c3":
        parents = np.array(C3_TREE, np.int32)
    elif shape == "c5":
        parents = np.array([-1, 0, 0, 0, 0] + [1 + i // 2 for i in range(8)] +
                           [5 + i // 2 for i in range(16)] + [13 + i // 2 for i in range(3)], np.int32)
    else:
        parents = np.stack([synthetic.random_tree(24, 6, g) for _ in range(B)])
    tgt, drf, tok, par, u = _tree_inputs(B, parents, V, T, seed=B + V)
    path, plen, bonus = ctx.accept_tree(tgt, drf, tok, par, u, T)
    rp, rl, rb = vo.accept_tree(tgt, drf, tok, par, u, T)
    assert np.array_equal(plen, rl)
    assert np.array_equal(path, rp)
    assert np.array_equal(bonus, rb)
    assert plen.max() >= 2  # drafts close to the target: some walks go below the root


def test_tree_acceptance_on_chains_equals_chain_kernel(ctx):
    B, k, V, T = 64, 8, 32000, 0.8
    tgt, drf, tok, u = synthetic.acceptance_inputs(B, k, V, T, seed=4)
    acc, bonus = ctx.accept(tgt, drf, tok, u, T)
    N = k + 1
    ttok = np.zeros((B, N), np.uint32)
    ttok[:, 1:] = tok
    par = np.tile(np.arange(-1, N - 1, dtype=np.int32), (B, 1))
    path, plen, tb = ctx.accept_tree(tgt, drf, ttok, par, u, T)
    assert np.array_equal(plen - 1, acc)
    assert np.array_equal(tb, bonus)


def test_tree_acceptance_device_form_repeats(ctx):
    import torch
    B, V, T = 16, 32000, 0.8
    tgt, drf, tok, par, u = _tree_inputs(B, np.array(C3_TREE, np.int32), V, T, seed=5)
    d = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (tgt, drf, tok.view(np.int32), par, u)]
    N = len(C3_TREE)
    torch.cuda.synchronize()
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    try:
        outs = []
        for _ in range(2):
            path = torch.full((B, N), -7, dtype=torch.int32, device="cuda")
            plen = torch.zeros(B, dtype=torch.int32, device="cuda")
            bonus = torch.zeros(B, dtype=torch.int32, device="cuda")
            ctx.accept_tree_device(*d, T, path, plen, bonus)
            ctx.sync()
            outs.append((path.cpu().numpy(), plen.cpu().numpy(), bonus.cpu().numpy().view(np.uint32)))
    finally:
        ctx.set_stream(None)
    rp, rl, rb = vo.accept_tree(tgt, drf, tok, par, u, T)
    for p_, l_, b_ in outs:
        assert np.array_equal(p_, rp) and np.array_equal(l_, rl) and np.array_equal(b_, rb)


def test_verify_step_samples_trees(cuda_device):
    """A temperature > 0 verify step on trees: the path, bonus token and
    committed K/V follow the spec applied to the step's own logits."""
    shape = dict(n_vocab=2048, n_embd=256, n_layer=2, n_head=2, n_head_kv=2, n_ff=512)
    meta, tensors = synthetic.llama_q4_model(**shape, seed=8)
    V, T = meta["n_vocab"], 0.9
    g = synthetic.rng(9, 92)
    B, N = 3, 12
    parents = np.stack([synthetic.random_tree(N, 4, g) for _ in range(B)])
    ctx = velo_cuda.Context(device=cuda_device, total_pages=48, max_slots=B, max_pages_per_slot=16)
    try:
        ctx.load_model(meta, tensors)
        for b in range(B):
            ctx.bind_slot(b, np.arange(16 * b, 16 * b + 16))
        slots = np.arange(B, dtype=np.uint32)
        cl = np.zeros(B, np.int32)
        tokens = g.integers(0, V, (B, N)).astype(np.uint32)
        first = ctx.verify_step(slots, cl, tokens, parents, commit=False, want_logits=True, n_vocab=V)
        lg = first["logits"]
        # drafts near the target's distribution at the parent, children drawn from them
        drf = (lg[:, :N - 1] + g.normal(0, 0.3, (B, N - 1, V))).astype(np.float32)
        for b in range(B):
            for n in range(1, N):
                q = synthetic.softmax64(drf[b, parents[b, n]] / T)
                tokens[b, n] = min(int((np.cumsum(q) < g.random()).sum()), V - 1)
        u = g.random((B, N)).astype(np.float32)
        res = ctx.verify_step(slots, cl, tokens, parents, temperature=T, draft_logits=drf, uniforms=u,
                              commit=True, want_logits=True, n_vocab=V)
        rp, rl, rb = vo.accept_tree(res["logits"], drf, tokens, parents, u, T)
        assert np.array_equal(res["accepted_len"], rl - 1)
        assert np.array_equal(res["accepted_nodes"], rp)
        assert np.array_equal(res["bonus"], rb)
        # the accepted path's K/V were committed: a greedy step over the same
        # prefix sees them (its node 0 sits after the committed path)
        for b in range(B):
            ora = vo.Model(dict(meta, n_ctx=64), synthetic.oracle_tensor_list(meta, tensors))
            ora.verify_tree(tokens[b], parents[b], 0)
            ora.commit_path(list(rp[b, :rl[b]]), 0)
            k, _ = ctx.read_kv(b, 1, 0, int(rl[b]), meta["n_head_kv"])
            rk = ora.read_kv(0, 1, int(rl[b])).reshape(int(rl[b]), meta["n_head_kv"], 128)
            assert np.abs(k.astype(np.float32) - rk).max() <= 2e-2
    finally:
        ctx.close()
