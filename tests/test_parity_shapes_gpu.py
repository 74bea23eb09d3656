"""Parity at the benchmarked shapes: the verify step and the q4_0 GEMMs at the
layer dimensions of BASELINE configs 3 (Llama-2-7B) and 5 (Llama-3-70B), not
only on toy models.

- verify step (velo_cuda_verify_step) against the oracle's forward
  (vo_verify_tree: llama_cpu.rs forward_one with the tree contract) on models
  with the configs' hidden size, heads, FFN and vocabulary and 1-2 layers,
  over a cached prefix written identically to both sides: logits of every
  node within 2e-2, paths and bonus tokens bit-exact against
  GreedySampler + find_best_path on the same logits, committed K/V within
  2e-2 of the oracle's cache;
- GEMMs at the config-5 layer shapes (M = 2048 rows = 64 sequences x 32
  nodes) against the reference's fp32 dequantisation, on a seeded sample of
  rows in float64.

The oracle splits each matvec's rows over the host's threads (vo.set_threads:
every row is still one sequential dot product, so the bits do not change)."""
import os

import numpy as np
import pytest

import synthetic
import velo_cuda
import vo

pytestmark = pytest.mark.gpu

TOL_LOGITS = 2e-2

C3_DIMS = dict(n_vocab=32000, n_embd=4096, n_head=32, n_head_kv=32, n_ff=11008)
C5_DIMS = dict(n_vocab=128256, n_embd=8192, n_head=64, n_head_kv=8, n_ff=28672)
C3_TREE = [-1, 0, 0, 0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5, 6]
C5_TREE = ([-1, 0, 0, 0, 0] + [1 + i // 2 for i in range(8)] + [5 + i // 2 for i in range(16)]
           + [13 + i // 2 for i in range(3)])


@pytest.fixture(autouse=True)
def _oracle_threads():
    vo.set_threads(min(64, os.cpu_count() or 1))
    yield
    vo.set_threads(1)


def _prefix_kv(g, P, Hkv):
    """Cached K/V rows [P][Hkv][128], f16 values (exact in both caches)."""
    k = g.normal(0, 1, (P, Hkv, 128)).astype(np.float16)
    v = g.normal(0, 1, (P, Hkv, 128)).astype(np.float16)
    return k, v


@pytest.mark.parametrize("case,n_layer,ctx_lens,rope_base", [
    ("c3", 2, [2048, 2048], 10000.0),
    ("c5", 1, [1000, 517], 500000.0),
])
def test_verify_step_at_config_dims(cuda_device, case, n_layer, ctx_lens, rope_base):
    dims = C3_DIMS if case == "c3" else C5_DIMS
    tree = np.array(C3_TREE if case == "c3" else C5_TREE, np.int32)
    meta, tensors = synthetic.llama_random_q4_model(**dims, n_layer=n_layer, seed=11,
                                                    rope_freq_base=rope_base)
    V, Hkv, L = meta["n_vocab"], meta["n_head_kv"], meta["n_layer"]
    B, N = len(ctx_lens), len(tree)
    g = synthetic.rng(12, 70)
    per_seq = (max(ctx_lens) + N + 15) // 16
    ctx = velo_cuda.Context(device=cuda_device, total_pages=B * per_seq + 3, max_slots=B,
                            max_pages_per_slot=per_seq)
    try:
        ctx.load_model(meta, tensors)
        perm = g.permutation(B * per_seq + 3).astype(np.uint32)
        oras = []
        tl = synthetic.oracle_tensor_list(meta, tensors)
        for b, P in enumerate(ctx_lens):
            ctx.bind_slot(b, perm[b * per_seq:(b + 1) * per_seq])
            ora = vo.Model(dict(meta, n_ctx=P + N + 1), tl)
            for l in range(L):
                k, v = _prefix_kv(g, P, Hkv)
                ora.write_kv(0, l, 0, k.astype(np.float32).reshape(P, -1))
                ora.write_kv(1, l, 0, v.astype(np.float32).reshape(P, -1))
                for p0 in range(0, P, 64):
                    ctx.write_kv(b, l, p0, k[p0:p0 + 64], v[p0:p0 + 64])
            oras.append(ora)
        slots = np.arange(B, dtype=np.uint32)
        cl = np.array(ctx_lens, np.int32)
        parents = np.tile(tree, (B, 1))
        # node tokens: a first pass gives the target's argmax after every node
        # of a random tree; children then take their parent's argmax with
        # probability 0.6, so paths of several nodes get accepted
        tokens = g.integers(0, V, (B, N)).astype(np.uint32)
        for _ in range(3):
            first = ctx.verify_step(slots, cl, tokens, parents, commit=False, n_vocab=V)
            for b in range(B):
                for n in range(1, N):
                    if g.random() < 0.6:
                        tokens[b, n] = first["expected"][b, tree[n]]
        res = ctx.verify_step(slots, cl, tokens, parents, commit=True, want_logits=True, n_vocab=V)
        got = res["logits"]
        for b, P in enumerate(ctx_lens):
            ref = oras[b].verify_tree(tokens[b], tree, P)
            err = np.abs(got[b] - ref).max()
            assert err <= TOL_LOGITS, (case, b, err)
            expected = np.array([vo.greedy(got[b, n])[0] for n in range(N)], np.uint32)
            assert np.array_equal(res["expected"][b], expected)
            path, bonus = vo.find_best_path(tree, tokens[b], expected)
            n_path = len(path)
            assert res["accepted_len"][b] == n_path - 1
            assert list(res["accepted_nodes"][b][:n_path]) == list(path)
            assert all(res["accepted_nodes"][b][n_path:] == -1)
            assert res["bonus"][b] == bonus
            oras[b].commit_path(path, P)
            for l in range(L):
                k, v = ctx.read_kv(b, l, P, n_path, Hkv)
                rk = oras[b].read_kv(0, l, P + n_path)[P:].reshape(n_path, Hkv, 128)
                rv = oras[b].read_kv(1, l, P + n_path)[P:].reshape(n_path, Hkv, 128)
                assert np.abs(k.astype(np.float32) - rk).max() <= TOL_LOGITS
                assert np.abs(v.astype(np.float32) - rv).max() <= TOL_LOGITS
        # at least one sequence accepted more than the root (the tree was built to)
        assert res["accepted_len"].max() >= 1
    finally:
        ctx.close()


def _gemm(ctx, q4, N, K, x16, mode, y_init=None, q4_b=None):
    import torch
    M = x16.shape[0]
    dev = torch.device("cuda")
    src = torch.from_numpy(np.ascontiguousarray(q4)).to(dev)
    src_b = None if q4_b is None else torch.from_numpy(np.ascontiguousarray(q4_b)).to(dev)
    w = torch.empty(velo_cuda.q4_0_repacked_bytes(N, K), dtype=torch.uint8, device=dev)
    # the context's own stream is not ordered after torch's: wait for every
    # copy before the library reads, and keep each buffer alive until it ran
    torch.cuda.synchronize()
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    try:
        ctx.q4_0_repack(src, N, K, w, src_b=src_b)
        ctx.sync()
        del src, src_b
        x = torch.from_numpy(x16).to(dev)
        ncol = N // 2 if mode == velo_cuda.EPI_SWIGLU else N
        dt = torch.float16 if mode == velo_cuda.EPI_SWIGLU else torch.float32
        if y_init is not None:
            y = torch.from_numpy(y_init).to(dev)
        else:
            y = torch.full((M, ncol), float("nan"), dtype=dt, device=dev)
        torch.cuda.synchronize()
        ctx.gemm_q4_0(w, x, M, N, K, y, ncol, mode)
        torch.cuda.synchronize()
        ctx.sync()
        out = y.float().cpu().numpy()
        del w, x, y
        torch.cuda.empty_cache()
    finally:
        ctx.set_stream(None)
    return out


# One config-5 layer at TP1 (M = 2048): fused QKV (8192 + 2 x 1024 outputs),
# o_proj / down_proj with the residual add, the w1/w3 SwiGLU pair and the LM
# head (128256 outputs).
@pytest.mark.parametrize("name,N,K,mode", [
    ("wqkv", 10240, 8192, velo_cuda.EPI_STORE_F32),
    ("w2_residual", 8192, 28672, velo_cuda.EPI_ADD_F32),
    ("w1w3_swiglu", 2 * 28672, 8192, velo_cuda.EPI_SWIGLU),
    ("lm_head", 128256, 8192, velo_cuda.EPI_STORE_F32),
])
def test_gemm_at_config5_shapes(ctx, name, N, K, mode):
    M = 2048
    x16 = synthetic.rng(21, 22).normal(0, 1, (M, K)).astype(np.float16)
    rows = np.sort(synthetic.rng(21, 23).choice(M, 48, replace=False))
    rows[-1] = M - 1  # the last tile's rows too
    if mode == velo_cuda.EPI_SWIGLU:
        F = N // 2
        q1 = synthetic.random_q4_0(F, K, 21, 24)
        q3 = synthetic.random_q4_0(F, K, 21, 25)
        y = _gemm(ctx, q1, N, K, x16, mode, q4_b=q3)
        xs = x16[rows].astype(np.float64)
        gt = xs @ synthetic.dequant_q4_0_f32(q1, F, K).astype(np.float64).T
        up = xs @ synthetic.dequant_q4_0_f32(q3, F, K).astype(np.float64).T
        ref = gt / (1.0 + np.exp(-gt)) * up
    else:
        q4 = synthetic.random_q4_0(N, K, 21, 26)
        resid = None
        if mode == velo_cuda.EPI_ADD_F32:
            resid = synthetic.rng(21, 27).normal(0, 1, (M, N)).astype(np.float32)
        y = _gemm(ctx, q4, N, K, x16, mode, y_init=resid)
        w = synthetic.dequant_q4_0_f32(q4, N, K)
        # the numpy dequantisation is the oracle's (quant.rs) bit for bit
        assert np.array_equal(w[:4], vo.dequant_matrix(2, q4[:4], 4, K))
        ref = x16[rows].astype(np.float64) @ w.astype(np.float64).T
        if resid is not None:
            ref += resid[rows]
    assert np.isfinite(y).all(), name
    # the SwiGLU output is stored as f16: its rounding (2^-11 relative) adds
    # to the bar for large values
    tol = TOL_LOGITS + (np.abs(ref) * 2.0 ** -10 if mode == velo_cuda.EPI_SWIGLU else 0.0)
    err = np.abs(y[rows] - ref)
    assert np.all(err <= tol), (name, err.max())
