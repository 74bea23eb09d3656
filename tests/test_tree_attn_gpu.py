"""Tree-masked paged attention (velo_cuda_tree_attention) against the CPU
oracle (oracle/velo_oracle.c vo_tree_attention: the semantics of
kernels.metal:512-599 / 672-732 in double precision).

Tolerance 1e-2 max-abs on outputs of magnitude ~1: the kernel multiplies f16
Q/K/V (exact inputs) on the tensor cores with fp32 accumulation and rounds the
probabilities to f16 for the PV product (relative 2^-11 per weight)."""
import numpy as np
import pytest

import synthetic
import velo_cuda
import vo

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _gpu(ctx, d, n_kv, out_f16=False):
    import torch
    dev = torch.device("cuda")
    T = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    q = T(d["q"])
    B, N, Hq, hd = q.shape
    out = torch.full((B, N, Hq, hd), float("nan"), device=dev,
                     dtype=torch.float16 if out_f16 else torch.float32)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    try:
        ctx.tree_attention(q, T(d["k_pool"]), T(d["v_pool"]),
                           T(None if d["k_scale"] is None else d["k_scale"].view(np.uint16)),
                           T(None if d["v_scale"] is None else d["v_scale"].view(np.uint16)),
                           T(d["page_table"]), T(d["ctx_len"]), T(d["node_k"]), T(d["node_v"]),
                           T(d["parents"]), n_kv, d["kv_dtype"], out)
        torch.cuda.synchronize()
        ctx.sync()
    finally:
        ctx.set_stream(None)
    return out.float().cpu().numpy()


def _oracle(d, n_head, n_kv):
    B = d["q"].shape[0]
    res = []
    for b in range(B):
        res.append(vo.tree_attention(
            d["q"][b].astype(np.float32), d["kv_dtype"], d["k_pool"], d["v_pool"],
            None if d["k_scale"] is None else d["k_scale"].view(np.uint16),
            None if d["v_scale"] is None else d["v_scale"].view(np.uint16),
            d["page_table"][b], int(d["ctx_len"][b]), d["node_k"][b].view(np.uint16),
            d["node_v"][b].view(np.uint16), d["parents"][b], n_head, n_kv, 128, 16))
    return np.stack(res)


@pytest.mark.parametrize("kv_dtype", [0, 1])
@pytest.mark.parametrize("B,N,Hq,Hkv,ctx_lens", [
    (3, 16, 8, 2, [0, 100, 700]),          # empty cache, ragged last tile
    (2, 64, 32, 8, [600, 1500]),           # config-4 head shape: 256 rows, 2 CTAs per head
    (2, 16, 4, 4, [64, 2048]),             # config-3 head shape (no GQA), exact tiles
    (1, 1, 8, 1, [333]),                   # single node, GQA 8
    (2, 33, 16, 2, [17, 4099]),            # odd node count, 264 rows -> 3 row tiles
    (2, 40, 32, 8, [0, 1000]),             # 160 rows: second query tile a quarter full
    (1, 64, 64, 8, [2500])])               # 512 rows: two CTAs of two query tiles
def test_tree_attention_matches_oracle(ctx, kv_dtype, B, N, Hq, Hkv, ctx_lens):
    d = synthetic.tree_attention_inputs(B, N, Hq, Hkv, ctx_lens, kv_dtype=kv_dtype, seed=B * 7 + N)
    got = _gpu(ctx, d, Hkv)
    ref = _oracle(d, Hq, Hkv)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max()
    assert err <= TOL, err


@pytest.mark.parametrize("kv_dtype", [0, 1])
def test_one_and_two_query_tiles_agree(ctx, monkeypatch, kv_dtype):
    # 256 rows per KV head in one CTA of two query tiles or two CTAs of one
    # (VELO_ATTN_QUERY_TILES forces the layout); both meet the oracle
    d = synthetic.tree_attention_inputs(2, 64, 32, 8, [700, 2100], kv_dtype=kv_dtype, seed=11)
    monkeypatch.setenv("VELO_ATTN_QUERY_TILES", "2")
    two = _gpu(ctx, d, 8)
    monkeypatch.setenv("VELO_ATTN_QUERY_TILES", "1")
    one = _gpu(ctx, d, 8)
    ref = _oracle(d, 32, 8)
    assert np.abs(two - ref).max() <= TOL
    assert np.abs(one - ref).max() <= TOL
    assert np.abs(two - one).max() <= TOL


def test_tree_attention_f16_output_and_repeat(ctx):
    d = synthetic.tree_attention_inputs(2, 64, 32, 8, [900, 3000], kv_dtype=1, seed=5)
    a = _gpu(ctx, d, 8, out_f16=True)
    b = _gpu(ctx, d, 8, out_f16=True)
    assert np.array_equal(a, b)
    ref = _oracle(d, 32, 8)
    assert np.abs(a - ref).max() <= TOL


def test_tree_attention_rejects_bad_parents(ctx):
    d = synthetic.tree_attention_inputs(1, 8, 8, 2, [64], seed=1)
    d["parents"] = d["parents"].copy()
    d["parents"][0, 5] = 7  # parent after the child
    with pytest.raises(velo_cuda.VeloError) as e:
        _gpu(ctx, d, 2)
    assert e.value.status == velo_cuda.ERR_DEVICE_FLAG
