"""Fused acceptance kernel vs the CPU oracle: accepted lengths and bonus tokens
must be bit-exact on the same logits and uniforms (greedy and sampling)."""
import numpy as np
import pytest

import synthetic
import velo_cuda
import vo

pytestmark = pytest.mark.gpu


def _both(ctx, tgt, drf, tok, u, T):
    a_gpu, b_gpu = ctx.accept(tgt, drf if T > 0 else None, tok, u, T)
    a_ref, b_ref = vo.accept(tgt, drf if T > 0 else None, tok, u, T)
    return (a_gpu, b_gpu), (a_ref, b_ref)


@pytest.mark.parametrize("T", [0.8, 0.0, 1.0])
def test_config2_full_size_bit_exact(ctx, T):
    """B=64, k=8, V=32000."""
    tgt, drf, tok, u = synthetic.acceptance_inputs(64, 8, 32000, temperature=T or 0.8)
    (ag, bg), (ar, br) = _both(ctx, tgt, drf, tok, u, T)
    assert np.array_equal(ag, ar)
    assert np.array_equal(bg, br)


@pytest.mark.parametrize("B,k,V", [(1, 1, 5), (3, 0, 4096), (5, 4, 1000), (4, 3, 1023),
                                   (2, 16, 2049), (2, 64, 300), (2, 2, 128256), (7, 5, 1024)])
@pytest.mark.parametrize("T", [0.7, 0.0])
def test_ragged_shapes_bit_exact(ctx, B, k, V, T):
    tgt, drf, tok, u = synthetic.acceptance_inputs(B, k, V, temperature=T or 0.7, seed=B * 31 + V)
    (ag, bg), (ar, br) = _both(ctx, tgt, drf, tok, u, T)
    assert np.array_equal(ag, ar), (ag, ar)
    assert np.array_equal(bg, br), (bg, br)


def test_device_entry_matches_host_entry(ctx):
    import torch
    tgt, drf, tok, u = synthetic.acceptance_inputs(16, 8, 32000)
    a_h, b_h = ctx.accept(tgt, drf, tok, u, 0.8)
    dev = lambda a: torch.from_numpy(a).cuda()
    acc = torch.empty(16, dtype=torch.int32, device="cuda")
    bonus = torch.empty(16, dtype=torch.int32, device="cuda")
    tok_d = torch.from_numpy(tok.view(np.int32)).cuda()
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    try:
        for _ in range(3):  # repeated launches reuse the self-resetting counters
            ctx.accept_device(dev(tgt), dev(drf), tok_d, dev(u), 0.8, acc, bonus)
            torch.cuda.synchronize()
            assert np.array_equal(acc.cpu().numpy(), a_h)
            assert np.array_equal(bonus.cpu().numpy().view(np.uint32), b_h)
    finally:
        ctx.set_stream(None)


def test_greedy_ties_take_last_max(ctx):
    """sampling.rs:49 / backend.rs:496-500 on device: equal maxima in
    different tiles and lanes -> the last index wins."""
    B, k, V = 4, 2, 5000
    tgt = np.zeros((B, k + 1, V), np.float32)
    for b in range(B):
        for i in range(k + 1):
            idx = np.random.default_rng(b * 10 + i).choice(V, 3, replace=False)
            tgt[b, i, idx] = 7.0
    tok = np.array([[np.flatnonzero(tgt[b, 0] == 7.0).max(), 0] for b in range(B)], np.uint32)
    (ag, bg), (ar, br) = _both(ctx, tgt, None, tok, None, 0.0)
    assert np.array_equal(ag, ar) and np.array_equal(bg, br)
    assert np.all(ag == 1)
    for b in range(B):
        assert bg[b] == np.flatnonzero(tgt[b, 1] == 7.0).max()


def test_identical_draft_accepts_everything(ctx):
    """p == q: u*q <= p always holds, so all k are accepted and the bonus is
    drawn from row k."""
    rng = np.random.default_rng(5)
    B, k, V = 8, 6, 3000
    tgt = rng.normal(0, 2, (B, k + 1, V)).astype(np.float32)
    drf = tgt[:, :k].copy()
    tok = rng.integers(0, V, (B, k)).astype(np.uint32)
    u = rng.random((B, k + 1)).astype(np.float32)
    (ag, bg), (ar, br) = _both(ctx, tgt, drf, tok, u, 0.9)
    assert np.all(ag == k) and np.array_equal(bg, br)


def test_invalid_token_is_rejected_on_host(ctx):
    tgt, drf, tok, u = synthetic.acceptance_inputs(2, 2, 100)
    tok[1, 1] = 100
    with pytest.raises(velo_cuda.VeloError) as e:
        ctx.accept(tgt, drf, tok, u, 0.8)
    assert e.value.status == velo_cuda.ERR_INVALID_ARGUMENT


def test_shape_changes_reuse_tag_block(ctx):
    """One context, launches of changing shapes (the fused kernel's tag block
    holds words of earlier launches at other offsets) and the one-kernel /
    two-kernel boundary (2k+1 rows <= 32 vs more): every launch bit-exact."""
    shapes = [(64, 8, 32000), (3, 15, 4096), (9, 16, 4096), (64, 8, 32000), (2, 1, 64000),
              (17, 7, 2048), (3, 15, 4096)]
    for n, (B, k, V) in enumerate(shapes):
        for T in (0.9, 0.0):
            tgt, drf, tok, u = synthetic.acceptance_inputs(B, k, V, temperature=T or 0.9, seed=n)
            (ag, bg), (ar, br) = _both(ctx, tgt, drf, tok, u, T)
            assert np.array_equal(ag, ar), (B, k, V, T)
            assert np.array_equal(bg, br), (B, k, V, T)
