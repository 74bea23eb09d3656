"""velo_cuda_accept_static, the acceptance entry point that allocates nothing.

Callers such as engines that own all device memory through their own pools
cannot let a library call cudaMalloc on the decode path; this entry keeps its
statistics in a fixed block inside the library instead.  Its outputs must equal
those of velo_cuda_accept_device (integer outputs: bit-exact) on the same
inputs, on two calls in a row (the block is reused and keeps stale contents).
This file is collected last so a failure here comes after every other test.
"""
import numpy as np
import pytest

import synthetic
import velo_cuda

pytestmark = pytest.mark.gpu


def _device(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("B,k,V,T", [(64, 8, 32000, 0.8), (64, 8, 32000, 0.0), (5, 3, 1000, 0.7)])
def test_static_matches_context_entry_twice(cuda_device, B, k, V, T):
    import torch
    tgt, drf, tok, u = synthetic.acceptance_inputs(B, k, V, temperature=T or 0.8, seed=7)
    t_d, d_d, u_d = _device(tgt), _device(drf), _device(u)
    tok_d = _device(tok.view(np.int32))
    acc_ref = torch.empty(B, dtype=torch.int32, device="cuda")
    bon_ref = torch.empty(B, dtype=torch.int32, device="cuda")
    with velo_cuda.Context(device=cuda_device) as ctx:
        ctx.accept_device(t_d, d_d if T else None, tok_d, u_d if T else None, T, acc_ref, bon_ref)
        ctx.sync()
    for _ in range(2):
        acc = torch.full((B,), -7, dtype=torch.int32, device="cuda")
        bon = torch.full((B,), -7, dtype=torch.int32, device="cuda")
        velo_cuda.accept_static(t_d, d_d if T else None, tok_d, u_d if T else None, T, acc, bon)
        torch.cuda.synchronize()
        assert torch.equal(acc, acc_ref)
        assert torch.equal(bon, bon_ref)


def test_static_rejects_sizes_beyond_its_block(cuda_device):
    import torch
    B, k, V = 1024, 64, 128 * 1024  # statistics far larger than the fixed block
    t = torch.empty((1,), device="cuda")
    with pytest.raises(velo_cuda.VeloError) as e:
        velo_cuda.check(velo_cuda.lib().velo_cuda_accept_static(
            velo_cuda._ptr(t), velo_cuda._ptr(t), velo_cuda._ptr(t), velo_cuda._ptr(t), B, k, V,
            0.8, velo_cuda._ptr(t), velo_cuda._ptr(t), None))
    assert e.value.status == velo_cuda.ERR_INVALID_ARGUMENT
    assert "scratch" in e.value.message


def test_static_reports_bad_tokens_through_its_error_word(cuda_device):
    """A draft token >= V is counted as a rejection on the device (the static
    entry cannot fail the call once it is queued); its error word says so, and
    the next call clears it."""
    import torch
    B, k, V, T = 5, 3, 1000, 0.7
    tgt, drf, tok, u = synthetic.acceptance_inputs(B, k, V, temperature=T, seed=9)
    bad = tok.copy()
    bad[2, 1] = V + 5
    t_d, d_d, u_d = _device(tgt), _device(drf), _device(u)
    acc = torch.empty(B, dtype=torch.int32, device="cuda")
    bon = torch.empty(B, dtype=torch.int32, device="cuda")
    flag = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    velo_cuda.accept_static(t_d, d_d, _device(bad.view(np.int32)), u_d, T, acc, bon)
    velo_cuda.accept_static_error(flag)
    torch.cuda.synchronize()
    assert int(flag.item()) != 0
    assert int(acc[2].item()) <= 1  # the bad token ends the accepted prefix
    velo_cuda.accept_static(t_d, d_d, _device(tok.view(np.int32)), u_d, T, acc, bon)
    velo_cuda.accept_static_error(flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0

