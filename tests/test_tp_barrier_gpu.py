"""Failure detection of the tensor-parallel peer sums without a GPU fault: the
cross-rank barriers of the sum kernels wait on flags that other ranks set over
NVLink, and every wait gives up after 2 s.  On one GPU the gather kernel runs
as rank 0 of a group of 2 whose rank 1 never arrives (its flags are memory
nothing writes): the kernel returns with error 0x7101 (entry barrier), and the
context and device stay usable afterwards."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_peer_barrier_gives_up_and_reports():
    import torch
    import velo_cuda
    t0 = time.time()
    code = velo_cuda.tp_wait_selftest(0)
    dt = time.time() - t0
    assert code == 0x7101
    assert 3.5 <= dt <= 30.0  # the entry wait and the exit wait, 2 s each
    # the device still runs work
    x = torch.arange(1024, device="cuda:0", dtype=torch.float32)
    assert float(x.sum().item()) == float(np.arange(1024).sum())
