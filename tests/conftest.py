"""Shared test setup.

Paths: the product package (velo-core_b200/, a directory name with a dash, so
it is put on sys.path and imported as `velo_cuda`) and the CPU oracle
(oracle/, test infrastructure).  The `gpu` marker selects tests that need a
B200; everything else runs on a CPU-only machine.
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "velo-core_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")


def _ensure_built():
    if not os.path.exists(os.path.join(ORACLE, "libvelo_oracle.so")):
        subprocess.check_call(["make", "-s", "-C", ORACLE])
    if not os.path.exists(os.path.join(PKG, "libvelo_cuda.so")):
        subprocess.check_call([sys.executable, os.path.join(PKG, "build.py")])


_ensure_built()


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test collected on a machine without a CUDA device")
    torch.cuda.init()
    return 0


@pytest.fixture(scope="session")
def ctx(cuda_device):
    import velo_cuda
    c = velo_cuda.Context(device=cuda_device)
    yield c
    c.close()
