"""The C ABI library loads and exports every function include/velo_cuda.h
declares; error conventions work without a GPU (no compute calls here)."""
import ctypes

import pytest

import velo_cuda


def test_library_exports_every_declared_symbol():
    lib = velo_cuda.lib()
    names = velo_cuda.header_functions()
    assert len(names) >= 8
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_wrapper_binds_every_declared_symbol():
    assert set(velo_cuda.header_functions()) <= set(velo_cuda._SIGS)


def test_abi_version():
    assert velo_cuda.lib().velo_cuda_abi_version() == 2


def test_create_rejects_bad_arguments():
    lib = velo_cuda.lib()
    h = ctypes.c_void_p()
    assert lib.velo_cuda_create(None, 0, 0, 1, None, None) == velo_cuda.ERR_INVALID_ARGUMENT
    assert "NULL" in velo_cuda.last_error()
    assert lib.velo_cuda_create(None, 0, 2, 1, None, ctypes.byref(h)) == velo_cuda.ERR_INVALID_ARGUMENT
    assert lib.velo_cuda_create(None, 0, 0, 2, None, ctypes.byref(h)) == velo_cuda.ERR_INVALID_ARGUMENT
    assert "NCCL" in velo_cuda.last_error()


def test_null_context_is_an_error_not_a_crash():
    lib = velo_cuda.lib()
    assert lib.velo_cuda_sync(None, 0) == velo_cuda.ERR_INVALID_ARGUMENT
    assert lib.velo_cuda_accept(None, None, None, None, None, 1, 1, 1, 0.0, None, None) \
        == velo_cuda.ERR_INVALID_ARGUMENT
    lib.velo_cuda_destroy(None)


def test_no_device_reports_no_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(velo_cuda.VeloError) as e:
        velo_cuda.Context(device=0)
    assert e.value.status == velo_cuda.ERR_NO_DEVICE
