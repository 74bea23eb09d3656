"""q4_0 tensor-core GEMM (velo_cuda_gemm_q4_0) against the CPU oracle.

Two bars: (1) against the oracle's fp32 dequantisation of the same q4_0 bytes
(src/quant.rs:50-73, llama_cpu.rs:75-90 matvec_quant) within the verify step's
logit tolerance 2e-2 max-abs; (2) against a float64 product of the f16-rounded
weights the tensor cores consume, within 1e-3 of the output scale (fp32
accumulation order only)."""
import numpy as np
import pytest

import synthetic
import velo_cuda
import vo

pytestmark = pytest.mark.gpu

TOL_ORACLE = 2e-2


def _run(ctx, q4, N, K, x16, mode, y_init=None, q4_b=None):
    import torch
    M = x16.shape[0]
    dev = torch.device("cuda")
    src = torch.from_numpy(np.ascontiguousarray(q4)).to(dev)
    src_b = None if q4_b is None else torch.from_numpy(np.ascontiguousarray(q4_b)).to(dev)
    w = torch.empty(velo_cuda.q4_0_repacked_bytes(N, K), dtype=torch.uint8, device=dev)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    try:
        ctx.q4_0_repack(src, N, K, w, src_b=src_b)
        x = torch.from_numpy(x16).to(dev)
        ncol = N // 2 if mode == velo_cuda.EPI_SWIGLU else N
        dt = torch.float16 if mode in (velo_cuda.EPI_STORE_F16, velo_cuda.EPI_SWIGLU) else torch.float32
        if y_init is not None:
            y = torch.from_numpy(y_init.copy()).to(dev)
        else:
            y = torch.full((M, ncol), float("nan"), dtype=dt, device=dev)
        ctx.gemm_q4_0(w, x, M, N, K, y, ncol, mode)
        torch.cuda.synchronize()
        ctx.sync()
    finally:
        ctx.set_stream(None)
    return y.float().cpu().numpy()


def _inputs(M, N, K, seed):
    q4 = synthetic.q4_0_weights(N, K, seed=seed)
    x16 = synthetic.rng(seed, 20).normal(0, 1, (M, K)).astype(np.float16)
    return q4, x16


# M <= 128 takes the shared-memory-weight kernel (256-row weight tiles when there are >= 148 of
# them, else 128); M > 128 the kernel with the dequantised weights in tensor memory, with
# 128-row activation tiles except at many waves ((2048, 10240, 256): 256-row tiles).
@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (5, 300, 96), (128, 512, 256), (200, 1000, 512),
                                   (512, 4096, 4096), (130, 256, 11008), (640, 7680, 512),
                                   (512, 12288, 1024), (2048, 10240, 256), (300, 700, 96),
                                   # odd k-tile counts (the kernels step over two 64-k tiles)
                                   (384, 640, 192), (260, 1024, 4160)])
def test_gemm_f32_matches_oracle(ctx, M, N, K):
    q4, x16 = _inputs(M, N, K, seed=M + N + K)
    y = _run(ctx, q4, N, K, x16, velo_cuda.EPI_STORE_F32)
    w32 = vo.dequant_matrix(2, q4, N, K).astype(np.float64)
    ref = x16.astype(np.float64) @ w32.T
    assert np.isfinite(y).all()
    assert np.abs(y - ref).max() <= TOL_ORACLE, np.abs(y - ref).max()
    w16 = synthetic.dequant_q4_0_f16(q4, N, K).astype(np.float64)
    ref16 = x16.astype(np.float64) @ w16.T
    scale = max(1.0, np.abs(ref16).max())
    assert np.abs(y - ref16).max() <= 1e-3 * scale


@pytest.mark.parametrize("mode", [0, 2, 3])
def test_weight_paths_agree(ctx, monkeypatch, mode):
    # M > 128: weights as the TMEM A operand (VELO_Q4_GEMM=tmem; the default
    # except for SwiGLU) or as the shared-memory B operand (=smem) agree
    M, N, K = 384, 1024, 1024
    q4, x16 = _inputs(M, N, K, seed=31 + mode)
    q4_b = _inputs(M, N // 2, K, seed=77)[0][: N // 2] if mode == velo_cuda.EPI_SWIGLU else None
    if mode == velo_cuda.EPI_SWIGLU:
        q4 = q4[: N // 2]
    resid = synthetic.rng(4, 4).normal(0, 1, (M, N)).astype(np.float32) if mode == velo_cuda.EPI_ADD_F32 else None
    monkeypatch.setenv("VELO_Q4_GEMM", "tmem")
    ta = _run(ctx, q4, N, K, x16, mode, y_init=resid, q4_b=q4_b)
    monkeypatch.setenv("VELO_Q4_GEMM", "smem")
    sm = _run(ctx, q4, N, K, x16, mode, y_init=resid, q4_b=q4_b)
    assert np.isfinite(ta).all() and np.isfinite(sm).all()
    scale = max(1.0, np.abs(sm).max())
    assert np.abs(ta - sm).max() <= 1e-3 * scale, np.abs(ta - sm).max()


def test_gemm_f16_and_residual_add(ctx):
    M, N, K = 256, 768, 1024
    q4, x16 = _inputs(M, N, K, seed=7)
    w32 = vo.dequant_matrix(2, q4, N, K).astype(np.float64)
    ref = x16.astype(np.float64) @ w32.T
    y16 = _run(ctx, q4, N, K, x16, velo_cuda.EPI_STORE_F16)
    assert np.abs(y16 - ref).max() <= TOL_ORACLE
    resid = synthetic.rng(3, 3).normal(0, 1, (M, N)).astype(np.float32)
    ya = _run(ctx, q4, N, K, x16, velo_cuda.EPI_ADD_F32, y_init=resid)
    assert np.abs(ya - (resid + ref)).max() <= TOL_ORACLE


@pytest.mark.parametrize("M,F,K", [(64, 688, 256), (512, 1408, 1024), (1280, 2048, 256), (200, 688, 96),
                                   (300, 640, 192), (256, 512, 4160)])
def test_gemm_swiglu_pair(ctx, M, F, K):
    """w1 (gate) and w3 (up) repacked as a pair: y = silu(x w1^T) * (x w3^T),
    llama_cpu.rs:326-341."""
    q1 = synthetic.q4_0_weights(F, K, seed=11)
    q3 = synthetic.q4_0_weights(F, K, seed=12)
    x16 = synthetic.rng(5, 20).normal(0, 1, (M, K)).astype(np.float16)
    y = _run(ctx, q1, 2 * F, K, x16, velo_cuda.EPI_SWIGLU, q4_b=q3)
    g = x16.astype(np.float64) @ vo.dequant_matrix(2, q1, F, K).astype(np.float64).T
    u = x16.astype(np.float64) @ vo.dequant_matrix(2, q3, F, K).astype(np.float64).T
    ref = g / (1.0 + np.exp(-g)) * u
    assert np.abs(y - ref).max() <= TOL_ORACLE


def test_gemm_repeated_launches_identical(ctx):
    M, N, K = 384, 1024, 2048
    q4, x16 = _inputs(M, N, K, seed=99)
    a = _run(ctx, q4, N, K, x16, velo_cuda.EPI_STORE_F32)
    b = _run(ctx, q4, N, K, x16, velo_cuda.EPI_STORE_F32)
    assert np.array_equal(a, b)


# (512, 4096, 11008) is config 3's down_proj: 64 tiles on 148 SMs, so k is split and the
# partial sums of each tile meet in the residual; (384, 1536, 4160): an odd step count split
@pytest.mark.parametrize("M,N,K", [(300, 700, 96), (2000, 4096, 1024), (512, 4096, 11008),
                                   (384, 1536, 4160)])
def test_residual_add_ragged(ctx, M, N, K):
    # the TMEM-weight kernel adds its tile into the residual with one reduction
    # per element: ragged rows and columns stay untouched outside [M) x [N)
    q4, x16 = _inputs(M, N, K, seed=M + 3 * N)
    resid = synthetic.rng(9, 9).normal(0, 1, (M, N)).astype(np.float32)
    y = _run(ctx, q4, N, K, x16, velo_cuda.EPI_ADD_F32, y_init=resid)
    w32 = vo.dequant_matrix(2, q4, N, K).astype(np.float64)
    ref = resid.astype(np.float64) + x16.astype(np.float64) @ w32.T
    assert np.abs(y - ref).max() <= TOL_ORACLE

