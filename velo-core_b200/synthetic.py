"""Seeded synthetic inputs for the verify-step workloads.

No public dataset is involved: every config is defined by shapes and value
distributions, generated here from numpy's Philox bit generator with seed 0
(one independent stream per tensor, `stream` below), so that the CUDA path and
the CPU oracle consume the same bytes.
"""
import numpy as np


def rng(seed=0, stream=0):
    """Philox counter-based generator; `stream` selects an independent key."""
    return np.random.Generator(np.random.Philox(key=seed * 1000003 + stream))


def softmax64(x, axis=-1):
    x = x.astype(np.float64)
    x = x - x.max(axis=axis, keepdims=True)
    e = np.exp(x)
    return e / e.sum(axis=axis, keepdims=True)


def acceptance_inputs(B=64, k=8, V=32000, temperature=0.8, seed=0, target_sigma=2.0,
                      draft_sigma=0.5):
    """Acceptance microbench.

    target logits ~ N(0, target_sigma^2)            [B][k+1][V] f32
    draft logits  = target rows 0..k-1 + N(0, draft_sigma^2)   [B][k][V] f32
    draft tokens  sampled from q = softmax(draft/T) (stream seed+1)
    uniforms      U(0,1): one per draft position + one residual draw [B][k+1]
    """
    tgt = rng(seed, 0).normal(0.0, target_sigma, (B, k + 1, V)).astype(np.float32)
    drf = (tgt[:, :k] + rng(seed, 1).normal(0.0, draft_sigma, (B, k, V))).astype(np.float32)
    g = rng(seed + 1, 2)
    tok = np.zeros((B, k), np.uint32)
    T = temperature if temperature > 0 else 1.0
    for b in range(B):
        q = softmax64(drf[b] / T)
        c = np.cumsum(q, axis=-1)
        uu = g.random(k)
        tok[b] = np.minimum((c < uu[:, None]).sum(-1), V - 1)
    u = rng(seed, 3).random((B, k + 1)).astype(np.float32)
    return tgt, drf, tok, u


def quantize_q4_0(x):
    """[rows][cols] float32 -> [rows][cols/32*18] uint8 q4_0 in velo-core's
    interleaved order (src/quant.rs:50-64: byte i of a block holds element 2i
    in the low nibble and 2i+1 in the high nibble).  Per 32-block: m = the
    element of largest magnitude, d = m / -8 (f32, stored as f16),
    q = clamp(trunc(x * (1/d) + 8.5), 0, 15) in f32 arithmetic."""
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    assert cols % 32 == 0
    xb = x.reshape(rows, cols // 32, 32)
    idx = np.abs(xb).argmax(axis=-1)
    m = np.take_along_axis(xb, idx[..., None], axis=-1)[..., 0]
    d = (m / np.float32(-8.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    qf = (xb * inv[..., None]).astype(np.float32) + np.float32(8.5)
    q = np.clip(np.trunc(qf), 0, 15).astype(np.uint8)
    out = np.zeros((rows, cols // 32, 18), np.uint8)
    out[..., 0:2] = d.astype(np.float16).view(np.uint8).reshape(rows, cols // 32, 2)
    out[..., 2:] = q[..., 0::2] | (q[..., 1::2] << 4)
    return out.reshape(rows, cols // 32 * 18)


def dequant_q4_0_f16(data, rows, cols):
    """The f16 weights the tensor-core GEMM multiplies: f16(d * (q - 8)),
    one rounding of the exact product."""
    blk = np.ascontiguousarray(data, np.uint8).reshape(rows, cols // 32, 18)
    d = blk[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    q = np.empty((rows, cols // 32, 32), np.float32)
    q[..., 0::2] = (blk[..., 2:] & 15).astype(np.float32) - 8
    q[..., 1::2] = (blk[..., 2:] >> 4).astype(np.float32) - 8
    return (d[..., None] * q).astype(np.float16).reshape(rows, cols)


def q4_0_weights(rows, cols, sigma=0.02, seed=0, stream=10):
    """Random-init weight N(0, sigma^2), quantised to q4_0."""
    w = rng(seed, stream).normal(0.0, sigma, (rows, cols)).astype(np.float32)
    return quantize_q4_0(w)
