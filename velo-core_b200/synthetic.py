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
