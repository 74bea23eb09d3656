"""The FMA-pipe exponential the attention softmax uses for a quarter of its
keys (exp2_fma2 in velo-core_b200/csrc/kernels/tree_attn.cu), restated step by
step in float32 (each add rounded, each fused multiply-add rounded once) and
checked against 2^y in float64: relative error below 1e-4 for y in [-125, 0]
(below that the results are subnormal floats that f16 rounds to 0 anyway),
i.e. below the 2^-11 rounding P takes on its way to f16, and masked keys
(-inf) vanish in f16."""
import numpy as np

C = [0.99992824, 0.69326094, 0.24260852, 0.0551705]
MAGIC = np.float32(12582912.0)


def _rn(x):
    return np.asarray(x, np.float64).astype(np.float32)


def exp2_fma(y):
    y = np.maximum(np.asarray(y, np.float32), np.float32(-126.0))
    t = _rn(y.astype(np.float64) + MAGIC)
    jf = _rn(t.astype(np.float64) - MAGIC)
    f = _rn(y.astype(np.float64) - jf)
    c = [np.float32(v) for v in C]
    p = _rn(c[3] * f.astype(np.float64) + c[2])  # exact product of two floats, one rounding
    p = _rn(p.astype(np.float64) * f + c[1])
    p = _rn(p.astype(np.float64) * f + c[0])
    j = t.view(np.int32) - MAGIC.view(np.int32)
    return (p.view(np.int32) + (j << 23)).view(np.float32)


def test_relative_error_over_the_softmax_domain():
    y = np.linspace(-125.0, 0.0, 4_000_001).astype(np.float32)
    r = exp2_fma(y).astype(np.float64)
    ref = np.exp2(y.astype(np.float64))
    rel = np.abs(r / ref - 1.0)
    assert rel.max() < 1e-4, rel.max()
    assert rel.max() < 2.0 ** -11


def test_masked_keys_vanish():
    r = exp2_fma(np.array([-np.inf, -200.0, -126.0], np.float32))
    assert np.all(r.astype(np.float16) == 0)
    assert np.all(r < 1e-37)


def test_exact_powers_of_two():
    y = np.arange(-20, 1, dtype=np.float32)
    r = exp2_fma(y).astype(np.float64)
    assert np.all(np.abs(r / np.exp2(y.astype(np.float64)) - 1) < 1e-4)
