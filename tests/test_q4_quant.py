"""CPU checks of the q4_0 host helpers: the numpy quantiser used to build
synthetic weights is byte-identical to the oracle's, and the f16 dequant model
of the GEMM's operand agrees with the oracle's fp32 dequant to f16 rounding."""
import numpy as np

import synthetic
import velo_cuda
import vo


def test_numpy_quantiser_matches_oracle():
    w = synthetic.rng(0, 10).normal(0, 0.02, (64, 256)).astype(np.float32)
    w[3, :32] = 0.0                    # all-zero block -> d = 0
    w[5, 7] = 1.0                      # positive max
    w[6, 9] = -1.0                     # negative max
    assert np.array_equal(synthetic.quantize_q4_0(w), vo.quantize_q4_0(w))


def test_f16_operand_model():
    q4 = synthetic.q4_0_weights(32, 128, seed=3)
    w32 = vo.dequant_matrix(2, q4, 32, 128)
    w16 = synthetic.dequant_q4_0_f16(q4, 32, 128)
    assert np.array_equal(w16, w32.astype(np.float16))


def test_repacked_bytes():
    # tiles of 256 rows x 64 elements, 36 bytes per row and tile (32 nibble + 4 scale)
    assert velo_cuda.q4_0_repacked_bytes(4096, 4096) == 16 * 64 * 9216
    assert velo_cuda.q4_0_repacked_bytes(300, 96) == 2 * 2 * 9216
    assert velo_cuda.q4_0_repacked_bytes(10, 33) == 0


def test_kv_int8_quantiser_matches_oracle():
    x = synthetic.rng(0, 31).normal(0, 1, (40, 128)).astype(np.float32)
    x[3] = 0.0
    q, s = synthetic.quantize_kv_int8(x)
    for r in range(x.shape[0]):
        rq, rs = vo.quantize_kv_int8(x[r])
        assert np.array_equal(q[r], rq)
        assert s[r].view(np.uint16) == rs
