"""Pins the CPU oracle to the reference's own known-answer tests.

Each test re-expresses one test of developertogo/velo-core (file:line given)
against oracle/velo_oracle.c.  These run on CPU only.
"""
import math

import numpy as np
import pytest

import vo


# ------------------------------------------------------------- src/quant.rs
def test_f16_basic_values():
    """quant.rs:210-225: 0 -> 0, 0x3C00 -> 1.0, 0xBC00 -> -1.0."""
    assert vo.f16_to_f32(0) == 0.0
    assert abs(vo.f16_to_f32(0x3C00) - 1.0) < 1e-6
    assert abs(vo.f16_to_f32(0xBC00) + 1.0) < 1e-6


def test_f16_edge_cases():
    """quant.rs:310-322: subnormal 2^-24, +-inf, NaN."""
    assert vo.f16_to_f32(0x0001) == 1.0 / (1 << 24)
    assert vo.f16_to_f32(0x8001) == -(1.0 / (1 << 24))
    assert math.isinf(vo.f16_to_f32(0x7C00))
    assert math.isinf(vo.f16_to_f32(0xFC00))
    assert math.isnan(vo.f16_to_f32(0x7C01))


def _block(delta, nib):
    return np.array([delta & 0xFF, delta >> 8] + [nib] * 16, np.uint8)


def test_q4_0_all_zeros():
    """quant.rs:240-249: delta 1.0, nibbles 0x88 -> all zeros."""
    out = vo.dequant_row(vo.Q4_0, _block(0x3C00, 0x88), 32)
    assert np.all(np.abs(out) < 1e-6)


def test_q4_0_scale_applies():
    """quant.rs:251-261: delta 2.0 (0x4000), nibbles 0x99 -> all 2.0."""
    out = vo.dequant_row(vo.Q4_0, _block(0x4000, 0x99), 32)
    assert np.all(np.abs(out - 2.0) < 1e-4)


def test_q4_0_interleaved_order():
    """quant.rs:57-63: element 2i is the low nibble, 2i+1 the high nibble."""
    blk = np.array([0x00, 0x3C] + [0x1F] + [0x88] * 15, np.uint8)  # byte0: lo=15, hi=1
    out = vo.dequant_row(vo.Q4_0, blk, 32)
    assert out[0] == 7.0 and out[1] == -7.0 and np.all(out[2:] == 0.0)


def test_dequant_f32_roundtrip_and_fallback():
    """quant.rs:263-308: f32 copy round-trips; unknown dtypes zero-fill."""
    vals = np.array([1.0, -2.5, 3.14, 0.0], np.float32)
    assert np.array_equal(vo.dequant_row(vo.F32, vals.view(np.uint8), 4), vals)
    assert np.array_equal(vo.dequant_row(99, np.zeros(100, np.uint8), 4), np.zeros(4))


def test_dequant_f16_matrix_multi_row():
    """quant.rs:324-334."""
    bits = np.array([0x3C00, 0x4000, 0x4200, 0x4400], np.uint16)
    out = vo.dequant_matrix(vo.F16, bits.view(np.uint8), 2, 2)
    assert out.ravel().tolist() == [1.0, 2.0, 3.0, 4.0]


def test_q4_0_quantiser_roundtrip():
    """Own quantiser: dequant(quant(x)) is within one step d = amax/8 of x (a
    full step only where +amax clips to nibble 15)."""
    rng = np.random.default_rng(0)
    x = rng.normal(0, 0.02, (4, 256)).astype(np.float32)
    q = vo.quantize_q4_0(x)
    y = vo.dequant_matrix(vo.Q4_0, q, 4, 256)
    step = np.abs(x.reshape(4, -1, 32)).max(-1, keepdims=True) / 8
    err = np.abs((x - y).reshape(4, -1, 32))
    assert np.all(err <= step * 1.001 + 1e-7)
    assert np.mean(err <= step * 0.5 * 1.001 + 1e-7) > 0.95


# ---------------------------------------------------------- src/llama_cpu.rs
def test_rms_norm_unit_weights():
    """llama_cpu.rs:428-436."""
    x = vo.rms_norm([1, 2, 3, 4], [1, 1, 1, 1], 1e-6)
    assert abs(math.sqrt(float(np.mean(x * x))) - 1.0) < 1e-4


def test_rms_norm_zero_safety():
    """llama_cpu.rs:482-488."""
    assert vo.rms_norm([0, 0], [1, 1], 1e-5).tolist() == [0.0, 0.0]


def test_softmax():
    """llama_cpu.rs:438-450: sums to one; the max element is largest."""
    s = vo.softmax([1, 2, 3])
    assert abs(float(s.sum()) - 1.0) < 1e-6
    s = vo.softmax([0.1, 10.0, 0.1])
    assert s[1] > s[0] and s[1] > s[2]


def test_silu():
    """llama_cpu.rs:452-460, 490-494, 540-543."""
    assert abs(vo.silu(0.0)) < 1e-7
    assert abs(vo.silu(-10.0)) < 1e-3
    assert 0.7 < vo.silu(1.0) < 0.8
    assert vo.silu(1.0) > 0


def test_matvec_identity():
    """llama_cpu.rs:462-470, 516-523, 545-554."""
    w = np.array([1, 0, 0, 1], np.float32)
    assert vo.matvec_quant(w.view(np.uint8), vo.F32, [1, 2], 2, 2).tolist() == [1.0, 2.0]
    assert vo.matvec_quant(w.view(np.uint8), vo.F32, [3, 4], 2, 2).tolist() == [3.0, 4.0]


def test_rope_preserves_norm():
    """llama_cpu.rs:556-564."""
    q0 = np.array([1, 0, 0, 1], np.float32)
    q, _ = vo.rope(q0, [0.5, 0.5, -0.5, -0.5], 0, 1, 1, 4, 10000.0)
    assert abs(np.linalg.norm(q0) - np.linalg.norm(q)) < 1e-4
    q, _ = vo.rope(q0, [0.5, 0.5, -0.5, -0.5], 7, 1, 1, 4, 10000.0)
    assert abs(np.linalg.norm(q0) - np.linalg.norm(q)) < 1e-4


def dummy_llama(n_vocab, n_embd, n_layer, tied=False):
    """model_loader.rs:236-285: all-zero f32 weights, 1 head, n_ff = 4*n_embd."""
    meta = dict(n_vocab=n_vocab, n_embd=n_embd, n_layer=n_layer, n_head=1, n_head_kv=1,
                n_ff=4 * n_embd, head_dim=n_embd, n_ctx=1024, rope_freq_base=10000.0,
                norm_eps=1e-5)
    z = lambda *s: (vo.F32, np.zeros(s, np.float32).view(np.uint8))
    t = [z(n_vocab, n_embd), z(n_embd), None if tied else z(n_vocab, n_embd)]
    for _ in range(n_layer):
        t += [z(n_embd), z(n_embd, n_embd), z(n_embd, n_embd), z(n_embd, n_embd),
              z(n_embd, n_embd), z(n_embd), z(4 * n_embd, n_embd), z(n_embd, 4 * n_embd),
              z(4 * n_embd, n_embd)]
    return vo.Model(meta, t)


def test_zero_weights_forward_gives_zero_logits():
    """llama_cpu.rs:525-538."""
    m = dummy_llama(32, 16, 1)
    logits = m.forward_one(1, 0)
    assert logits.shape == (32,) and np.all(logits == 0.0)


def test_tied_weights():
    """llama_cpu.rs:566-581: without output.weight the LM head is token_embd."""
    m = dummy_llama(32, 16, 1, tied=True)
    assert m.forward_one(1, 0).shape == (32,)


def test_forward_sequence_advances_pos():
    """llama_cpu.rs:583-592."""
    m = dummy_llama(32, 16, 1)
    assert m.forward_sequence([1, 2, 3]).shape == (32,)
    assert m.pos == 3


def test_verify_rows_per_node():
    """llama_cpu.rs:496-505 (verify returns one row per verified token).  The
    build's contract verifies root + drafts, one row per tree node."""
    m = dummy_llama(32, 16, 1)
    m.forward_sequence([1])
    rows = m.verify_tree([1, 2, 3], [-1, 0, 1], n_cached=0)
    assert rows.shape == (3, 32)


# ----------------------------------------------------------- src/sampling.rs
def test_greedy_selects_highest():
    """backend.rs:411-422 and sampling.rs:272-280."""
    assert vo.greedy([0.1, 0.8, 0.2])[0] == 1
    tok, conf = vo.greedy([1.0, 5.0, 2.0, 4.0])
    assert tok == 1 and conf == 5.0


def test_greedy_single_and_last_max():
    """backend.rs:487-500: one logit -> 0; ties -> the LAST maximal index."""
    tok, conf = vo.greedy([0.5])
    assert tok == 0 and conf == 0.5
    assert vo.greedy([0.5, 0.5])[0] == 1


def test_greedy_with_mask():
    """sampling.rs:282-293."""
    tok, conf = vo.greedy([1.0, 5.0, 2.0, 4.0], mask=[1, 0, 1, 0])
    assert tok == 2 and conf == 2.0


def test_greedy_nan_is_skipped():
    """sampling.rs:49 compares with >=, so NaN never wins; all-NaN -> 0."""
    assert vo.greedy([1.0, float("nan"), 0.5])[0] == 0
    assert vo.greedy([float("nan")] * 3)[0] == 0


def test_argmax_kat_token_1234():
    """tests/metal_perf_tests.rs:53-66: V=32000, logits -1 except 100 at 1234."""
    lg = np.full(32000, -1.0, np.float32)
    lg[1234] = 100.0
    assert vo.greedy(lg)[0] == 1234


# -------------------------------------------------------- src/speculative.rs
def test_tree_best_path():
    """speculative.rs:796-825."""
    parents = [-1, 0, 0, 1]
    tokens = [10, 20, 30, 40]
    path, bonus = vo.find_best_path(parents, tokens, [30, 99, 99, 99])
    assert [tokens[i] for i in path] == [10, 30] and bonus == 99
    path, bonus = vo.find_best_path(parents, tokens, [20, 40, 99, 99])
    assert [tokens[i] for i in path] == [10, 20, 40] and bonus == 99


def test_tree_best_path_ties_to_later_node():
    """speculative.rs:116 uses >=, so among equal lengths the later node wins."""
    parents = [-1, 0, 0]
    path, bonus = vo.find_best_path(parents, [5, 7, 7], [7, 1, 2])
    assert path == [0, 2] and bonus == 2


# ---------------------------------------------------- src/paged_attention.rs
def test_allocator_fixed_budget():
    """paged_attention.rs:237-258: 24 tokens, block 16, 4 pages -> 2 pages."""
    a = vo.Allocator(16, 4)
    pages = a.allocate(1, 24)
    assert len(pages) == 2 and a.free_pages() == 2
    assert vo.pages_for_tokens(24, 16) == 2


def test_allocator_release():
    """paged_attention.rs:260-280."""
    a = vo.Allocator(8, 2)
    a.allocate(2, 8)
    a.release(2)
    assert a.free_pages() == 2


def test_allocator_out_of_pages():
    """paged_attention.rs:282-305: OutOfPages{requested: 2, available: 1}."""
    a = vo.Allocator(32, 1)
    with pytest.raises(vo.OutOfPages) as e:
        a.allocate(3, 64)
    assert (e.value.requested, e.value.available) == (2, 1)


def test_allocator_unknown_handle_and_bad_block():
    """paged_attention.rs:313-317 and :103-106."""
    a = vo.Allocator(16, 32)
    with pytest.raises(KeyError):
        a.release(1)
    with pytest.raises(ValueError):
        vo.Allocator(0, 4)


def test_allocator_fifo_order():
    """paged_attention.rs:126-137, 171-176, 194-196: FIFO free list."""
    a = vo.Allocator(16, 4)
    assert a.allocate(1, 16) == [0]
    assert a.allocate(2, 32) == [1, 2]
    a.release(1)
    assert a.allocate(3, 32) == [3, 0]
