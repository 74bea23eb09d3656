"""The fp32 path of the verify step (an f32 KV pool: f32 weights, f32 pages,
FFMA kernels) on the CPU-runnable tiny Llama pair (hidden 256, 4 heads x 64,
FFN 688, vocab 4096) against the CPU oracle of LlamaCpuModel
(src/llama_cpu.rs:191-358, f32 math over f32 weights):

- logits of every node within 1e-4 max-abs (the fp32 bar);
- prefill K/V and the committed path's K/V equal to the oracle's cache within
  1e-5 (f32 pages);
- greedy tree decisions and rejection-sampling decisions bit-exact against
  the oracle's rules applied to the same (GPU) logits;
- a whole speculative session (64-token prompt, k = 4 fixed window, 128 new
  tokens) equal to the same session over the oracle's models."""
import numpy as np
import pytest

import synthetic
import velo_cuda
import vo
from speculative import (CudaDraft, CudaTarget, NextTokenPrediction, SpeculativeDecoder,
                         VerifyStep, sample_token)
from test_speculative_gpu import OracleDraft, OracleTarget

pytestmark = pytest.mark.gpu

TOL_LOGITS = 1e-4
TOL_KV = 1e-5


def _ctx(pages=32, slots=2):
    return velo_cuda.Context(device=0, kv_dtype=velo_cuda.KV_F32, total_pages=pages,
                             max_slots=slots, max_pages_per_slot=pages // slots)


def test_f32_prefill_tree_verify_commit():
    tm, tw, _, _ = synthetic.c1_pair()
    V, Hkv, hd = tm["n_vocab"], tm["n_head_kv"], tm["head_dim"]
    g = synthetic.rng(0, 90)
    prompt = g.integers(0, V, 64).astype(np.uint32)
    P = len(prompt) - 1  # cached tokens; the last prompt token is the tree root
    ora = vo.Model(dict(tm, n_ctx=512), synthetic.oracle_tensor_list(tm, tw))
    ora.forward_sequence(prompt[:P])
    with _ctx() as ctx:
        ctx.load_model(tm, tw)
        pages = g.permutation(32)[:16].astype(np.uint32)
        ctx.bind_slot(1, pages)
        velo_cuda.prefill(ctx, 1, prompt[:P], n_vocab=V)
        for l in range(tm["n_layer"]):
            k, v = ctx.read_kv(1, l, 0, P, Hkv, head_dim=hd)
            np.testing.assert_allclose(k.reshape(P, -1), ora.read_kv(0, l, P), atol=TOL_KV, rtol=0)
            np.testing.assert_allclose(v.reshape(P, -1), ora.read_kv(1, l, P), atol=TOL_KV, rtol=0)
        # a 9-node tree whose first branch follows the target's argmax
        parents = np.array([-1, 0, 1, 2, 0, 4, 1, 6, 3], np.int32)
        tokens = g.integers(0, V, len(parents)).astype(np.uint32)
        tokens[0] = prompt[P]
        for n in (1, 2, 3, 8):
            lg = ora.verify_tree(tokens[:n], parents[:n], P)
            tokens[n] = vo.greedy(lg[parents[n]])[0]
        ref = ora.verify_tree(tokens, parents, P)
        r = ctx.verify_step([1], [P], tokens[None], parents[None], commit=True, want_logits=True,
                            n_vocab=V)
        lg = r["logits"][0]
        assert np.abs(lg - ref).max() <= TOL_LOGITS
        exp = np.array([vo.greedy(lg[n])[0] for n in range(len(parents))], np.uint32)
        path, bonus = vo.find_best_path(parents, tokens, exp)
        acc = int(r["accepted_len"][0])
        assert acc == len(path) - 1 and acc >= 3
        assert list(r["accepted_nodes"][0][:acc + 1]) == list(path)
        assert int(r["bonus"][0]) == bonus
        ora.commit_path(list(path), P)
        n_path = len(path)
        for l in range(tm["n_layer"]):
            k, v = ctx.read_kv(1, l, P, n_path, Hkv, head_dim=hd)
            np.testing.assert_allclose(k.reshape(n_path, -1), ora.read_kv(0, l, P + n_path)[P:],
                                       atol=TOL_KV, rtol=0)
            np.testing.assert_allclose(v.reshape(n_path, -1), ora.read_kv(1, l, P + n_path)[P:],
                                       atol=TOL_KV, rtol=0)


def test_f32_sampling_chain_bit_exact():
    """T = 1.0 on a k = 4 chain: the rejection-sampling decision of the step
    equals the oracle's rule on the step's own logits."""
    tm, tw, _, _ = synthetic.c1_pair()
    V = tm["n_vocab"]
    g = synthetic.rng(0, 92)
    B, k, P = 2, 4, 40
    with _ctx(pages=16, slots=2) as ctx:
        ctx.load_model(tm, tw)
        for b in range(B):
            ctx.bind_slot(b, np.arange(8 * b, 8 * b + 8))
            velo_cuda.prefill(ctx, b, g.integers(0, V, P), n_vocab=V)
        tokens = g.integers(0, V, (B, k + 1)).astype(np.uint32)
        parents = np.tile(np.arange(-1, k, dtype=np.int32), (B, 1))
        drf = g.normal(0, 1.0, (B, k, V)).astype(np.float32)
        uni = g.random((B, k + 1)).astype(np.float32)
        # draft tokens sampled from q = softmax(drf), so some of them are accepted
        for b in range(B):
            for i in range(k):
                q = np.exp(drf[b, i].astype(np.float64) - drf[b, i].max())
                tokens[b, i + 1] = min(int(np.searchsorted(np.cumsum(q / q.sum()), g.random())), V - 1)
        r = ctx.verify_step(list(range(B)), [P] * B, tokens, parents, temperature=1.0,
                            draft_logits=drf, uniforms=uni, commit=False, want_logits=True,
                            n_vocab=V)
        acc, bonus = vo.accept(r["logits"], drf, tokens[:, 1:], uni, 1.0)
        assert list(r["accepted_len"]) == list(acc)
        assert list(r["bonus"]) == list(bonus)


def test_f32_session_matches_oracle():
    """The tiny pair's workload: 64-token prompt, k = 4 (window fixed by
    with_max_window(4, 4)), 128 new tokens, greedy."""
    tm, tw, dm, dw = synthetic.c1_pair()
    V = tm["n_vocab"]
    prompt = [int(t) for t in synthetic.rng(0, 91).integers(0, V, 64)]
    dec = SpeculativeDecoder(4, 4)
    ref = dec.generate(OracleDraft(vo.Model(dict(dm, n_ctx=512), synthetic.oracle_tensor_list(dm, dw))),
                       OracleTarget(vo.Model(dict(tm, n_ctx=512), synthetic.oracle_tensor_list(tm, tw))),
                       prompt, 128)
    with _ctx(pages=16, slots=1) as tctx, _ctx(pages=16, slots=1) as dctx:
        tctx.load_model(tm, tw)
        dctx.load_model(dm, dw)
        tctx.bind_slot(0, np.arange(16))
        dctx.bind_slot(0, np.arange(16))
        out = dec.generate(CudaDraft(dctx, 0, V), CudaTarget(tctx, 0, V), prompt, 128)
    assert out.stats.accepted_tokens > 0
    assert out.tokens == ref.tokens
    assert out.stats == ref.stats


class _OracleSamplingDraft:
    """The oracle's draft at T > 0: the same host sampler as CudaDraft."""

    def __init__(self, model, T, rng):
        self.m, self.T, self.rng, self.tokens, self.last_logits = model, T, rng, [], None

    def draft(self, context, n):
        common = 0
        for a, b in zip(self.tokens, context[:-1]):
            if a != b:
                break
            common += 1
        self.tokens = self.tokens[:common]
        for i in range(common, len(context) - 1):
            self.m.forward_one(int(context[i]), i)
            self.tokens.append(int(context[i]))
        out, last, lgs = [], int(context[-1]), []
        for _ in range(n):
            lg = self.m.forward_one(last, len(self.tokens))
            self.tokens.append(last)
            lgs.append(lg)
            last = sample_token(lg, self.T, self.rng.random())
            out.append(NextTokenPrediction(last))
        self.last_logits = np.stack(lgs)
        return out


class _OracleSamplingTarget:
    def __init__(self, model, T, draft, rng):
        self.m, self.T, self.draft, self.rng, self.cached = model, T, draft, rng, 0

    def verify(self, context, drafted):
        for i in range(self.cached, len(context) - 1):
            self.m.forward_one(int(context[i]), i)
        pos = len(context) - 1
        nodes = np.array([context[-1]] + list(drafted), np.uint32)
        lg = self.m.verify_tree(nodes, np.arange(-1, len(nodes) - 1, dtype=np.int32), pos)
        u = self.rng.random((1, len(nodes))).astype(np.float32)
        acc, bonus = vo.accept(lg[None], self.draft.last_logits[None, :len(drafted)],
                               np.array([drafted], np.uint32), u, self.T)
        acc, bonus = int(acc[0]), int(bonus[0])
        self.m.commit_path(list(range(acc + 1)), pos)
        self.cached = pos + acc + 1
        return [VerifyStep(t) for t in drafted[:acc]] + [VerifyStep(bonus)] * (len(drafted) - acc)


def test_f32_session_sampling_matches_oracle():
    """The same workload at T = 1.0: the draft samples from its logits, the
    verify step runs rejection sampling (seeded uniforms shared by both sides).
    Device and oracle logits differ by <= 1e-4, so the sampled tokens agree
    unless a uniform lands within that distance of a CDF step."""
    tm, tw, dm, dw = synthetic.c1_pair()
    V = tm["n_vocab"]
    prompt = [int(t) for t in synthetic.rng(0, 91).integers(0, V, 64)]
    dec = SpeculativeDecoder(4, 4)
    g = np.random.Generator(np.random.Philox(5))
    od = _OracleSamplingDraft(vo.Model(dict(dm, n_ctx=512), synthetic.oracle_tensor_list(dm, dw)), 1.0, g)
    ot = _OracleSamplingTarget(vo.Model(dict(tm, n_ctx=512), synthetic.oracle_tensor_list(tm, tw)),
                               1.0, od, g)
    ref = dec.generate(od, ot, prompt, 64)
    g = np.random.Generator(np.random.Philox(5))
    with _ctx(pages=16, slots=1) as tctx, _ctx(pages=16, slots=1) as dctx:
        tctx.load_model(tm, tw)
        dctx.load_model(dm, dw)
        tctx.bind_slot(0, np.arange(16))
        dctx.bind_slot(0, np.arange(16))
        d = CudaDraft(dctx, 0, V, 1.0, g)
        out = dec.generate(d, CudaTarget(tctx, 0, V, 1.0, d, g), prompt, 64)
    assert out.stats.accepted_tokens > 0 and out.stats.rejected_tokens > 0
    assert out.tokens == ref.tokens
    assert out.stats == ref.stats
