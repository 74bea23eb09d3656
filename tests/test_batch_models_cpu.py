"""The batched device models' host logic on the CPU: CudaBatchDraft /
CudaBatchTarget and the per-request CudaDraft / CudaTarget run over a stand-in
context whose verify_step is the CPU oracle (one oracle model per slot,
greedy chains), so the batching glue, the slot bookkeeping and the native
session callbacks are checked without a GPU.  The GPU tests run the same
classes over velo_cuda.Context."""
import numpy as np

import synthetic
import vo
from speculative import (CudaBatchDraft, CudaBatchTarget, CudaDraft, CudaTarget, SpeculativeDecoder,
                         SpeculativeEngine, native_generate)


class OracleContext:
    """velo_cuda.Context.verify_step for greedy chains, on the oracle: each
    slot is a vo.Model whose cache plays the slot's pages."""

    def __init__(self, meta, tensors, n_slots):
        tl = synthetic.oracle_tensor_list(meta, tensors)
        self.models = [vo.Model(dict(meta, n_ctx=512), tl) for _ in range(n_slots)]
        self.calls = []

    def verify_step(self, slots, ctx_len, tokens, parents, commit=True, n_vocab=None, **_):
        tokens = np.asarray(tokens)
        B, N = tokens.shape
        self.calls.append((B, N, commit))
        acc, bonus = np.zeros(B, np.int32), np.zeros(B, np.uint32)
        for b in range(B):
            m = self.models[slots[b]]
            lg = m.verify_tree(tokens[b], np.asarray(parents)[b], int(ctx_len[b]))
            exp = [vo.greedy(lg[i])[0] for i in range(N)]
            if commit == "all":
                a = N - 1
            else:
                a = 0
                while a < N - 1 and int(tokens[b][a + 1]) == exp[a]:
                    a += 1
            if commit:
                m.commit_path(list(range(a + 1)), int(ctx_len[b]))
            acc[b], bonus[b] = a, exp[a]
        return {"accepted_len": acc, "bonus": bonus}


V = 256


def _models():
    meta, target_w = synthetic.llama_q4_model(V, 256, 2, 2, 1, 512, seed=51, sigma=0.05)
    _, draft_w = synthetic.llama_q4_model(V, 256, 1, 2, 1, 512, seed=51, sigma=0.05)
    return meta, target_w, dict(meta, n_layer=1), draft_w


class PerRequest:
    def __init__(self, models):
        self.models = models

    def draft_batch(self, reqs):
        return [self.models[rid].draft(c, m) for rid, c, m in reqs]

    def verify_batch(self, reqs):
        return [self.models[rid].verify(c, d) for rid, c, d in reqs]


def test_batched_models_match_per_request_models():
    meta, target_w, dmeta, draft_w = _models()
    g = synthetic.rng(52, 91)
    requests = [(list(g.integers(0, V, n)), m) for n, m in ((12, 14), (30, 6), (5, 11))]
    eng = SpeculativeEngine(3, max_slots=3)
    t1, d1 = OracleContext(meta, target_w, 3), OracleContext(dmeta, draft_w, 3)
    ref = eng.generate_batch(PerRequest([CudaDraft(d1, s, V) for s in range(3)]),
                             PerRequest([CudaTarget(t1, s, V) for s in range(3)]), requests)
    t2, d2 = OracleContext(meta, target_w, 3), OracleContext(dmeta, draft_w, 3)
    out = eng.generate_batch(CudaBatchDraft(d2, [0, 1, 2], V), CudaBatchTarget(t2, [0, 1, 2], V), requests)
    assert sum(o.stats.rejected_tokens for o in out) > 0
    for o, r, (_, m) in zip(out, ref, requests):
        assert len(o.tokens) == m
        assert o.tokens == r.tokens and o.stats == r.stats
    # the batched target ran fewer, wider verify steps (prefill chains aside)
    wide = [c for c in t2.calls if c[2] is True]
    assert max(b for b, _, _ in wide) == 3
    assert len(wide) < len([c for c in t1.calls if c[2] is True])
    # and each batched draft step covered every request still drafting
    assert max(b for b, n, c in d2.calls if c == "all" and n == 1) == 3


def test_native_session_over_device_model_classes():
    meta, target_w, dmeta, draft_w = _models()
    prompt = [int(t) for t in synthetic.rng(62, 91).integers(0, V, 16)]
    runs = []
    for native in (False, True):
        d = CudaDraft(OracleContext(dmeta, draft_w, 1), 0, V)
        t = CudaTarget(OracleContext(meta, target_w, 1), 0, V)
        runs.append(native_generate(4, d, t, prompt, 20) if native
                    else SpeculativeDecoder(4).generate(d, t, prompt, 20))
    assert len(runs[1].tokens) == 20
    assert runs[1].tokens == runs[0].tokens and runs[1].stats == runs[0].stats


def test_native_engine_over_batched_model_classes():
    from speculative import native_generate_batch
    meta, target_w, dmeta, draft_w = _models()
    g = synthetic.rng(53, 91)
    requests = [(list(g.integers(0, V, n)), m) for n, m in ((9, 10), (20, 7))]
    ref = SpeculativeEngine(3, max_slots=2).generate_batch(
        CudaBatchDraft(OracleContext(dmeta, draft_w, 2), [0, 1], V),
        CudaBatchTarget(OracleContext(meta, target_w, 2), [0, 1], V), requests)
    out = native_generate_batch(3, CudaBatchDraft(OracleContext(dmeta, draft_w, 2), [0, 1], V),
                                CudaBatchTarget(OracleContext(meta, target_w, 2), [0, 1], V), requests,
                                max_slots=2)
    assert [(o.tokens, o.stats) for o in out] == [(r.tokens, r.stats) for r in ref]
