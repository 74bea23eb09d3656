"""End-to-end speculative decoding on the device: a q4_0 draft model and a
q4_0 target model in two contexts, the session loop of speculative.py, every
model call through the C ABI (prefill, one-token draft steps, verify steps
with KV commit and rollback by length).  The same session over the CPU
oracle's models must produce the same tokens and the same statistics."""
import numpy as np
import pytest

import synthetic
import velo_cuda
import vo
from speculative import (CudaBatchDraft, CudaBatchTarget, CudaDraft, CudaTarget, NextTokenPrediction,
                         SpeculativeDecoder, SpeculativeEngine, VerifyStep, native_generate)

pytestmark = pytest.mark.gpu


class OracleTarget:
    def __init__(self, model):
        self.m = model
        self.cached = 0

    def _prefill(self, context):
        for i in range(self.cached, len(context) - 1):
            self.m.forward_one(int(context[i]), i)
        self.cached = max(self.cached, len(context) - 1)

    def verify(self, context, drafted):
        self._prefill(context)
        pos = len(context) - 1
        nodes = np.array([context[-1]] + list(drafted), np.uint32)
        parents = np.arange(-1, len(nodes) - 1, dtype=np.int32)
        lg = self.m.verify_tree(nodes, parents, pos)
        exp = [vo.greedy(lg[i])[0] for i in range(len(drafted))]
        acc = 0
        while acc < len(drafted) and drafted[acc] == exp[acc]:
            acc += 1
        self.m.commit_path(list(range(acc + 1)), pos)
        self.cached = pos + acc + 1
        return [VerifyStep(e) for e in exp]


class OracleDraft:
    def __init__(self, model):
        self.m = model
        self.tokens = []

    def draft(self, context, max_tokens):
        common = 0
        for a, b in zip(self.tokens, context[:-1]):
            if a != b:
                break
            common += 1
        self.tokens = self.tokens[:common]
        for i in range(common, len(context) - 1):
            self.m.forward_one(int(context[i]), i)
            self.tokens.append(int(context[i]))
        out, last = [], int(context[-1])
        for _ in range(max_tokens):
            lg = self.m.forward_one(last, len(self.tokens))
            self.tokens.append(last)
            last = vo.greedy(lg)[0]
            out.append(NextTokenPrediction(last))
        return out


def test_speculative_generate_device_matches_oracle():
    V = 256
    # draft = target plus a perturbation, so drafts are often but not always accepted
    meta, target_w = synthetic.llama_q4_model(V, 256, 2, 2, 1, 512, seed=41, sigma=0.05)
    _, draft_w = synthetic.llama_q4_model(V, 256, 1, 2, 1, 512, seed=41, sigma=0.05)
    dmeta = dict(meta, n_layer=1)
    prompt = list(synthetic.rng(42, 91).integers(0, V, 20))
    dec = SpeculativeDecoder(4)
    ref = dec.generate(OracleDraft(vo.Model(dict(dmeta, n_ctx=512),
                                            synthetic.oracle_tensor_list(dmeta, draft_w))),
                       OracleTarget(vo.Model(dict(meta, n_ctx=512),
                                             synthetic.oracle_tensor_list(meta, target_w))),
                       prompt, 40)
    tctx = velo_cuda.Context(device=0, total_pages=8, max_slots=1, max_pages_per_slot=8)
    dctx = velo_cuda.Context(device=0, total_pages=8, max_slots=1, max_pages_per_slot=8)
    try:
        tctx.load_model(meta, target_w)
        dctx.load_model(dmeta, draft_w)
        tctx.bind_slot(0, np.arange(8))
        dctx.bind_slot(0, np.arange(8))
        out = dec.generate(CudaDraft(dctx, 0, V), CudaTarget(tctx, 0, V), prompt, 40)
    finally:
        tctx.close()
        dctx.close()
    assert out.stats.accepted_tokens > 0 and out.stats.rejected_tokens > 0
    assert out.tokens == ref.tokens
    assert out.stats == ref.stats


class PerRequest:
    """One single-sequence model per request id behind the engine's batch interface."""

    def __init__(self, models):
        self.models = models

    def draft_batch(self, reqs):
        return [self.models[rid].draft(c, m) for rid, c, m in reqs]

    def verify_batch(self, reqs):
        return [self.models[rid].verify(c, d) for rid, c, d in reqs]


def test_batched_engine_matches_per_request_device_models():
    """generate_batch over CudaBatchDraft / CudaBatchTarget (one draft step per
    position and one verify step per round for all requests) gives every
    request the tokens and statistics of the same engine over per-request
    CudaDraft / CudaTarget models (one sequence per call): batching changes
    no result.  The per-request session path is checked against the oracle in
    test_speculative_generate_device_matches_oracle."""
    V = 256
    meta, target_w = synthetic.llama_q4_model(V, 256, 2, 2, 1, 512, seed=51, sigma=0.05)
    _, draft_w = synthetic.llama_q4_model(V, 256, 1, 2, 1, 512, seed=51, sigma=0.05)
    dmeta = dict(meta, n_layer=1)
    g = synthetic.rng(52, 91)
    requests = [(list(g.integers(0, V, n)), m) for n, m in ((12, 24), (30, 9), (5, 17))]
    eng = SpeculativeEngine(3, max_slots=3)

    def run(batched):
        tctx = velo_cuda.Context(device=0, total_pages=24, max_slots=3, max_pages_per_slot=8)
        dctx = velo_cuda.Context(device=0, total_pages=24, max_slots=3, max_pages_per_slot=8)
        try:
            tctx.load_model(meta, target_w)
            dctx.load_model(dmeta, draft_w)
            for s in range(3):
                tctx.slot_allocate(s, 8 * 16)
                dctx.slot_allocate(s, 8 * 16)
            if batched:
                draft, target = CudaBatchDraft(dctx, [0, 1, 2], V), CudaBatchTarget(tctx, [0, 1, 2], V)
            else:
                draft = PerRequest([CudaDraft(dctx, s, V) for s in range(3)])
                target = PerRequest([CudaTarget(tctx, s, V) for s in range(3)])
            return eng.generate_batch(draft, target, requests)
        finally:
            tctx.close()
            dctx.close()

    ref, out = run(False), run(True)
    assert sum(o.stats.rejected_tokens for o in out) > 0
    assert sum(o.stats.accepted_tokens for o in out) > 0
    for o, r, (_, m) in zip(out, ref, requests):
        assert len(o.tokens) == m
        assert o.tokens == r.tokens
        assert o.stats == r.stats


def test_native_session_drives_device_models():
    """The native session loop (velo_spec_generate) over the device models
    gives the tokens and statistics of the Python session loop over them."""
    V = 256
    meta, target_w = synthetic.llama_q4_model(V, 256, 2, 2, 1, 512, seed=61, sigma=0.05)
    _, draft_w = synthetic.llama_q4_model(V, 256, 1, 2, 1, 512, seed=61, sigma=0.05)
    dmeta = dict(meta, n_layer=1)
    prompt = [int(t) for t in synthetic.rng(62, 91).integers(0, V, 16)]

    def run(native):
        tctx = velo_cuda.Context(device=0, total_pages=8, max_slots=1, max_pages_per_slot=8)
        dctx = velo_cuda.Context(device=0, total_pages=8, max_slots=1, max_pages_per_slot=8)
        try:
            tctx.load_model(meta, target_w)
            dctx.load_model(dmeta, draft_w)
            tctx.slot_allocate(0, 128)
            dctx.slot_allocate(0, 128)
            d, t = CudaDraft(dctx, 0, V), CudaTarget(tctx, 0, V)
            if native:
                return native_generate(4, d, t, prompt, 30)
            return SpeculativeDecoder(4).generate(d, t, prompt, 30)
        finally:
            tctx.close()
            dctx.close()

    ref, out = run(False), run(True)
    assert len(out.tokens) == 30
    assert out.tokens == ref.tokens
    assert out.stats == ref.stats
