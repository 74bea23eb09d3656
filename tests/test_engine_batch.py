"""The batched engine loop (SpeculativeEngine.generate_batch, no GPU): the
reference's engine tests re-expressed (src/engine.rs:825-947) with scripted
models, and the batching contract: one verify_batch call per round covering
every unfinished request, windows of min(remaining, draft_window)."""
import numpy as np
import pytest

from speculative import (NextTokenPrediction, SlotsExhausted, SpeculativeEngine, VerifyStep,
                         native_generate_batch)


class ScriptedDraft:
    """Drafts script[len(context):][:max_tokens] (engine.rs:552-586)."""

    def __init__(self, script):
        self.script, self.bound_slots = script, []

    def bind_slot(self, slot):
        self.bound_slots.append(slot)

    def draft(self, context, max_tokens):
        return [NextTokenPrediction(t) for t in self.script[len(context):][:max_tokens]]


class ScriptedTarget:
    """Expects script[len(context) + i] after drafted[:i] (engine.rs:588-630)."""

    def __init__(self, script):
        self.script, self.bound_slots = script, []

    def bind_slot(self, slot):
        self.bound_slots.append(slot)

    def verify(self, context, drafted):
        return [VerifyStep(self.script[len(context) + i]) for i in range(len(drafted))]


def test_multi_request_batching():  # engine.rs:825-852
    script = [0, 2, 3, 0, 0, 0, 0, 0, 0, 0, 0, 11, 12, 13]
    draft, target = ScriptedDraft(script), ScriptedTarget(script)
    out = SpeculativeEngine(2, max_slots=4).generate_batch(draft, target, [([0], 2), ([0] * 11, 3)])
    assert [o.tokens for o in out] == [[2, 3], [11, 12, 13]]
    assert len(draft.bound_slots) == 2 and draft.bound_slots[0] != draft.bound_slots[1]


def test_batch_with_mixed_finishing():  # engine.rs:853-889
    script = [0, 2, 0, 0, 0, 0, 0, 0, 0, 0, 0, 11, 12]
    out = SpeculativeEngine(1, max_slots=4).generate_batch(ScriptedDraft(script), ScriptedTarget(script),
                                                          [([1], 1), ([10] * 11, 2)])
    assert [o.tokens for o in out] == [[2], [11, 12]]


def test_batch_slot_exhaustion():  # engine.rs:890-917
    with pytest.raises(SlotsExhausted):
        SpeculativeEngine(1, max_slots=1).generate_batch(ScriptedDraft([1, 2]), ScriptedTarget([1, 2]),
                                                          [([0], 1), ([0], 1)])


class CountingBatchTarget(ScriptedTarget):
    def __init__(self, script):
        super().__init__(script)
        self.calls = []

    def verify_batch(self, reqs):
        self.calls.append([(rid, len(d)) for rid, _, d in reqs])
        return [self.verify(c, d) for _, c, d in reqs]


def test_one_verify_call_per_round_for_all_unfinished_requests():
    script = list(range(100))
    draft, target = ScriptedDraft(script), CountingBatchTarget(script)
    out = SpeculativeEngine(4, max_slots=3).generate_batch(draft, target, [([0], 10), ([0, 1], 3), ([0], 6)])
    assert [o.tokens for o in out] == [list(range(1, 11)), [2, 3, 4], list(range(1, 7))]
    # round 1: all three with min(remaining, 4); round 2: requests 0 and 2; round 3: request 0
    assert target.calls == [[(0, 4), (1, 3), (2, 4)], [(0, 4), (2, 2)], [(0, 2)]]
    assert [o.stats.target_calls for o in out] == [3, 1, 2]
    assert [o.stats.accepted_tokens for o in out] == [10, 3, 6]


def test_rejections_emit_the_target_token_per_request():
    draft = ScriptedDraft([0, 5, 6, 7, 8, 9, 10, 11, 12])
    target = ScriptedTarget([0, 5, 6, 99, 8, 9, 10, 11, 12])
    out = SpeculativeEngine(4, max_slots=2).generate_batch(draft, target, [([0], 4), ([0, 5, 6, 99], 2)])
    # request 0: drafts 5 6 7 8, the target wants 99 at the third -> 5 6 99, then one more round
    assert out[0].tokens[:3] == [5, 6, 99]
    assert out[0].stats.rejected_tokens == 2
    assert out[1].tokens == [8, 9]


def test_a_draft_model_returning_nothing_ends_the_loop():
    out = SpeculativeEngine(2).generate_batch(ScriptedDraft([0]), ScriptedTarget([0]), [([0], 3)])
    assert out[0].tokens == []


# ---- the native engine loop (velo_spec_generate_batch) -----------------------


def test_native_reference_cases():  # engine.rs:825-917
    script = [0, 2, 3, 0, 0, 0, 0, 0, 0, 0, 0, 11, 12, 13]
    out = native_generate_batch(2, ScriptedDraft(script), ScriptedTarget(script), [([0], 2), ([0] * 11, 3)],
                                max_slots=4)
    assert [o.tokens for o in out] == [[2, 3], [11, 12, 13]]
    script = [0, 2, 0, 0, 0, 0, 0, 0, 0, 0, 0, 11, 12]
    out = native_generate_batch(1, ScriptedDraft(script), ScriptedTarget(script), [([1], 1), ([10] * 11, 2)],
                                max_slots=4)
    assert [o.tokens for o in out] == [[2], [11, 12]]
    with pytest.raises(SlotsExhausted):
        native_generate_batch(1, ScriptedDraft([1, 2]), ScriptedTarget([1, 2]), [([0], 1), ([0], 1)], max_slots=1)


def test_native_batch_calls_and_stats_match_python_engine():
    script = list(range(100))
    py_t, nat_t = CountingBatchTarget(script), CountingBatchTarget(script)
    reqs = [([0], 10), ([0, 1], 3), ([0], 6)]
    ref = SpeculativeEngine(4, max_slots=3).generate_batch(ScriptedDraft(script), py_t, reqs)
    out = native_generate_batch(4, ScriptedDraft(script), nat_t, reqs, max_slots=3)
    assert nat_t.calls == py_t.calls
    assert [(o.tokens, o.stats) for o in out] == [(r.tokens, r.stats) for r in ref]


class NoisyDraft:
    """Drafts the target's script with seeded corruptions (per request)."""

    def __init__(self, script, p, seed):
        self.script, self.p, self.seed = script, p, seed

    def draft(self, context, max_tokens):
        g = np.random.default_rng(self.seed * 100003 + len(context))
        return [NextTokenPrediction(t if g.random() > self.p else t + 1)
                for t in self.script[len(context):][:max_tokens]]


@pytest.mark.parametrize("seed", range(5))
def test_native_batch_matches_python_engine_on_random_models(seed):
    g = np.random.default_rng(seed)
    script = [int(x) for x in g.integers(0, 40, 300)]
    reqs = [(script[:int(g.integers(1, 30))], int(g.integers(1, 60))) for _ in range(int(g.integers(1, 6)))]
    window, p = int(g.integers(1, 6)), float(g.choice([0.0, 0.2, 0.6]))
    ref = SpeculativeEngine(window).generate_batch(NoisyDraft(script, p, seed), ScriptedTarget(script), reqs)
    out = native_generate_batch(window, NoisyDraft(script, p, seed), ScriptedTarget(script), reqs)
    assert [(o.tokens, o.stats) for o in out] == [(r.tokens, r.stats) for r in ref]
