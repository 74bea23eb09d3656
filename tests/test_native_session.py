"""The native session loop (include/velo_session.h, no GPU): the reference's
session tests (src/speculative.rs:605-797) run against it with the same
scripted models, and seeded random model pairs give the same tokens, stats
and windows as the Python restatement (velo-core_b200/speculative.py)."""
import numpy as np
import pytest

from speculative import (DraftReturnedTooMany, EmptyDraftWindow, NativeSession, NextTokenPrediction,
                         SpeculativeDecoder, SpeculativeStats, TargetReturnedWrongLength, VerifyStep,
                         native_generate)
from test_speculative_session import ScriptedDraft, ScriptedTarget


def test_accepts_full_draft_windows():  # speculative.rs:605-631
    out = native_generate(3, ScriptedDraft([1, 2, 3, 4, 5, 6]), ScriptedTarget([1, 2, 3, 4, 5, 6]), [1, 2], 4)
    assert out.tokens == [3, 4, 5, 6]
    assert out.stats == SpeculativeStats(draft_calls=2, target_calls=2, drafted_tokens=4, accepted_tokens=4,
                                         rejected_tokens=0)


def test_falls_back_to_target_token_on_first_rejection():  # :633-650
    out = native_generate(4, ScriptedDraft([1, 2, 9, 4, 5]), ScriptedTarget([1, 2, 3, 4, 5]), [1, 2], 3)
    assert out.tokens == [3, 4, 5]
    assert out.stats.accepted_tokens == 2 and out.stats.rejected_tokens == 3


def test_stops_at_max_new_tokens_and_rejects_zero_window():  # :652-677
    out = native_generate(8, ScriptedDraft(list(range(100))), ScriptedTarget(list(range(100))), [0], 5)
    assert out.tokens == [1, 2, 3, 4, 5]
    with pytest.raises(EmptyDraftWindow):
        native_generate(0, ScriptedDraft([1]), ScriptedTarget([1]), [0], 1)
    with pytest.raises(EmptyDraftWindow):
        NativeSession(4, [1], max_window=3)


def test_session_commit_stats_and_dynamic_window():  # :717-739, 781-797
    s = NativeSession(2, [1])
    assert s.context == [1] and s.draft_window == 2
    assert s.commit([NextTokenPrediction(2), NextTokenPrediction(3)], [VerifyStep(2), VerifyStep(3)]) == [2, 3]
    assert s.draft_window == 3
    assert s.commit([NextTokenPrediction(4), NextTokenPrediction(9)], [VerifyStep(4), VerifyStep(5)]) == [4]
    assert s.draft_window == 2
    assert s.has_pending_rejection() and s.take_rejected_token() == 5 and s.take_rejected_token() is None
    assert s.context == [1, 2, 3, 4, 5]
    s.record_draft_call()
    s.record_target_call()
    assert s.stats == SpeculativeStats(draft_calls=1, target_calls=1, drafted_tokens=4, accepted_tokens=3,
                                       rejected_tokens=1)
    with pytest.raises(TargetReturnedWrongLength):
        s.commit([NextTokenPrediction(1)], [])


def test_draft_error_paths():  # :741-779
    s = NativeSession(4, [1])

    class BadDraft:
        def draft(self, c, m):
            return [NextTokenPrediction(1)] * 10

    class EmptyDraft:
        def draft(self, c, m):
            return []

    class OkTarget:
        def verify(self, c, d):
            return [VerifyStep(1)] * len(d)

    class BadTarget:
        def verify(self, c, d):
            return []

    class Failing:
        def draft(self, c, m):
            raise RuntimeError("draft backend down")

    with pytest.raises(DraftReturnedTooMany) as e:
        s.draft(BadDraft(), OkTarget(), 4)
    assert (e.value.requested, e.value.returned) == (4, 10)
    assert s.draft(EmptyDraft(), OkTarget(), 4) == []
    with pytest.raises(TargetReturnedWrongLength):
        s.draft(ScriptedDraft([1, 2, 3]), BadTarget(), 4)
    with pytest.raises(RuntimeError, match="backend down"):
        s.draft(Failing(), OkTarget(), 4)


class RandomDraft:
    """Drafts the target's script with seeded corruptions."""

    def __init__(self, script, p, seed):
        self.script, self.p, self.g = script, p, np.random.default_rng(seed)

    def draft(self, context, max_tokens):
        out = []
        for t in self.script[len(context):][:max_tokens]:
            out.append(NextTokenPrediction(int(t) if self.g.random() > self.p else int(t) + 1))
        return out


@pytest.mark.parametrize("seed", range(6))
def test_matches_python_session(seed):
    g = np.random.default_rng(seed)
    script = [int(x) for x in g.integers(0, 50, 400)]
    prompt, window, n = script[:int(g.integers(1, 20))], int(g.integers(1, 6)), int(g.integers(1, 120))
    p = float(g.choice([0.0, 0.1, 0.4, 0.9]))
    ref = SpeculativeDecoder(window).generate(RandomDraft(script, p, seed), ScriptedTarget(script), prompt, n)
    out = native_generate(window, RandomDraft(script, p, seed), ScriptedTarget(script), prompt, n)
    assert out.tokens == ref.tokens
    assert out.stats == ref.stats
