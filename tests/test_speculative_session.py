"""The session loop (velo-core_b200/speculative.py) against the reference's
own tests of src/speculative.rs (:605-825), re-expressed with the same
scripted draft / target models and the same expected tokens and stats."""
import pytest

from speculative import (DraftReturnedTooMany, EmptyDraftWindow, NextTokenPrediction,
                         SpeculativeDecoder, SpeculativeStats, TargetReturnedWrongLength,
                         VerifyStep)


class ScriptedDraft:
    def __init__(self, script):
        self.script = script

    def draft(self, context, max_tokens):
        return [NextTokenPrediction(t) for t in self.script[len(context):][:max_tokens]]


class ScriptedTarget:
    def __init__(self, script):
        self.script = script

    def verify(self, context, drafted):
        return [VerifyStep(t) for t in self.script[len(context):][:len(drafted)]]


def test_accepts_full_draft_windows():  # speculative.rs:605-631
    out = SpeculativeDecoder(3).generate(ScriptedDraft([1, 2, 3, 4, 5, 6]),
                                         ScriptedTarget([1, 2, 3, 4, 5, 6]), [1, 2], 4)
    assert out.tokens == [3, 4, 5, 6]
    assert out.stats == SpeculativeStats(draft_calls=2, target_calls=2, drafted_tokens=4,
                                         accepted_tokens=4, rejected_tokens=0)


def test_falls_back_to_target_token_on_first_rejection():  # :633-650
    out = SpeculativeDecoder(4).generate(ScriptedDraft([1, 2, 9, 4, 5]),
                                         ScriptedTarget([1, 2, 3, 4, 5]), [1, 2], 3)
    assert out.tokens == [3, 4, 5]
    assert out.stats.accepted_tokens == 2
    assert out.stats.rejected_tokens == 3


def test_stops_at_max_new_tokens():  # :652-669
    out = SpeculativeDecoder(8).generate(ScriptedDraft([1, 2, 3, 4, 5]),
                                         ScriptedTarget([1, 2, 3, 4, 5]), [1], 2)
    assert out.tokens == [2, 3]
    assert out.stats.drafted_tokens == 2


def test_rejects_zero_draft_window():  # :671-677
    with pytest.raises(EmptyDraftWindow):
        SpeculativeDecoder(0)
    with pytest.raises(EmptyDraftWindow):
        SpeculativeDecoder(4, max_window=3)


def test_error_display():  # :679-685
    assert "draft window must be greater than zero" in str(EmptyDraftWindow())
    assert "draft model returned 2 tokens" in str(DraftReturnedTooMany(1, 2))
    assert "target model returned 2 verification steps" in str(TargetReturnedWrongLength(1, 2))


def test_session_exposes_prompt_and_context():  # :694-701
    s = SpeculativeDecoder(2).begin([7, 8])
    assert s.prompt == [7, 8] and s.context == [7, 8]


def test_commit_logic():  # :717-729
    s = SpeculativeDecoder(4).begin([1])
    assert s.commit([NextTokenPrediction(2)], [VerifyStep(2)]) == [2]
    assert s.context == [1, 2]
    with pytest.raises(TargetReturnedWrongLength):
        s.commit([NextTokenPrediction(2)], [])


def test_record_stats():  # :731-739
    s = SpeculativeDecoder(4).begin([])
    s.record_draft_call()
    s.record_target_call()
    assert s.stats.draft_calls == 1 and s.stats.target_calls == 1


def test_draft_error_paths():  # :741-779
    s = SpeculativeDecoder(4).begin([1])

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

    with pytest.raises(DraftReturnedTooMany):
        s.draft(BadDraft(), OkTarget(), 4)
    assert s.draft(EmptyDraft(), OkTarget(), 4) == []
    with pytest.raises(TargetReturnedWrongLength):
        s.draft(ScriptedDraft([1, 2, 3]), BadTarget(), 4)


def test_dynamic_draft_window():  # :781-797: 2 -> 3 -> 2
    s = SpeculativeDecoder(2).begin([1])
    assert s.current_window() == 2
    s.commit([NextTokenPrediction(2), NextTokenPrediction(3)], [VerifyStep(2), VerifyStep(3)])
    assert s.current_window() == 3
    s.commit([NextTokenPrediction(4), NextTokenPrediction(9)], [VerifyStep(4), VerifyStep(5)])
    assert s.current_window() == 2
