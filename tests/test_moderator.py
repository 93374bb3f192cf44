"""CPU tests of the moderator host layer (ShieldstralModerator.cs): result
fields and verdict rule, the cached system prefix and PrefilledTokens, the
SHKV path, argument errors and cancellation, driven against a stand-in for
ShieldContext that returns what the binding returns (the GPU calls behind it,
score_batch / last_logits / set_prefix / prefix state, are GPU-tested)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from llm_shield_b200 import binding, prefix_file
from llm_shield_b200.moderator import ModerationResult, ShieldModerator

VOCAB = 64


class FakeContext:
    def __init__(self):
        self.calls = []
        self.state = None

    @staticmethod
    def _logits(ids):
        rng = np.random.default_rng(int(np.asarray(ids, np.int64).sum()) + ids.size)
        return (rng.standard_normal(VOCAB) * 4).astype(np.float32)

    def score_batch(self, requests, verdict_ids, n_yes, cancel=None):
        if cancel is not None and cancel[0]:
            raise binding.ShieldCancelled(binding.ERR_CANCELLED, "cancelled")
        self.calls.append(("score", len(requests)))
        v = np.asarray(verdict_ids)
        logits = np.stack([self._logits(r)[v] for r in requests])
        out = [oracle.score(row, n_yes, v.size - n_yes) for row in logits]
        score, yes, no = (np.array(c, np.float32) for c in zip(*out))
        return yes, no, score, logits

    def last_logits(self, requests, cancel=None):
        return np.stack([self._logits(r) for r in requests])

    def set_prefix(self, ids):
        ids = list(np.asarray(ids).reshape(-1))
        self.calls.append(("prefix", ids))
        self.state = np.arange(len(ids), dtype=np.float32) if ids else None

    def get_prefix_state(self):
        return self.state.copy()

    def set_prefix_state(self, ids, state):
        self.calls.append(("restore", list(ids)))
        self.state = np.asarray(state).copy()


YES, NO = [3, 9], [5]


def test_results_carry_the_reference_fields():
    ctx = FakeContext()
    m = ShieldModerator(ctx, YES, NO)
    assert ctx.calls == [("prefix", [])] and m.cached_prefix_tokens == 0
    prompts = [np.arange(1, n + 1, dtype=np.int32) for n in (5, 12, 30)]
    got = m.moderate_batch(prompts)
    assert ctx.calls[-1] == ("score", 3)  # one batched call
    for p, r in zip(prompts, got):
        logits = FakeContext._logits(p)[YES + NO]
        s, y, n = oracle.score(logits, len(YES), len(NO))
        assert (r.score, r.yes_logit, r.no_logit) == (np.float32(s), np.float32(y), np.float32(n))
        assert r.yes_logit == logits[:2].max() and r.no_logit == logits[2]
        assert r.prompt_tokens == p.size and r.prefilled_tokens == 0
        assert r.is_unsafe == (r.score > 0.5)
        assert r == m.moderate(p)
    assert m.moderate_batch([]) == []


def test_verdict_threshold_and_text():
    at = ModerationResult(0.5, 1.0, 1.0, 10, 0)
    assert not at.is_unsafe and at.is_unsafe_at(0.25) and not at.is_unsafe_at(0.75)
    above = ModerationResult(float(np.nextafter(np.float32(0.5), np.float32(1))), 2.0, 1.5, 10, 0)
    assert above.is_unsafe
    assert str(ModerationResult(0.75, 1.25, 0.125, 7, 3)) == "UNSAFE score=0.750000 (yes=1.2500 no=0.1250)"
    assert str(at) == "safe score=0.500000 (yes=1.0000 no=1.0000)"


def test_prefix_and_prefilled_tokens():
    ctx = FakeContext()
    prefix = np.array([1, 7, 7, 2], np.int32)
    m = ShieldModerator(ctx, YES, NO, system_prefix=prefix)
    assert ctx.calls == [("prefix", [1, 7, 7, 2])] and m.cached_prefix_tokens == 4
    longer = np.array([1, 7, 7, 2, 40, 41], np.int32)
    assert m.moderate(longer).prefilled_tokens == 4
    assert m.moderate(prefix).prefilled_tokens == 0          # nothing after it: forwarded whole
    assert m.moderate(prefix[:3]).prefilled_tokens == 0      # shorter
    assert m.moderate(np.array([1, 7, 8, 2, 40], np.int32)).prefilled_tokens == 0
    got = m.moderate_batch([longer, prefix])
    assert [r.prefilled_tokens for r in got] == [4, 0]


def test_prefix_file_is_written_then_restored(tmp_path):
    weights = tmp_path / "model.gguf"
    weights.write_bytes(b"w")
    ident = prefix_file.ModelIdentity(str(weights), "mistral3", 2, 8, 128)
    path = tmp_path / "prefix.shkv"
    prefix = [1, 2, 3]
    ctx = FakeContext()
    ShieldModerator(ctx, YES, NO, system_prefix=prefix, prefix_cache_path=path, model=ident)
    assert ctx.calls == [("prefix", prefix)] and path.exists()
    ctx2 = FakeContext()
    m = ShieldModerator(ctx2, YES, NO, system_prefix=prefix, prefix_cache_path=path, model=ident)
    assert ctx2.calls == [("restore", prefix)] and m.cached_prefix_tokens == 3


def test_argument_errors():
    with pytest.raises(ValueError):
        ShieldModerator(FakeContext(), [], NO)
    with pytest.raises(ValueError):
        ShieldModerator(FakeContext(), YES, [])
    with pytest.raises(ValueError):
        ShieldModerator(FakeContext(), YES, NO, system_prefix=[1], prefix_cache_path="p.shkv")


def test_cancellation_leaves_the_moderator_usable():
    m = ShieldModerator(FakeContext(), YES, NO)
    p = np.arange(1, 9, dtype=np.int32)
    with pytest.raises(binding.ShieldCancelled):
        m.moderate(p, cancel=np.ones(1, np.int32))
    assert m.moderate(p) == m.moderate(p, cancel=np.zeros(1, np.int32))


def test_full_head_and_top_token():
    m = ShieldModerator(FakeContext(), YES, NO)
    p = np.arange(1, 6, dtype=np.int32)
    logits = m.verdict_logits(p)
    assert logits.shape == (VOCAB,)
    assert m.top_verdict_token(p) == int(np.argmax(logits))
