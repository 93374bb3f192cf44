"""ShieldstralModerator over token ids, on the GPUs
(src/LlmShield.Shieldstral/ShieldstralModerator.cs:22-386).

The reference tokenizes a rendered chat prompt and scores it; the tokenizer,
chat template and verdict-token resolution stay with the caller (they are
host string work), so this class starts from the prompt's token ids and the
resolved yes/no vocabulary ids. What it keeps from the reference:

- ModerationResult (:22-33): Score, YesLogit, NoLogit, PromptTokens,
  PrefilledTokens, and the verdict IsUnsafe = Score > 0.5;
- the system-prompt prefix cached at open (:152-160), optionally through
  the SHKV file (SystemPromptCache.LoadOrCaptureAsync), and reported per
  request as PrefilledTokens (:277-284);
- ModerateAsync (:246-263) as moderate / moderate_batch (one batched call
  through shield_score_batch), VerdictLogitsAsync (:269-277) as
  verdict_logits, TopVerdictTokenAsync (:370-378) as top_verdict_token
  (the token id; decoding it stays with the tokenizer);
- errors: no yes or no ids raise ValueError (the reference's
  InvalidDataException, :100-104); cancellation raises the binding's
  ShieldCancelled (OperationCanceledException) and leaves the moderator
  usable.

One difference in an edge case: a prompt that equals the cached prefix
exactly is forwarded whole here (PrefilledTokens 0), where the reference
would restore the prefix and forward no tokens.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import prefix_file


@dataclass(frozen=True)
class ModerationResult:
    """One request's answer (ShieldstralModerator.cs:22-33)."""
    score: float
    yes_logit: float
    no_logit: float
    prompt_tokens: int
    prefilled_tokens: int

    @property
    def is_unsafe(self) -> bool:
        """The verdict at the model card's 0.5 threshold."""
        return self.is_unsafe_at(0.5)

    def is_unsafe_at(self, threshold: float) -> bool:
        return bool(np.float32(self.score) > np.float32(threshold))

    def __str__(self) -> str:
        word = "UNSAFE" if self.is_unsafe else "safe"
        return f"{word} score={self.score:.6f} (yes={self.yes_logit:.4f} no={self.no_logit:.4f})"


class ShieldModerator:
    """Scores prompts (token ids) with a ShieldContext whose model is uploaded.

    system_prefix: the BOS + system-message ids every prompt starts with
    (ShieldstralModerator.BuildSystemPrefixTokens); None turns the cache off.
    prefix_cache_path / model: persist the prefix state in an SHKV file tied
    to `model` (a prefix_file.ModelIdentity), as OpenAsync's prefixCachePath.
    Not thread-safe, like the reference (one context, one cached prefix).
    """

    def __init__(self, ctx, yes_ids, no_ids, system_prefix=None, prefix_cache_path=None,
                 model: prefix_file.ModelIdentity | None = None):
        yes = np.asarray(yes_ids, np.int32).reshape(-1)
        no = np.asarray(no_ids, np.int32).reshape(-1)
        if yes.size == 0 or no.size == 0:
            raise ValueError("The model's vocabulary has no 'yes'/'no' tokens; "
                             "this does not look like a Shieldstral checkpoint.")
        if prefix_cache_path is not None and model is None:
            raise ValueError("prefix_cache_path needs the model identity the snapshot is tied to")
        self.ctx = ctx
        self.yes_ids, self.no_ids = yes, no
        self.verdict_ids = np.concatenate([yes, no])
        self._prefix = np.zeros(0, np.int32)
        if system_prefix is not None:
            prefix = np.ascontiguousarray(system_prefix, np.int32)
            if prefix_cache_path is None:
                ctx.set_prefix(prefix)
            else:
                prefix_file.load_or_capture(ctx, model, prefix, prefix_cache_path)
            self._prefix = prefix.copy()
        else:
            ctx.set_prefix([])

    @property
    def cached_prefix_tokens(self) -> int:
        """CachedPrefixTokens: tokens of the cached system prefix, 0 when off."""
        return int(self._prefix.size)

    def prefilled_tokens(self, ids) -> int:
        """How many leading tokens of a prompt come from the cached prefix."""
        ids = np.asarray(ids)
        p = self._prefix.size
        if p and ids.size > p and np.array_equal(ids[:p], self._prefix):
            return int(p)
        return 0

    def moderate(self, ids, cancel: np.ndarray | None = None) -> ModerationResult:
        """ModerateAsync for one prompt's token ids."""
        return self.moderate_batch([ids], cancel)[0]

    def moderate_batch(self, prompts, cancel: np.ndarray | None = None) -> list[ModerationResult]:
        """ModerateAsync for many prompts in one batched pass over the GPUs;
        each result is the one moderate() gives for that prompt alone."""
        reqs = [np.ascontiguousarray(p, np.int32).reshape(-1) for p in prompts]
        if not reqs:
            return []
        yes, no, score, _ = self.ctx.score_batch(reqs, self.verdict_ids, self.yes_ids.size, cancel)
        return [ModerationResult(float(score[i]), float(yes[i]), float(no[i]), int(r.size),
                                 self.prefilled_tokens(r)) for i, r in enumerate(reqs)]

    def verdict_logits(self, ids, cancel: np.ndarray | None = None) -> np.ndarray:
        """VerdictLogitsAsync: every vocabulary logit at the verdict position."""
        return self.ctx.last_logits([np.ascontiguousarray(ids, np.int32).reshape(-1)], cancel)[0]

    def top_verdict_token(self, ids, cancel: np.ndarray | None = None) -> int:
        """TopVerdictTokenAsync's token, as an id: Kernels.ArgMax
        (Kernels.cs:223, TensorPrimitives.IndexOfMax) takes the first of equal
        maxima, as numpy's argmax does."""
        return int(np.argmax(self.verdict_logits(ids, cancel)))
