"""GPU parity on the benchmark configurations the other files do not reach.

* full depth (26 layers, the 3B shape) with Q5_1 and Q8_0 weights, short
  requests, bit-identical to the oracle;
* config 3's shape: full width, Q5_1, a ragged batch of 64 requests with
  lengths uniform in [128, 1024], reduced depth (2 layers) so the oracle can
  check several requests bit for bit, the rest through batch invariance;
* config 4's shape: full width, Q8_0, 16 requests of exactly 4096 tokens
  (several micro-batches, several attention groups), reduced depth, one
  request against the oracle and the rest through batch invariance;
* the attention temperature past the training window
  (MinistralModel.ApplyPositionScale, MinistralModel.cs:476-482), on a small
  model whose window is 64 positions.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest

import oracle
from llm_shield_b200 import binding, synth
from helpers import oracle_model

pytestmark = pytest.mark.gpu


def _check_exact(om, spec, reqs, yes, no, score, logits, which):
    n_yes, n_no = len(spec.yes_ids), len(spec.no_ids)
    for r in which:
        ref = om.forward(reqs[r], np.asarray(spec.verdict_ids, np.int32))
        np.testing.assert_array_equal(logits[r], ref, err_msg=f"request {r} ({len(reqs[r])} tokens)")
        rs, ry, rn = oracle.score(ref, n_yes, n_no)
        assert (score[r], yes[r], no[r]) == (np.float32(rs), np.float32(ry), np.float32(rn))
        assert (score[r] > 0.5) == (rs > 0.5)


def _model(spec, max_positions, max_batch_tokens):
    tensors = synth.make_model(spec)
    ctx = binding.ShieldContext(1)
    ctx.set_config(spec, max_positions=max_positions, max_batch_tokens=max_batch_tokens)
    ctx.upload_model(tensors)
    return tensors, ctx


@pytest.mark.parametrize("qtype", [synth.Q5_1, synth.Q8_0], ids=lambda q: synth.TYPE_NAMES[q])
def test_full_depth_model_matches_the_oracle(shield_lib, qtype):
    spec = dataclasses.replace(synth.SHIELDSTRAL_3B, qtype=qtype)
    tensors, ctx = _model(spec, 4096, 16384)
    try:
        reqs = synth.random_requests(3, [32, 90, 200], seed=600 + qtype, vocab=spec.vocab)
        out = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))
        _check_exact(oracle_model(spec, tensors), spec, reqs, *out, which=range(len(reqs)))
    finally:
        ctx.close()


def _invariance(ctx, spec, reqs, logits, picks):
    """Each picked request scored alone, and the batch reversed, give the
    batch's bits (MatMulTilingTests.cs:42-65 at the model level)."""
    args = (spec.verdict_ids, len(spec.yes_ids))
    for r in picks:
        np.testing.assert_array_equal(ctx.score_batch([reqs[r]], *args)[3][0], logits[r], err_msg=f"request {r}")
    np.testing.assert_array_equal(ctx.score_batch(reqs[::-1], *args)[3][::-1], logits)


def test_config3_shape_q5_1_ragged_batch(shield_lib):
    """Config 3: Q5_1, 64 requests with lengths uniform in [128, 1024]."""
    spec = dataclasses.replace(synth.SHIELDSTRAL_3B, qtype=synth.Q5_1, n_layers=2)
    tensors, ctx = _model(spec, 1024, 16384)
    try:
        lengths = np.random.default_rng(700).integers(128, 1025, size=64)
        lengths[5], lengths[40] = 128, 1024
        reqs = synth.random_requests(len(lengths), lengths, seed=701, vocab=spec.vocab)
        out = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))
        assert np.isfinite(out[3]).all()
        _check_exact(oracle_model(spec, tensors), spec, reqs, *out, which=(5, 40, 63))
        _invariance(ctx, spec, reqs, out[3], picks=(0, 40))
    finally:
        ctx.close()


def test_config4_shape_q8_0_long_documents(shield_lib):
    """Config 4: Q8_0, 16 requests of exactly 4096 tokens (4 micro-batches of
    16384 tokens, 2 attention groups in each)."""
    spec = dataclasses.replace(synth.SHIELDSTRAL_3B, qtype=synth.Q8_0, n_layers=2)
    tensors, ctx = _model(spec, 4096, 16384)
    try:
        reqs = synth.random_requests(16, [4096] * 16, seed=800, vocab=spec.vocab)
        out = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))
        assert np.isfinite(out[3]).all()
        _check_exact(oracle_model(spec, tensors), spec, reqs, *out, which=(11,))
        _invariance(ctx, spec, reqs, out[3], picks=(3,))
    finally:
        ctx.close()


def test_attention_temperature_past_the_training_window(shield_lib):
    """q *= 1 + beta * ln(1 + floor(pos / n_orig)) from position n_orig on
    (MinistralModel.cs:476-482): with a 64-position window, requests of 100
    and 200 tokens cross one, two and three window boundaries."""
    spec = dataclasses.replace(synth.small_spec(qtype=synth.Q4_0, n_layers=2, seed=71), yarn_orig_ctx=64,
                               attn_temperature_beta=0.1)
    tensors, ctx = _model(spec, 1024, 2048)
    try:
        reqs = synth.random_requests(3, [100, 200, 40], seed=900, vocab=spec.vocab)
        out = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))
        _check_exact(oracle_model(spec, tensors), spec, reqs, *out, which=range(3))
        # the factor is live: without it the long requests differ, the short one not
        ctx.set_config(dataclasses.replace(spec, attn_temperature_beta=0.0), max_positions=1024,
                       max_batch_tokens=2048)
        ctx.upload_model(tensors)
        plain = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))[3]
        assert not np.array_equal(plain[0], out[3][0]) and not np.array_equal(plain[1], out[3][1])
        np.testing.assert_array_equal(plain[2], out[3][2])
    finally:
        ctx.close()


@pytest.mark.parametrize("qtype,length", [(synth.Q8_0, 4096), (synth.Q5_1, 1024), (synth.Q4_0, 2048)],
                         ids=["config4-Q8_0-4096", "config3-Q5_1-1024", "config5-Q4_0-2048"])
def test_full_depth_long_request_matches_the_oracle(shield_lib, qtype, length):
    """The longest requests of configs 4, 3 and 5 through all 26 layers of the
    3B model, bit for bit against the oracle (each takes the oracle one to two
    minutes on the host cores), inside a batch with a short request."""
    spec = dataclasses.replace(synth.SHIELDSTRAL_3B, qtype=qtype)
    tensors, ctx = _model(spec, 4096, 16384)
    try:
        reqs = synth.random_requests(2, [length, 48], seed=1000 + qtype, vocab=spec.vocab)
        out = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))
        _check_exact(oracle_model(spec, tensors), spec, reqs, *out, which=(0,))
    finally:
        ctx.close()
