"""GPU parity of the whole scoring prefill (shield_score_batch) against the
oracle's restatement of MinistralModel.ForwardSelectedAsync + Score.

Bars: the north star's (yes/no logits within 1e-3 relative, Score within
1e-4 absolute, identical verdicts at 0.5) and, stricter, bit-identical logits:
the GPU path evaluates every step in the oracle's order with the same exp, so
nothing but the operations themselves can differ.  Bit-exactness matters here
because the activations are re-quantized to int8 before every GEMM: a one-ulp
difference upstream can flip a rounding and move later layers by ~1e-3."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from llm_shield_b200 import binding, synth
from helpers import oracle_model

pytestmark = pytest.mark.gpu
LOGIT_RTOL = 1e-3
SCORE_ATOL = 1e-4


def check_against_oracle(om, spec, requests, yes, no, score, logits, exact=True):
    nyes = len(spec.yes_ids)
    for r, ids in enumerate(requests):
        ref = om.forward(ids, spec.verdict_ids)
        rs, ry, rn = oracle.score(ref, nyes, len(spec.no_ids))
        if exact:
            np.testing.assert_array_equal(logits[r], ref, err_msg=f"request {r}")
            assert score[r] == np.float32(rs) and yes[r] == np.float32(ry) and no[r] == np.float32(rn)
        scale = max(1.0, float(np.abs(ref).max()))
        assert np.abs(logits[r] - ref).max() <= LOGIT_RTOL * scale, (r, logits[r], ref)
        assert abs(score[r] - rs) <= SCORE_ATOL
        assert (score[r] > 0.5) == (rs > 0.5)
        assert abs(yes[r] - ry) <= LOGIT_RTOL * scale and abs(no[r] - rn) <= LOGIT_RTOL * scale


@pytest.fixture(scope="module", params=[synth.Q4_0, synth.Q5_1, synth.Q8_0, synth.Q5_0, synth.Q4_1],
                ids=lambda q: synth.TYPE_NAMES[q])
def small(request, shield_lib):
    spec = synth.small_spec(qtype=request.param, n_layers=3, seed=31 + request.param)
    tensors = synth.make_model(spec)
    ctx = binding.ShieldContext(1)
    ctx.set_config(spec, max_positions=1024, max_batch_tokens=2048)
    ctx.upload_model(tensors)
    om = oracle_model(spec, tensors)
    yield spec, tensors, ctx, om
    ctx.close()


def test_ragged_batch_matches_oracle(small):
    spec, _, ctx, om = small
    lengths = [1, 7, 33, 100, 2, 257]
    reqs = synth.random_requests(len(lengths), lengths, seed=5, vocab=spec.vocab)
    yes, no, score, logits = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))
    check_against_oracle(om, spec, reqs, yes, no, score, logits)


@pytest.mark.parametrize("rows", [64, 128])
def test_attention_rows_per_cta_bit_identical_to_oracle(small, rows):
    """Both sizes of the attention kernel's CTA (64 or 128 query rows; the
    automatic choice takes 64 for small or sparsely filled micro-batches)
    give the oracle's logits bit for bit, with requests that end inside and
    exactly at a CTA's rows."""
    spec, _, ctx, om = small
    lengths = [1, 4, 5, 17, 64, 130]
    reqs = synth.random_requests(len(lengths), lengths, seed=rows, vocab=spec.vocab)
    ctx.set_attention_rows(rows)
    try:
        yes, no, score, logits = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))
    finally:
        ctx.set_attention_rows(0)
    check_against_oracle(om, spec, reqs, yes, no, score, logits)


def test_results_do_not_depend_on_batching(small):
    """A request's logits are bit-identical alone and inside any batch."""
    spec, _, ctx, _ = small
    lengths = [5, 40, 1, 64, 13]
    reqs = synth.random_requests(len(lengths), lengths, seed=9, vocab=spec.vocab)
    _, _, s_all, l_all = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))
    for r, ids in enumerate(reqs):
        _, _, s1, l1 = ctx.score_batch([ids], spec.verdict_ids, len(spec.yes_ids))
        np.testing.assert_array_equal(l1[0], l_all[r])
        assert s1[0] == s_all[r]
    _, _, s_rev, l_rev = ctx.score_batch(reqs[::-1], spec.verdict_ids, len(spec.yes_ids))
    np.testing.assert_array_equal(l_rev[::-1], l_all)


@pytest.mark.parametrize("what", [binding.ACT_ATTN_NORM, binding.ACT_Q_ROPE, binding.ACT_K_ROPE, binding.ACT_V,
                                  binding.ACT_ATTN_WEIGHTED, binding.ACT_POST_ATTN, binding.ACT_OUTPUT])
def test_layer_activations_match_oracle(small, what):
    """Every IActivationSink tensor of every layer against the oracle."""
    spec, _, ctx, om = small
    ids = synth.random_requests(1, [48], seed=3, vocab=spec.vocab)[0]
    for layer in range(spec.n_layers):
        got = ctx.activation(ids, layer, what)
        _, ref = om.forward(ids, spec.verdict_ids, capture_layer=layer, capture_what=what)
        np.testing.assert_array_equal(got, ref, err_msg=f"layer {layer} activation {what}")


def test_micro_batches_split_across_calls_give_identical_results(shield_lib):
    """max_batch_tokens smaller than the batch forces several micro-batches."""
    spec = synth.small_spec(qtype=synth.Q4_0, n_layers=2, seed=4)
    tensors = synth.make_model(spec)
    reqs = synth.random_requests(6, [100, 90, 80, 70, 60, 50], seed=1, vocab=spec.vocab)
    out = []
    for mbt in (128, 4096):
        with binding.ShieldContext(1) as ctx:
            ctx.set_config(spec, max_positions=128, max_batch_tokens=mbt)
            ctx.upload_model(tensors)
            out.append(ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))[3])
    np.testing.assert_array_equal(out[0], out[1])


def test_bad_token_ids_and_cancellation(shield_lib):
    spec = synth.small_spec(qtype=synth.Q4_0, n_layers=2, seed=8)
    tensors = synth.make_model(spec)
    with binding.ShieldContext(1) as ctx:
        ctx.set_config(spec, max_positions=256)
        ctx.upload_model(tensors)
        reqs = synth.random_requests(2, [10, 20], seed=2, vocab=spec.vocab)
        before = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))[3]
        with pytest.raises(binding.ShieldArgumentOutOfRange):
            ctx.score_batch([np.array([1, spec.vocab], np.int32)], spec.verdict_ids, len(spec.yes_ids))
        with pytest.raises(binding.ShieldArgumentOutOfRange):
            ctx.score_batch([np.zeros(300, np.int32)], spec.verdict_ids, len(spec.yes_ids))
        cancel = np.ones(1, np.int32)
        with pytest.raises(binding.ShieldCancelled):
            ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids), cancel=cancel)
        # a cancelled pass leaves the context usable with identical results
        after = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))[3]
        np.testing.assert_array_equal(before, after)


def test_full_width_model_matches_oracle(shield_lib):
    """Shieldstral's real dimensions (d 3072, 32/8 heads x 128, FFN 9216,
    vocab 131072, YaRN) with a reduced layer count, Q4_0."""
    spec = synth.ModelSpec(n_layers=2, qtype=synth.Q4_0, seed=99)
    tensors = synth.make_model(spec)
    with binding.ShieldContext(1) as ctx:
        ctx.set_config(spec, max_positions=512)
        ctx.upload_model(tensors)
        om = oracle_model(spec, tensors)
        reqs = synth.random_requests(3, [1, 17, 200], seed=7, vocab=spec.vocab)
        yes, no, score, logits = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))
        check_against_oracle(om, spec, reqs, yes, no, score, logits)
