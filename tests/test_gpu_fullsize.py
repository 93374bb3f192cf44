"""The benchmark's model at full size: Shieldstral-3B's shape (26 layers,
d 3072, 32/8 heads x 128, FFN 9216, vocab 131072, YaRN), Q4_0, the same
seeded synthetic weights bench.py scores, on requests drawn like its
config-5 workload (lognormal lengths, median 300, sigma 0.6, [32, 4096]).

Short requests are checked against the oracle bit for bit (logits, scores,
the full head); the rest through properties that hold at any size: results
independent of batch composition, order and micro-batching
(MatMulTilingTests.cs:42-65), a 4096-token request at the length limit,
incremental forwards equal to whole ones, Score consistent with the logits
(ShieldstralModerator.cs:348-364).
"""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest

import oracle
from llm_shield_b200 import binding, gguf_file, synth
from helpers import oracle_model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def big(shield_lib, tmp_path_factory):
    """The model written as a GGUF file and uploaded from its read-only
    mapping (GgufFile.GetTensorPointer, GgufFile.cs:195-199); the config comes
    from the file's metadata (ModelConfig.FromGguf)."""
    path = gguf_file.write_model(tmp_path_factory.mktemp("gguf") / "shieldstral_q4_0.gguf", synth.SHIELDSTRAL_3B)
    g = gguf_file.GgufFile(path)
    spec = dataclasses.replace(synth.SHIELDSTRAL_3B, **{f: getattr(g.spec(), f) for f in (
        "n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab", "yes_ids", "no_ids", "qtype")})
    tensors = g.tensors()
    ctx = binding.ShieldContext(1)
    ctx.set_config(spec, max_positions=4096, max_batch_tokens=16384)
    ctx.upload_model(tensors)
    yield spec, tensors, ctx
    ctx.close()


def _args(spec):
    return spec.verdict_ids, len(spec.yes_ids)


def test_short_requests_match_the_oracle_bit_for_bit(big):
    spec, tensors, ctx = big
    reqs = synth.random_requests(3, [32, 90, 200], seed=501, vocab=spec.vocab)
    yes, no, score, logits = ctx.score_batch(reqs, *_args(spec))
    om = oracle_model(spec, tensors)
    n_yes, n_no = len(spec.yes_ids), len(spec.no_ids)
    for r, ids in enumerate(reqs):
        ref = om.forward(ids, np.asarray(spec.verdict_ids, np.int32))
        np.testing.assert_array_equal(logits[r], ref, err_msg=f"request {r}")
        rs, ry, rn = oracle.score(ref, n_yes, n_no)
        assert (score[r], yes[r], no[r]) == (np.float32(rs), np.float32(ry), np.float32(rn))
    full = ctx.last_logits(reqs[:1])[0]
    np.testing.assert_array_equal(full, om.forward(reqs[0], np.arange(spec.vocab, dtype=np.int32)))


def test_config5_batch_is_independent_of_composition_and_order(big):
    spec, _, ctx = big
    lengths = synth.lognormal_lengths(96, seed=502)
    lengths[17] = 4096  # one request at the length limit
    reqs = synth.random_requests(len(lengths), lengths, seed=503, vocab=spec.vocab)
    yes, no, score, logits = ctx.score_batch(reqs, *_args(spec))  # several micro-batches
    assert np.isfinite(logits).all()
    assert ((score >= 0) & (score <= 1)).all()
    n_yes = len(spec.yes_ids)
    np.testing.assert_array_equal(yes, logits[:, :n_yes].max(axis=1))
    np.testing.assert_array_equal(no, logits[:, n_yes:].max(axis=1))
    for r in (0, 17, 50):
        np.testing.assert_array_equal(score[r], np.float32(oracle.score(logits[r], n_yes, len(spec.no_ids))[0]))
    rev = ctx.score_batch(reqs[::-1], *_args(spec))[3][::-1]
    np.testing.assert_array_equal(rev, logits)
    for lo, hi in ((0, 7), (7, 40), (40, 96)):
        np.testing.assert_array_equal(ctx.score_batch(reqs[lo:hi], *_args(spec))[3], logits[lo:hi])
    for r in (3, 17, 95):
        np.testing.assert_array_equal(ctx.score_batch([reqs[r]], *_args(spec))[3][0], logits[r])


def test_incremental_forwards_equal_whole_ones(big):
    spec, _, ctx = big
    prompt = synth.random_requests(1, [300], seed=504, vocab=spec.vocab)[0]
    s = ctx.seq_create(320)
    try:
        ctx.seq_forward([s], [prompt[:120]], want_logits=False)
        out = ctx.seq_forward([s], [prompt[120:]])[0]
        np.testing.assert_array_equal(out, ctx.last_logits([prompt])[0])
        nxt = np.array([int(np.argmax(out))], np.int32)
        step = ctx.seq_forward([s], [nxt])[0]
        np.testing.assert_array_equal(step, ctx.last_logits([np.concatenate([prompt, nxt])])[0])
    finally:
        ctx.seq_release(s)
