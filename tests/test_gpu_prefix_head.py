"""GPU tests of the two rows after the scoring path: the system-prompt prefix
cache and the full vocabulary head at the last position.

The prefix cache must not change a single bit (SystemPromptCacheTests.cs:41-74
asserts the same of the reference's cache), and the full head must agree with
the row-subset head used for verdicts (MatMulTilingTests.cs:67-87) and with
the oracle.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from llm_shield_b200 import binding, prefix_file, synth
from helpers import oracle_model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=[synth.Q4_0, synth.Q5_1], ids=lambda q: synth.TYPE_NAMES[q])
def model(request, shield_lib):
    spec = synth.small_spec(qtype=request.param, n_layers=3, seed=61 + request.param)
    tensors = synth.make_model(spec)
    ctx = binding.ShieldContext(1)
    ctx.set_config(spec, max_positions=512, max_batch_tokens=1024)
    ctx.upload_model(tensors)
    yield spec, tensors, ctx
    ctx.close()


def _requests(spec, prefix):
    rng = np.random.default_rng(11)
    suffix = lambda n: rng.integers(1, spec.vocab, size=n, dtype=np.int32)
    return [
        np.concatenate([prefix, suffix(1)]),          # one token after the prefix
        np.concatenate([prefix, suffix(37)]),
        np.concatenate([prefix, suffix(150)]),        # crosses several attention tiles
        suffix(60),                                    # does not start with the prefix
        prefix.copy(),                                 # the prefix alone: forwarded whole
        prefix[:20].copy(),                            # shorter than the prefix
        np.concatenate([prefix[:-1], suffix(9)]),     # differs in the prefix's last token
        np.concatenate([prefix, suffix(64)]),
    ]


def test_prefix_cache_leaves_every_bit_unchanged(model):
    spec, _, ctx = model
    prefix = np.random.default_rng(5).integers(1, spec.vocab, size=34, dtype=np.int32)
    reqs = _requests(spec, prefix)
    args = (spec.verdict_ids, len(spec.yes_ids))
    y0, n0, s0, l0 = ctx.score_batch(reqs, *args)
    ctx.set_prefix(prefix)
    try:
        y1, n1, s1, l1 = ctx.score_batch(reqs, *args)
        np.testing.assert_array_equal(l1, l0)
        np.testing.assert_array_equal(s1, s0)
        np.testing.assert_array_equal(y1, y0)
        np.testing.assert_array_equal(n1, n0)
        # alone and reordered, with the cache in place
        for r in (0, 2, 3):
            np.testing.assert_array_equal(ctx.score_batch([reqs[r]], *args)[3][0], l0[r])
        np.testing.assert_array_equal(ctx.score_batch(reqs[::-1], *args)[3][::-1], l0)
    finally:
        ctx.set_prefix([])
    np.testing.assert_array_equal(ctx.score_batch(reqs, *args)[3], l0)


def test_prefix_cache_is_dropped_when_the_weights_change(model):
    spec, tensors, ctx = model
    prefix = np.random.default_rng(6).integers(1, spec.vocab, size=16, dtype=np.int32)
    reqs = [np.concatenate([prefix, np.arange(1, 30, dtype=np.int32)])]
    args = (spec.verdict_ids, len(spec.yes_ids))
    ref = ctx.score_batch(reqs, *args)[3]
    ctx.set_prefix(prefix)
    name = "blk.1.attn_v.weight"
    t = tensors[name]
    ctx.upload(name, t["type"], t["rows"], t["cols"], t["data"])  # same bytes, cache must go anyway
    np.testing.assert_array_equal(ctx.score_batch(reqs, *args)[3], ref)


def test_prefix_arguments_are_checked(model):
    spec, _, ctx = model
    with pytest.raises(binding.ShieldError) as e:
        ctx.set_prefix(np.ones(512, np.int32))  # max_positions 512 leaves no room after it
    assert e.value.code == binding.ERR_RANGE
    with pytest.raises(binding.ShieldError) as e:
        ctx.set_prefix(np.array([1, spec.vocab], np.int32))
    assert e.value.code == binding.ERR_RANGE


def test_full_head_matches_the_verdict_rows_and_the_oracle(model):
    spec, tensors, ctx = model
    prefix = np.random.default_rng(7).integers(1, spec.vocab, size=34, dtype=np.int32)
    reqs = _requests(spec, prefix)
    full = ctx.last_logits(reqs)
    assert full.shape == (len(reqs), spec.vocab)
    _, _, _, verdict = ctx.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))
    np.testing.assert_array_equal(full[:, spec.verdict_ids], verdict)
    om = oracle_model(spec, tensors)
    vocab = np.arange(spec.vocab, dtype=np.int32)
    for r in (0, 3, 5):
        np.testing.assert_array_equal(full[r], om.forward(reqs[r], vocab), err_msg=f"request {r}")
    ctx.set_prefix(prefix)
    try:
        np.testing.assert_array_equal(ctx.last_logits(reqs), full)
    finally:
        ctx.set_prefix([])


def _oracle_snapshot(spec, tensors, prefix):
    """KvCache.Snapshot (KvCache.cs:102-118) of the oracle's forward of the
    prefix: per layer its keys after RoPE and its values, [kv head][position]
    [head_dim], keys of every layer first."""
    om = oracle_model(spec, tensors)
    parts = {oracle.CAP_K_ROPE: [], oracle.CAP_V: []}
    for what in parts:
        for layer in range(spec.n_layers):
            _, cap = om.forward(prefix, np.array([0], np.int32), capture_layer=layer, capture_what=what)
            parts[what].append(cap.reshape(prefix.size, spec.n_kv_heads, spec.head_dim).transpose(1, 0, 2).ravel())
    return np.concatenate(parts[oracle.CAP_K_ROPE] + parts[oracle.CAP_V])


def test_prefix_state_is_the_oracle_snapshot_and_restores_bit_identically(model):
    spec, tensors, ctx = model
    prefix = np.random.default_rng(12).integers(1, spec.vocab, size=34, dtype=np.int32)
    reqs = _requests(spec, prefix)
    args = (spec.verdict_ids, len(spec.yes_ids))
    ref = ctx.score_batch(reqs, *args)[3]
    ctx.set_prefix(prefix)
    try:
        assert ctx.prefix_length() == prefix.size
        state = ctx.get_prefix_state()
        np.testing.assert_array_equal(state, _oracle_snapshot(spec, tensors, prefix))
        ctx.set_prefix([])
        assert ctx.prefix_length() == 0
        with pytest.raises(binding.ShieldError) as e:
            ctx.get_prefix_state()
        assert e.value.code == binding.ERR_STATE
        ctx.set_prefix_state(prefix, state)  # no prefill: the snapshot goes to the GPU as it is
        assert ctx.prefix_length() == prefix.size
        np.testing.assert_array_equal(ctx.score_batch(reqs, *args)[3], ref)
        np.testing.assert_array_equal(ctx.get_prefix_state(), state)
        with pytest.raises(binding.ShieldError) as e:  # KvCache.Restore's size check
            ctx.set_prefix_state(prefix[:-1], state)
        assert e.value.code == binding.ERR_ARG
        assert ctx.prefix_length() == prefix.size  # a rejected snapshot leaves the cache alone
        with pytest.raises(binding.ShieldError) as e:
            ctx.set_prefix_state(np.full(34, spec.vocab, np.int32), state)
        assert e.value.code == binding.ERR_RANGE
        np.testing.assert_array_equal(ctx.get_prefix_state(), state)
    finally:
        ctx.set_prefix([])


def test_snapshot_file_skips_the_prefill(model, tmp_path):
    spec, _, ctx = model
    weights = tmp_path / "model.gguf"
    weights.write_bytes(b"synthetic")
    ident = prefix_file.ModelIdentity(str(weights), "mistral3", spec.n_layers, spec.n_kv_heads, spec.head_dim)
    prefix = np.random.default_rng(13).integers(1, spec.vocab, size=20, dtype=np.int32)
    reqs = _requests(spec, prefix)
    args = (spec.verdict_ids, len(spec.yes_ids))
    ref = ctx.score_batch(reqs, *args)[3]
    path = tmp_path / "prefix.shkv"
    try:
        captured = prefix_file.load_or_capture(ctx, ident, prefix, path)
        ctx.set_prefix([])
        restored = prefix_file.load_or_capture(ctx, ident, prefix, path)
        np.testing.assert_array_equal(restored.state, captured.state)
        np.testing.assert_array_equal(ctx.score_batch(reqs, *args)[3], ref)
    finally:
        ctx.set_prefix([])
