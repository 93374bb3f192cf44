"""GPU tests of incremental forwards on a KV cache: prefill, then decode one
token at a time, as the reference's Benchmark decode loop does
(Benchmark.cs:399-410) through MinistralModel.ForwardAsync and its KvCache.

Every logit after every step must equal the full head of the whole history
forwarded in one piece — the reference's own cache invariant.
"""
from __future__ import annotations

import numpy as np
import pytest

from llm_shield_b200 import binding, synth
from helpers import oracle_model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=[synth.Q4_0, synth.Q8_0], ids=lambda q: synth.TYPE_NAMES[q])
def model(request, shield_lib):
    spec = synth.small_spec(qtype=request.param, n_layers=3, seed=71 + request.param)
    tensors = synth.make_model(spec)
    ctx = binding.ShieldContext(1)
    ctx.set_config(spec, max_positions=512, max_batch_tokens=1024)
    ctx.upload_model(tensors)
    yield spec, tensors, ctx
    ctx.close()


def test_prefill_then_greedy_decode_matches_whole_forwards(model):
    spec, tensors, ctx = model
    prompt = np.random.default_rng(1).integers(1, spec.vocab, size=45, dtype=np.int32)
    s = ctx.seq_create(128)
    try:
        logits = ctx.seq_forward([s], [prompt])[0]
        history = list(prompt)
        np.testing.assert_array_equal(logits, ctx.last_logits([np.array(history, np.int32)])[0])
        for step in range(6):
            nxt = int(np.argmax(logits))  # greedy, as the benchmark picks its token
            logits = ctx.seq_forward([s], [np.array([nxt], np.int32)])[0]
            history.append(nxt)
            np.testing.assert_array_equal(logits, ctx.last_logits([np.array(history, np.int32)])[0],
                                          err_msg=f"decode step {step}")
        assert ctx.seq_length(s) == len(history)
        om = oracle_model(spec, tensors)
        np.testing.assert_array_equal(logits, om.forward(np.array(history, np.int32),
                                                         np.arange(spec.vocab, dtype=np.int32)))
    finally:
        ctx.seq_release(s)


def test_batched_decode_of_unequal_sequences_and_chunked_prefill(model):
    spec, _, ctx = model
    rng = np.random.default_rng(2)
    prompts = [rng.integers(1, spec.vocab, size=n, dtype=np.int32) for n in (3, 70, 31)]
    seqs = [ctx.seq_create(160) for _ in prompts]
    try:
        # prefill in uneven chunks, the three sequences together
        ctx.seq_forward(seqs, [p[:2] for p in prompts])
        out = ctx.seq_forward(seqs, [p[2:] for p in prompts])
        ref = ctx.last_logits(prompts)
        np.testing.assert_array_equal(out, ref)
        hist = [list(p) for p in prompts]
        for step in range(4):  # one token per sequence per step, all in one forward
            toks = [int(rng.integers(1, spec.vocab)) for _ in seqs]
            out = ctx.seq_forward(seqs, [np.array([t], np.int32) for t in toks])
            for h, t in zip(hist, toks):
                h.append(t)
            np.testing.assert_array_equal(out, ctx.last_logits([np.array(h, np.int32) for h in hist]),
                                          err_msg=f"step {step}")
        # a reset sequence starts over
        ctx.seq_reset(seqs[1])
        assert ctx.seq_length(seqs[1]) == 0
        again = ctx.seq_forward([seqs[1]], [prompts[1]])[0]
        np.testing.assert_array_equal(again, ref[1])
    finally:
        for s in seqs:
            ctx.seq_release(s)


def test_sequence_arguments_are_checked(model):
    spec, _, ctx = model
    s = ctx.seq_create(8)
    try:
        ids = np.arange(1, 7, dtype=np.int32)
        ctx.seq_forward([s], [ids], want_logits=False)
        with pytest.raises(binding.ShieldError) as e:  # 6 + 3 > capacity 8: nothing appended
            ctx.seq_forward([s], [ids[:3]])
        assert e.value.code == binding.ERR_RANGE
        assert ctx.seq_length(s) == 6
        with pytest.raises(binding.ShieldError) as e:
            ctx.seq_forward([s, s], [ids[:1], ids[:1]])
        assert e.value.code == binding.ERR_ARG
        with pytest.raises(binding.ShieldError) as e:
            ctx.seq_create(513)  # more than max_positions
        assert e.value.code == binding.ERR_RANGE
    finally:
        ctx.seq_release(s)
    with pytest.raises(binding.ShieldError) as e:
        ctx.seq_length(s)
    assert e.value.code == binding.ERR_ARG
