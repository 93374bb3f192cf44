"""Several GPUs in one context: requests are sharded over the GPUs (longest
processing time first), each with a full weight replica and no collective.
The results must not depend on the number of GPUs (the GPU analogue of
MatMulTilingTests.cs:42-65). Skipped on a box with one GPU."""
from __future__ import annotations

import numpy as np
import pytest

from llm_shield_b200 import binding, synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def two(shield_lib):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    spec = synth.small_spec(qtype=synth.Q4_0, n_layers=2, seed=91)
    tensors = synth.make_model(spec)
    ctxs = []
    for mask in (1, 3):
        c = binding.ShieldContext(mask)
        c.set_config(spec, max_positions=512, max_batch_tokens=1024)
        c.upload_model(tensors)
        ctxs.append(c)
    yield spec, ctxs
    for c in ctxs:
        c.close()


def test_scores_and_full_head_do_not_depend_on_the_gpu_count(two):
    spec, (one, both) = two
    assert both.device_count == 2
    lengths = [3, 200, 17, 64, 1, 120, 45, 9, 300, 33, 77, 2]
    reqs = synth.random_requests(len(lengths), lengths, seed=4, vocab=spec.vocab)
    a = one.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))
    b = both.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)
    np.testing.assert_array_equal(one.last_logits(reqs), both.last_logits(reqs))


def test_prefix_cache_on_both_gpus(two):
    spec, (one, both) = two
    prefix = np.random.default_rng(8).integers(1, spec.vocab, size=30, dtype=np.int32)
    rng = np.random.default_rng(9)
    reqs = [np.concatenate([prefix, rng.integers(1, spec.vocab, size=n, dtype=np.int32)]) for n in (5, 90, 1, 40)]
    ref = one.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))[3]
    both.set_prefix(prefix)
    try:
        np.testing.assert_array_equal(both.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))[3], ref)
        # a snapshot taken on one GPU, restored onto both without a prefill
        one.set_prefix(prefix)
        state = one.get_prefix_state()
        np.testing.assert_array_equal(both.get_prefix_state(), state)
        both.set_prefix([])
        both.set_prefix_state(prefix, state)
        np.testing.assert_array_equal(both.score_batch(reqs, spec.verdict_ids, len(spec.yes_ids))[3], ref)
    finally:
        one.set_prefix([])
        both.set_prefix([])


def test_sequences_on_the_second_gpu(two):
    spec, (one, both) = two
    prompt = np.random.default_rng(10).integers(1, spec.vocab, size=50, dtype=np.int32)
    s0, s1 = both.seq_create(64, device=0), both.seq_create(64, device=1)
    try:
        out = both.seq_forward([s0, s1], [prompt, prompt[:20]])
        np.testing.assert_array_equal(out, one.last_logits([prompt, prompt[:20]]))
        step = both.seq_forward([s1, s0], [np.array([7], np.int32), np.array([9], np.int32)])
        ref = one.last_logits([np.concatenate([prompt[:20], [7]]).astype(np.int32),
                               np.concatenate([prompt, [9]]).astype(np.int32)])
        np.testing.assert_array_equal(step, ref)
    finally:
        both.seq_release(s0)
        both.seq_release(s1)
