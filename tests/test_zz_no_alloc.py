"""GPU test of shield_qmatmul_noalloc, the GEMM entry point that allocates no
device memory.

Callers that hand all GPU memory to their own pool, or that may not allocate
on their request path, use it instead of shield_qmatmul_device; its scratch
is a fixed device array inside the library.  This file is collected last so
that a run stopping at its first failure has already run every other test.
"""
from __future__ import annotations

import numpy as np
import pytest

from llm_shield_b200 import binding, synth
from helpers import random_weights

pytestmark = pytest.mark.gpu

LIMIT = 1 << 21  # SHIELD_NOALLOC_MAX_ELEMENTS


@pytest.fixture(scope="module")
def ctx(shield_lib):
    c = binding.ShieldContext(1)
    c.set_config(synth.small_spec())
    yield c
    c.close()


def _run(ctx, torch, name, x, rows, noalloc):
    dx = torch.from_numpy(x).cuda()
    dy = torch.full((x.shape[0], rows), float("nan"), dtype=torch.float32, device="cuda")
    if noalloc:
        ctx.qmatmul_noalloc(name, dx.data_ptr(), x.shape[0], dy.data_ptr())
    else:
        ctx.qmatmul_device(name, dx.data_ptr(), x.shape[0], dy.data_ptr())
    torch.cuda.synchronize()
    return dy.cpu().numpy()


def test_noalloc_matches_the_allocating_entry_point_on_consecutive_calls(ctx):
    """Two calls in a row (tensor-core shape, then a CUDA-core shape with a
    different type) each give exactly what shield_qmatmul_device gives: the
    shared scratch keeps the previous call's contents, which must not leak."""
    torch = pytest.importorskip("torch")
    cases = [(synth.Q4_0, 256, 3072, 200, "blk.0.attn_q.weight"),
             (synth.Q5_1, 100, 256, 13, "blk.0.attn_k.weight")]
    for i, (qtype, rows, cols, M, name) in enumerate(cases):
        w = random_weights(qtype, rows, cols, seed=40 + i)
        ctx.upload(name, qtype, rows, cols, w)
        x = np.random.default_rng(i).standard_normal((M, cols)).astype(np.float32)
        got = _run(ctx, torch, name, x, rows, noalloc=True)
        ref = _run(ctx, torch, name, x, rows, noalloc=False)
        np.testing.assert_array_equal(got, ref)
    # and the first shape again, after the second call overwrote the scratch
    qtype, rows, cols, M, name = cases[0]
    x = np.random.default_rng(7).standard_normal((M, cols)).astype(np.float32)
    np.testing.assert_array_equal(_run(ctx, torch, name, x, rows, noalloc=True),
                                  _run(ctx, torch, name, x, rows, noalloc=False))


def test_noalloc_rejects_sizes_beyond_its_scratch(ctx):
    torch = pytest.importorskip("torch")
    rows, cols = 128, 3072
    ctx.upload("blk.0.attn_v.weight", synth.Q4_0, rows, cols, random_weights(synth.Q4_0, rows, cols, seed=3))
    M = LIMIT // cols + 1
    dx = torch.zeros((M, cols), dtype=torch.float32, device="cuda")
    dy = torch.zeros((M, rows), dtype=torch.float32, device="cuda")
    with pytest.raises(binding.ShieldError) as e:
        ctx.qmatmul_noalloc("blk.0.attn_v.weight", dx.data_ptr(), M, dy.data_ptr())
    assert e.value.code == binding.ERR_ARG and "scratch limit" in str(e.value)
