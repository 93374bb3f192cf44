"""GPU test of shield_qmatmul_noalloc, the GEMM entry point that allocates no
device memory.

Callers that hand all GPU memory to their own pool, or that may not allocate
on their request path, use it instead of shield_qmatmul_device; its scratch
is a fixed device array inside the library.  This file is collected last so
that a run stopping at its first failure has already run every other test.

Each case is checked against the allocating entry point and against the CPU
oracle (the reference's integer GEMM arithmetic), bit for bit: the kernels
are the same, only where their scratch lives differs.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
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


# (type, rows, cols, M, weight name): the tensor-core kernel on the
# once-unpacked layer copy (M = 200, and M = 600 at K = 3072, just under the
# scratch limit), the few-token kernel (M = 5), and the CUDA-core kernel
# (K = 256 has no tensor-core tile); the raw-block kernel is checked below
CASES = [(synth.Q4_0, 256, 3072, 200, "blk.0.attn_q.weight"),
         (synth.Q5_1, 100, 256, 13, "blk.0.attn_k.weight"),
         (synth.Q4_0, 512, 3072, 600, "blk.0.ffn_gate.weight"),
         (synth.Q8_0, 384, 3072, 5, "blk.0.ffn_up.weight")]


def test_noalloc_matches_the_allocating_entry_point_and_the_oracle(ctx):
    """Calls in a row, each equal to shield_qmatmul_device and to the oracle:
    the shared scratch keeps the previous call's contents, which must not
    leak into the next call."""
    torch = pytest.importorskip("torch")
    weights = {}
    for i, (qtype, rows, cols, M, name) in enumerate(CASES):
        assert M * cols <= LIMIT
        w = random_weights(qtype, rows, cols, seed=40 + i)
        weights[name] = w
        ctx.upload(name, qtype, rows, cols, w)
    for i, (qtype, rows, cols, M, name) in enumerate(CASES):
        x = np.random.default_rng(i).standard_normal((M, cols)).astype(np.float32)
        got = _run(ctx, torch, name, x, rows, noalloc=True)
        np.testing.assert_array_equal(got, _run(ctx, torch, name, x, rows, noalloc=False), err_msg=name)
        np.testing.assert_array_equal(got, oracle.qmatmul(qtype, weights[name], rows, cols, x, M), err_msg=name)
    # the first shape again, after the other calls overwrote the scratch
    qtype, rows, cols, M, name = CASES[0]
    x = np.random.default_rng(7).standard_normal((M, cols)).astype(np.float32)
    got = _run(ctx, torch, name, x, rows, noalloc=True)
    np.testing.assert_array_equal(got, _run(ctx, torch, name, x, rows, noalloc=False))
    np.testing.assert_array_equal(got, oracle.qmatmul(qtype, weights[name], rows, cols, x, M))


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


def test_noalloc_follows_the_selected_kernel(ctx):
    """shield_set_gemm_path applies here too: the raw-block tensor-core kernel
    (path 2) gives the oracle's outputs, and the few-token kernel alone
    (path 4) refuses 17 tokens, as the allocating entry points do."""
    torch = pytest.importorskip("torch")
    rows, cols = 128, 3072
    w = random_weights(synth.Q4_0, rows, cols, seed=9)
    ctx.upload("blk.0.attn_output.weight", synth.Q4_0, rows, cols, w)
    x = np.random.default_rng(3).standard_normal((200, cols)).astype(np.float32)
    ctx.set_gemm_path(2)
    try:
        got = _run(ctx, torch, "blk.0.attn_output.weight", x, rows, noalloc=True)
    finally:
        ctx.set_gemm_path(0)
    np.testing.assert_array_equal(got, oracle.qmatmul(synth.Q4_0, w, rows, cols, x, 200))
    dx = torch.zeros((17, cols), dtype=torch.float32, device="cuda")
    dy = torch.zeros((17, rows), dtype=torch.float32, device="cuda")
    ctx.set_gemm_path(4)
    try:
        with pytest.raises(binding.ShieldError) as e:
            ctx.qmatmul_noalloc("blk.0.attn_output.weight", dx.data_ptr(), 17, dy.data_ptr())
        assert e.value.code == binding.ERR_UNSUPPORTED
    finally:
        ctx.set_gemm_path(0)
