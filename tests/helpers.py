"""Shared builders for the parity tests: synthetic models and their oracle twins."""
from __future__ import annotations

import numpy as np

import oracle
from llm_shield_b200 import synth


def oracle_config(spec: synth.ModelSpec) -> dict:
    yarn = spec.yarn_factor > 1.0 and spec.yarn_orig_ctx > 0
    freqs, mscale = oracle.rope_freqs(spec.head_dim, spec.rope_theta, spec.yarn_factor if yarn else 1.0, yarn,
                                      spec.yarn_orig_ctx, spec.yarn_beta_fast, spec.yarn_beta_slow, 1.0, 1.0, 1.0, 1.0)
    return dict(n_layers=spec.n_layers, hidden=spec.hidden, n_heads=spec.n_heads, n_kv_heads=spec.n_kv_heads,
                head_dim=spec.head_dim, ffn=spec.ffn, vocab=spec.vocab, rms_eps=spec.rms_eps, rope_freqs=freqs,
                rope_mscale=mscale, attn_temperature_beta=spec.attn_temperature_beta,
                rope_orig_ctx=spec.yarn_orig_ctx)


def oracle_model(spec: synth.ModelSpec, tensors: dict) -> oracle.Model:
    return oracle.Model(oracle_config(spec), tensors)


def random_weights(qtype: int, rows: int, cols: int, seed: int) -> np.ndarray:
    """Random payload bytes with every f16 scale (and offset) forced to a sane
    value, as the reference's MatMulTilingTests.Weights does (:131-154)."""
    rng = np.random.default_rng(seed)
    bb = synth.BLOCK_BYTES[qtype]
    raw = rng.integers(0, 256, size=rows * cols // 32 * bb, dtype=np.uint8).reshape(-1, bb)
    raw[:, 0:2] = np.frombuffer(
        (0.005 + 0.02 * rng.random(raw.shape[0])).astype(np.float16).tobytes(), np.uint8).reshape(-1, 2)
    if qtype in (synth.Q4_1, synth.Q5_1):
        raw[:, 2:4] = np.frombuffer((-0.03 * rng.random(raw.shape[0])).astype(np.float16).tobytes(),
                                    np.uint8).reshape(-1, 2)
    return raw.reshape(-1)
