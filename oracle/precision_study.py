"""What a tensor-core attention would do to the scores -- TEST
INFRASTRUCTURE, run on the CPU, never by the product.

The CUDA library's attention keeps the reference's f32 order of arithmetic
(MinistralModel.cs:372-440), which keeps it on the CUDA cores. A tensor-core
version would feed the products TF32 or BF16 operands with f32 accumulation.
This script runs the oracle's forward with exactly that operand rounding in
both attention products (orc_config.attn_operand_bits) on the benchmark's 3B
Q4_0 model and config-5-shaped requests, and reports the drift of the yes/no
logits, of Score and of the verdicts against the exact forward, next to the
north star's bars (logits 1e-3 relative, Score 1e-4 absolute, identical
verdicts).

    python oracle/precision_study.py [--requests 12] [--seed 7]
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests"))

import oracle  # noqa: E402
from helpers import oracle_config  # noqa: E402
from llm_shield_b200 import synth  # noqa: E402


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--requests", type=int, default=12)
    ap.add_argument("--seed", type=int, default=7)
    args = ap.parse_args(argv)
    spec = synth.SHIELDSTRAL_3B
    tensors = synth.make_model(spec)
    lengths = synth.lognormal_lengths(args.requests, seed=args.seed)
    reqs = synth.random_requests(args.requests, lengths, seed=args.seed + 1, vocab=spec.vocab)
    vid = np.asarray(spec.verdict_ids, np.int32)
    n_yes, n_no = len(spec.yes_ids), len(spec.no_ids)
    models = {}
    for name, bits in (("f32 (reference order)", 0), ("TF32 operands", 10), ("BF16 operands", 7)):
        cfg = oracle_config(spec)
        cfg["attn_operand_bits"] = bits
        models[name] = oracle.Model(cfg, tensors)
    exact = [models["f32 (reference order)"].forward(r, vid) for r in reqs]
    rows = []
    for name, m in models.items():
        if name.startswith("f32"):
            continue
        rel = ds = 0.0
        flips = 0
        for r, ref in zip(reqs, exact):
            got = m.forward(r, vid)
            rel = max(rel, float(np.abs(got - ref).max() / max(1.0, np.abs(ref).max())))
            s_got = oracle.score(got, n_yes, n_no)[0]
            s_ref = oracle.score(ref, n_yes, n_no)[0]
            ds = max(ds, abs(s_got - s_ref))
            flips += (s_got > 0.5) != (s_ref > 0.5)
        rows.append({"attention operands": name, "max_logit_rel": rel, "max_score_abs": ds, "verdict_flips": flips,
                     "requests": len(reqs), "passes": rel <= 1e-3 and ds <= 1e-4 and flips == 0})
    for row in rows:
        print(json.dumps(row), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
