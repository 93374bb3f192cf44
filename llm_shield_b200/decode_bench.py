"""Decode throughput on one GPU: the reference benchmark's decode shape
(Benchmark.cs:399-410: single-token forwards onto a 256-token context),
batched over sequences.

    python -m llm_shield_b200.decode_bench --batch 1,16,64 --context 256 --tokens 32

For each batch size: every sequence is prefilled with a seeded random
256-token prompt, then `--tokens` decode steps append one token per sequence
(greedy on the full head). Times the decode steps with CUDA events on the
library's stream and prints one JSON line per batch size (the Shieldstral-3B
shape with random weights).
"""
from __future__ import annotations

import argparse
import json

import numpy as np

from . import binding, synth


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--batch", default="1,16,64")
    ap.add_argument("--context", type=int, default=256)
    ap.add_argument("--tokens", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--gemm-path", type=int, default=0, help="0 auto, 1 CUDA-core, 2/3 tensor-core (shield_set_gemm_path)")
    args = ap.parse_args(argv)

    import torch

    spec = synth.SHIELDSTRAL_3B
    tensors = synth.make_model(spec)
    ctx = binding.ShieldContext(1)
    try:
        ctx.set_config(spec, max_positions=4096, max_batch_tokens=32768)
        ctx.upload_model(tensors)
        ctx.set_gemm_path(args.gemm_path)
        stream = torch.cuda.ExternalStream(ctx.stream())
        rng = np.random.default_rng(20261202)
        for b in (int(x) for x in args.batch.split(",")):
            cap = args.context + args.warmup + args.tokens + 1
            seqs = [ctx.seq_create(cap) for _ in range(b)]
            try:
                prompts = [rng.integers(1000, spec.vocab, size=args.context, dtype=np.int32) for _ in range(b)]
                logits = ctx.seq_forward(seqs, prompts)
                step = lambda lg: ctx.seq_forward(seqs, [np.array([int(np.argmax(r))], np.int32) for r in lg])
                for _ in range(args.warmup):
                    logits = step(logits)
                torch.cuda.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(args.tokens):
                    logits = step(logits)
                e1.record(stream)
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1) / args.tokens
                print(json.dumps({"batch": b, "context": args.context, "gemm_path": args.gemm_path, "ms_per_step": round(ms, 3),
                                  "tokens_per_s": round(b * 1000.0 / ms, 1),
                                  "note": "includes the full 131072-row head and its logits copied to the host"}),
                      flush=True)
            finally:
                for s in seqs:
                    ctx.seq_release(s)
    finally:
        ctx.close()


if __name__ == "__main__":
    main()
