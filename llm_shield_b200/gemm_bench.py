"""Micro-benchmark of the quantized GEMM entry point on one GPU.

    python -m llm_shield_b200.gemm_bench --type Q4_0 --tokens 16384 --rows 9216 --cols 3072

Uploads one synthetic weight as a layer tensor (so the tensor-core path and its
pre-unpacked copy apply), then times `shield_qmatmul_device` on device-resident
f32 activations: the whole call (activation quantization + GEMM) with CUDA
events on the library's stream, and the GEMM launches alone with the library's
level-2 timing. Prints one JSON line per GEMM path.

    python -m llm_shield_b200.gemm_bench --int8-peak

instead measures the dense int8 tensor-core rate the roofline compares
against: cuBLASLt through `torch._int_mm` on square int8 operands, best of
`--reps` per size, 2·n^3 ops per call.
"""
from __future__ import annotations

import argparse
import json

from . import binding, synth

PATHS = {"auto": 0, "simt": 1, "raw": 2, "pre": 3}


def int8_peak(sizes=(8192, 16384), reps: int = 10, warmup: int = 3) -> None:
    import torch

    for n in sizes:
        g = torch.Generator(device="cuda").manual_seed(n)
        a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda", generator=g)
        b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda", generator=g).t()  # column-major
        for _ in range(warmup):
            torch._int_mm(a, b)
        best = float("inf")
        for _ in range(reps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        print(json.dumps({"int8_dense": "torch._int_mm", "n": n, "best_ms": round(best, 4),
                          "tops": round(2.0 * n ** 3 / best / 1e9, 1), "nominal_tops": 4500}), flush=True)
        del a, b


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--type", default="Q4_0", choices=[synth.TYPE_NAMES[t] for t in synth.BLOCK_BYTES])
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--rows", type=int, default=3072)
    ap.add_argument("--cols", type=int, default=3072)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--paths", default="pre", help="comma list of auto, simt, raw, pre")
    ap.add_argument("--int8-peak", action="store_true", help="measure the dense int8 rate instead")
    args = ap.parse_args(argv)
    if args.int8_peak:
        int8_peak(reps=args.reps, warmup=args.warmup)
        return

    import torch

    qtype = {v: k for k, v in synth.TYPE_NAMES.items()}[args.type]
    M, N, K = args.tokens, args.rows, args.cols
    ctx = binding.ShieldContext(1)
    try:
        ctx.set_config(synth.small_spec())
        name = "blk.0.attn_q.weight"
        ctx.upload(name, qtype, N, K, synth.tensor(qtype, N, K, seed=1, stream=2))
        x = torch.randn(M, K, device="cuda")
        y = torch.empty(M, N, device="cuda")
        stream = torch.cuda.ExternalStream(ctx.stream())
        ctx.set_timing(2)
        for path in args.paths.split(","):
            ctx.set_gemm_path(PATHS[path])
            for _ in range(args.warmup):
                ctx.qmatmul_device(name, x.data_ptr(), M, y.data_ptr())
            torch.cuda.synchronize()
            ctx.read_timing(reset=True)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.reps):
                ctx.qmatmul_device(name, x.data_ptr(), M, y.data_ptr())
            e1.record(stream)
            torch.cuda.synchronize()
            t = ctx.read_timing(reset=True)
            call_ms = e0.elapsed_time(e1) / args.reps
            gemm_ms = t["gemm_ms"] / max(1, t["gemm_launches"])
            print(json.dumps({"path": path, "type": args.type, "M": M, "N": N, "K": K,
                              "call_ms": round(call_ms, 4), "gemm_ms": round(gemm_ms, 4),
                              "gemm_tops": round(2 * M * N * K / gemm_ms / 1e9, 1)}), flush=True)
    finally:
        ctx.close()


if __name__ == "__main__":
    main()
