#!/usr/bin/env python3
"""Benchmark of the Shieldstral scoring prefill on B200 (one JSON line on rank 0).

Metric: prefill tokens/s and verdicts/s per B200, Q4_0 3B, at
1/2/4/8 GPUs.  Workload: config 5 — the Shieldstral-shaped 3B decoder with
Q4_0 weights (seeded synthetic N(0, 0.02), gguf-py block semantics) and 4096
independent requests with lognormal lengths (median 300, sigma 0.6, clipped to
[32, 4096]), ids uniform over non-special ids.  Requests are independent, so
ranks shard them with no collective on the data path: each step every rank
scores its own --batch requests of that set (weak scaling).

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and a
device synchronize; device time from CUDA events (the library's events on its
own stream for ``value``; events on that stream around the public C-ABI call
for ``e2e``), max over ranks.  The weights (1.8 GiB) and each micro-batch's
activations are far larger than L2, so no flush is needed between steps.

``--impl reference`` times the reference's CPU path instead: the reference is
C# and cannot run here (no dotnet), so its C restatement (oracle/) runs on the
host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "prefill tokens/s and verdicts/s per B200 (Q4_0 3B) at 1/2/4/8 GPUs"
N_REQUESTS = 4096
SET_SEED = 20261205


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=512, help="requests per rank per step")
    ap.add_argument("--max-batch-tokens", type=int, default=32768)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    return rank, world, local, local_world


def request_set(spec):
    from llm_shield_b200 import synth
    lengths = synth.lognormal_lengths(N_REQUESTS, seed=SET_SEED)
    rng = np.random.default_rng(SET_SEED + 1)
    ids = rng.integers(synth.FIRST_ORDINARY_ID, spec.vocab, size=int(lengths.sum()), dtype=np.int32)
    offsets = np.zeros(N_REQUESTS + 1, np.int64)
    np.cumsum(lengths, out=offsets[1:])
    return ids, offsets, lengths


def step_slice(step, rank, world, batch):
    """Requests of one rank's step: a contiguous run of the set, cycling."""
    start = ((step * world + rank) * batch) % N_REQUESTS
    idx = (np.arange(batch) + start) % N_REQUESTS
    return idx


def combine_ranks(dist, fwd_ms, e2e_ms, tokens, reqs, launches, device):
    """The whole job's numbers: the slowest rank's device times (max), the
    ranks' tokens, requests and kernel launches summed. dist None: one rank."""
    if dist is None:
        return fwd_ms, e2e_ms, tokens, reqs, launches
    import torch
    t = torch.tensor([fwd_ms, e2e_ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    c = torch.tensor([tokens, reqs, launches], dtype=torch.float64, device=device)
    dist.all_reduce(c, op=dist.ReduceOp.SUM)
    return float(t[0]), float(t[1]), int(c[0]), int(c[1]), int(c[2])


def pack(ids, offsets, idx):
    parts = [ids[offsets[i]:offsets[i + 1]] for i in idx]
    lens = np.array([p.size for p in parts], np.int64)
    off = np.zeros(len(parts) + 1, np.int64)
    np.cumsum(lens, out=off[1:])
    return np.ascontiguousarray(np.concatenate(parts), np.int32), off


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc:
            self.proc.terminate()
            try:
                self.out = self.proc.communicate(timeout=5)[0]
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = self.proc.communicate()[0]

    def summary(self):
        rows = [r.split(", ") for r in (self.out or "").strip().splitlines() if r.count(",") >= 7]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in rows for j in range(4) if r[4 + j].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def gemm_traffic():
    """DRAM bytes per GEMM launch (read + write), averaged over the GEMM
    launches of one ncu capture of this command (profiles/)."""
    p = REPO / "profiles" / "k_gemm_tc_traffic.json"
    if not p.exists():
        return None
    return json.loads(p.read_text()).get("dram_bytes_per_launch")


def host_cpu() -> dict:
    """The host the CPU numbers ran on: model name, logical cores, the SIMD
    flags the reference's integer GEMM chooses between (IntegerGemm.cs:58-65)
    and the tier the oracle picked from them."""
    import oracle
    model, flags = "unknown", set()
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name") and model == "unknown":
                    model = line.split(":", 1)[1].strip()
                elif line.startswith("flags") and not flags:
                    flags = set(line.split(":", 1)[1].split())
    except OSError:
        pass
    tier = {3: "AVX-VNNI", 2: "AVX512-VNNI", 1: "AVX2", 0: "scalar"}.get(oracle.lib().orc_simd_level(), "unknown")
    return {"model": model, "nproc": os.cpu_count(),
            "isa": sorted(flags & {"avx2", "fma", "avx_vnni", "avx512f", "avx512_vnni"}),
            "oracle_gemm_tier": tier}


def cpu_baseline(spec, tensors, ids, offsets, budget_s: float = 20.0):
    """The oracle (C restatement of the reference CPU path) on the host cores,
    on the first requests of the same set, until about budget_s of work."""
    sys.path.insert(0, str(REPO / "tests"))
    import oracle
    from helpers import oracle_model
    om = oracle_model(spec, tensors)
    threads = oracle.default_threads()
    t0 = time.perf_counter()
    tokens = reqs = 0
    for r in range(N_REQUESTS):
        om.forward(ids[offsets[r]:offsets[r + 1]], spec.verdict_ids, threads=threads)
        tokens += int(offsets[r + 1] - offsets[r])
        reqs += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": tokens / dt, "unit": "tokens/s", "verdicts_per_s": reqs / dt, "cores": threads,
            "kind": "port", "sample": f"first {reqs} requests of the config-5 set ({tokens} tokens), "
                                     f"oracle/ C restatement of the reference CPU integer path, {dt:.1f} s",
            "host": host_cpu()}


def run_reference(args):
    rank, world, local, _ = dist_env()
    if rank != 0:
        return 0
    from llm_shield_b200 import synth
    spec = synth.SHIELDSTRAL_3B
    tensors = synth.make_model(spec)
    ids, offsets, lengths = request_set(spec)
    sys.path.insert(0, str(REPO / "tests"))
    import oracle
    from helpers import oracle_model
    om = oracle_model(spec, tensors)
    threads = oracle.default_threads()
    # each step: a bounded sample (one request of the set, cycling) so K+W steps end in minutes
    times, toks = [], []
    for s in range(args.warmup + args.steps):
        r = s % N_REQUESTS
        n = int(offsets[r + 1] - offsets[r])
        t0 = time.perf_counter()
        om.forward(ids[offsets[r]:offsets[r + 1]], spec.verdict_ids, threads=threads)
        dt = time.perf_counter() - t0
        if s >= args.warmup:
            times.append(dt)
            toks.append(n)
    total_t, total_tok = sum(times), sum(toks)
    value = total_tok / total_t
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total_t / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8+f32",
        "data": "synthetic", "verdicts_per_s": len(times) / total_t,
        "config": {"workload": "config 5: Q4_0 3B, lognormal requests (median 300, sigma 0.6, [32,4096])",
                   "per_step": "one request of the set per step (bounded CPU sample)",
                   "model": "Shieldstral-shaped 3B (26L, d3072, 32/8x128, ffn 9216, vocab 131072)"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{len(times)} requests ({total_tok} tokens), C restatement of the "
                                   f"reference's C# integer path (dotnet absent)", "host": host_cpu()},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    rank, world, local, local_world = dist_env()
    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    from llm_shield_b200 import binding, synth

    cores = len(os.sched_getaffinity(0))
    os.environ.setdefault("SHIELD_SYNTH_THREADS", str(max(1, cores // max(1, local_world))))
    spec = synth.SHIELDSTRAL_3B
    tensors = synth.make_model(spec)
    ids, offsets, lengths = request_set(spec)

    ctx = binding.ShieldContext(1 << local)
    ctx.set_config(spec, max_positions=4096, max_batch_tokens=args.max_batch_tokens)
    t_up = time.perf_counter()
    ctx.upload_model(tensors)
    upload_s = time.perf_counter() - t_up
    upload_bytes = sum(int(t["data"].nbytes) for t in tensors.values())
    vid = np.asarray(spec.verdict_ids, np.int32)
    nyes = len(spec.yes_ids)
    stream = torch.cuda.ExternalStream(ctx.stream())

    def one_step(s):
        sid, soff = pack(ids, offsets, step_slice(s, rank, world, args.batch))
        ctx.score_packed(sid, soff, vid, nyes)
        return int(soff[-1])

    for s in range(args.warmup):
        one_step(s)
    ctx.read_timing(reset=True)
    ctx.set_timing(1)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    tokens = 0
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for s in range(args.warmup, args.warmup + args.steps):
            tokens += one_step(s)
        e1.record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e2e_ms = e0.elapsed_time(e1)
    tm = ctx.read_timing(reset=True)
    fwd_ms = tm["forward_ms"]
    reqs = args.steps * args.batch

    # roofline of the dominant kernel (the quantized GEMM): one extra step with
    # every GEMM launch bracketed by events
    ctx.set_timing(2)
    one_step(args.warmup + args.steps)
    g = ctx.read_timing(reset=True)
    ctx.set_timing(0)

    fwd_ms, e2e_ms, tokens, reqs, launches = combine_ranks(dist, fwd_ms, e2e_ms, tokens, reqs,
                                                           tm["kernel_launches"], "cuda")

    hbm, bf16, src = measured_peaks()
    achieved = g["gemm_ops"] / (g["gemm_ms"] * 1e-3) / 1e12 if g["gemm_ms"] > 0 else 0.0
    line = {
        "metric": METRIC,
        "value": tokens / (fwd_ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": e2e_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8+f32",
        "data": "synthetic",
        "verdicts_per_s": reqs / (fwd_ms * 1e-3),
        "config": {
            "workload": "config 5: Q4_0 3B, 4096 lognormal requests (median 300, sigma 0.6, [32,4096])",
            "model": "Shieldstral-shaped 3B (26L, d3072, 32/8x128 GQA, ffn 9216, vocab 131072, YaRN)",
            "per_rank_step": f"{args.batch} requests of the set", "tokens_per_step": tokens // args.steps,
            "parallelism": f"request shards x{world}, full weight replicas, no collective",
            "l2": "inputs larger than L2 (1.8 GiB weights streamed per layer)",
        },
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": tm["h2d_bytes"] // args.steps,
                "d2h_bytes_per_step": tm["d2h_bytes"] // args.steps},
        "gpu_launches": launches,
        "roofline": {"bound": "tensor", "kernel": "quantized GEMM (all projections)",
                     "achieved": achieved, "peak": bf16, "unit": "TFLOP/s",
                     "frac": achieved / bf16, "peak_source": f"{src} bf16_tflops (the f16 MMA rate)",
                     "traffic": gemm_traffic(),
                     "algorithmic_bytes_per_launch": g["gemm_bytes"] / max(1, g["gemm_launches"]),
                     "gemm_launches_profiled": g["gemm_launches"],
                     "gemm_share_of_forward": g["gemm_ms"] / g["forward_ms"] if g["forward_ms"] else None},
    }
    line["upload"] = {"seconds": upload_s, "bytes": upload_bytes, "gb_per_s": upload_bytes / upload_s / 1e9,
                      "what": "every GGUF tensor host->GPU, plus the scale planes and f16 layer copies built there"}
    line["clocks"] = clocks.summary()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(spec, tensors, ids, offsets)
    ctx.close()
    if dist:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
