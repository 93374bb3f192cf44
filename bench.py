#!/usr/bin/env python3
"""Benchmark of the Shieldstral scoring prefill on B200 (one JSON line on rank 0).

Metric: prefill tokens/s and verdicts/s per B200, Q4_0 3B, at
1/2/4/8 GPUs.  The reference publishes no suite, so seeded synthetic inputs
with BASELINE.json's shapes stand in: the Shieldstral-shaped 3B decoder
(26 layers, d 3072, 32/8 heads x 128, FFN 9216, vocab 131072) with N(0, 0.02)
weights quantized with gguf-py's block semantics, ids uniform over the
non-special ids.

  --config 5 (default)  Q4_0, a set of 4096 requests with lognormal lengths
                        (median 300, sigma 0.6, clipped to [32, 4096]); each
                        step every rank scores --batch requests, the ranks'
                        shares balanced by longest-processing-time on cost
                        S * (1 + S / 8192) (weak scaling, no collective on
                        the data path)
  --config 1            Q4_0, one request of 256 ids per rank per step
  --config 2            the isolated quantized-GEMM sweep: Q4_0/Q5_0/Q5_1/Q8_0
                        x {3072x3072, 1024x3072, 9216x3072, 3072x9216, and the
                        model's 4096x3072, 3072x4096} x M in {1, 64, 512, 4096};
                        the line's value is the 512-token Q4_0 projection set
  --config 3            Q5_1, 64 requests with lengths uniform in [128, 1024]
  --config 4            Q8_0, 16 requests of 4096 tokens

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and a
device synchronize; device time from CUDA events on the library's stream
(``value``: the library's events around each micro-batch, ids already on the
GPU; ``e2e``: events around the public C-ABI call with host buffers), max
over ranks.  Inputs are larger than L2 (the weights stream through every
layer), so no flush is needed between steps.

``--impl reference`` times the reference's CPU path instead: the reference is
C# and cannot run here (no dotnet), so its C restatement (oracle/) runs on the
host cores, rank 0 only.  ``--decode`` times decode steps (one token per
sequence onto a 256-token context, Benchmark.cs:399-410); ``--int8-peak``
prints the dense int8 tensor-core rate (cuBLASLt through torch._int_mm).
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
SET_SEED = 20261205
MODEL_DESC = "Shieldstral-shaped 3B (26L, d3072, 32/8x128 GQA, ffn 9216, vocab 131072, YaRN)"
SWEEP_SHAPES = [(3072, 3072), (1024, 3072), (9216, 3072), (3072, 9216), (4096, 3072), (3072, 4096)]
SWEEP_TOKENS = [1, 64, 512, 4096]
# the model's seven projections of one layer: q, k, v, o, gate, up, down
PROJECTIONS = [(4096, 3072), (1024, 3072), (1024, 3072), (3072, 4096), (9216, 3072), (9216, 3072), (3072, 9216)]


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=[1, 2, 3, 4, 5], default=5)
    ap.add_argument("--batch", type=int, default=512, help="config 5: requests per rank per step")
    ap.add_argument("--max-batch-tokens", type=int, default=32768)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--types", default="Q4_0,Q5_0,Q5_1,Q8_0", help="config 2: weight types")
    ap.add_argument("--shapes", default="", help="config 2: NxK list (default: the sweep's six)")
    ap.add_argument("--tokens", default="", help="config 2: M list (default 1,64,512,4096)")
    ap.add_argument("--gemm-path", type=int, default=0, help="shield_set_gemm_path for the run")
    ap.add_argument("--attention-rows", type=int, default=0, help="shield_set_attention_rows for the run")
    ap.add_argument("--decode", default="", help="decode mode: comma list of sequence counts")
    ap.add_argument("--int8-peak", action="store_true")
    ap.add_argument("--layers", type=int, default=0, help="model configs: first N layers only (profiling a small case)")
    ap.add_argument("--requests", type=int, default=0, help="configs 3 and 4: first N requests of the set only")
    return ap.parse_args(argv)


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    return rank, world, local, local_world


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.out = ""

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
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


def measured_peaks() -> dict:
    """The roofline denominators: MEASURED_PEAKS.json (driver-written) when
    present, else this pool's fallback figures."""
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm": d.get("hbm_gbs", 6650.0), "bf16": d.get("bf16_tflops", 1590.0),
                "bf16_sustained": d.get("bf16_tflops_sustained", 1400.0), "source": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def int8_peak(n: int = 8192, reps: int = 10, warmup: int = 3) -> float:
    """Dense int8 tensor-core rate on this GPU, TOP/s: cuBLASLt through
    torch._int_mm on n x n x n int8 operands, best of reps, 2 n^3 ops per call.
    This is the library rate the north star's int8 fraction is quoted against."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(n)
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda", generator=g)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda", generator=g).t()
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
    del a, b
    torch.cuda.empty_cache()
    return 2.0 * n ** 3 / best / 1e9


def gemm_traffic() -> dict | None:
    """DRAM traffic of the tensor-core GEMM from one ncu capture of one launch
    (profiles/k_gemm_tc_traffic.json: the capture's command, its launch, its
    dram__bytes_read.sum + dram__bytes_write.sum and that launch's algorithmic
    bytes). The bench scales it to its own launches by the ratio measured /
    algorithmic, which holds while the traffic grows with the shape."""
    p = REPO / "profiles" / "k_gemm_tc_traffic.json"
    if not p.exists():
        return None
    return json.loads(p.read_text())


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


# ------------------------------------------------------------ workloads

def model_spec(config: int, layers: int = 0):
    import dataclasses
    from llm_shield_b200 import synth
    qtype = {1: synth.Q4_0, 3: synth.Q5_1, 4: synth.Q8_0, 5: synth.Q4_0}[config]
    spec = dataclasses.replace(synth.SHIELDSTRAL_3B, qtype=qtype)
    return dataclasses.replace(spec, n_layers=layers) if layers else spec


WORKLOAD = {
    1: "config 1: Q4_0 3B, one request of 256 ids",
    3: "config 3: Q5_1 3B, 64 requests, lengths uniform in [128, 1024]",
    4: "config 4: Q8_0 3B, 16 requests of 4096 tokens",
    5: "config 5: Q4_0 3B, 4096 lognormal requests (median 300, sigma 0.6, [32,4096])",
}


def request_set(config: int, vocab: int, limit: int = 0):
    """(ids, offsets, lengths) of the config's seeded request set (configs 3
    and 4: its first `limit` requests when limit > 0)."""
    from llm_shield_b200 import synth
    if config == 5:
        lengths = synth.lognormal_lengths(4096, seed=SET_SEED)
    elif config == 3:
        lengths = np.random.default_rng(SET_SEED + 3).integers(128, 1025, size=64).astype(np.int64)
    elif config == 4:
        lengths = np.full(16, 4096, np.int64)
    else:
        lengths = np.array([256], np.int64)
    if limit and config in (3, 4):
        lengths = lengths[:limit]
    rng = np.random.default_rng(SET_SEED + config)
    ids = rng.integers(synth.FIRST_ORDINARY_ID, vocab, size=int(lengths.sum()), dtype=np.int32)
    offsets = np.zeros(lengths.size + 1, np.int64)
    np.cumsum(lengths, out=offsets[1:])
    return ids, offsets, lengths


def cost(length) -> float:
    """Relative device cost of a request of `length` tokens: linear layers in
    S plus attention in S^2 (the library's own LPT weight)."""
    return float(length) * (1.0 + float(length) / 8192.0)


def rank_requests(config: int, step: int, rank: int, world: int, batch: int, lengths: np.ndarray) -> np.ndarray:
    """Requests rank `rank` scores in step `step`. Config 5: the step's window
    of world * batch consecutive requests of the set (cycling), split across
    ranks longest-processing-time first on cost(S), so every rank gets an
    equal share of the device work; every rank computes the same split.
    Configs 1, 3, 4: the whole set on every rank (weak scaling)."""
    n = lengths.size
    if config != 5:
        return np.arange(n)
    window = (np.arange(world * batch) + step * world * batch) % n
    order = sorted(window.tolist(), key=lambda r: (-cost(lengths[r]), r))
    load = [0.0] * world
    mine = [[] for _ in range(world)]
    for r in order:
        k = min(range(world), key=lambda j: (load[j], j))
        load[k] += cost(lengths[r])
        mine[k].append(r)
    return np.array(sorted(mine[rank]), np.int64)


def pack(ids, offsets, idx):
    parts = [ids[offsets[i]:offsets[i + 1]] for i in idx]
    lens = np.array([p.size for p in parts], np.int64)
    off = np.zeros(len(parts) + 1, np.int64)
    np.cumsum(lens, out=off[1:])
    return np.ascontiguousarray(np.concatenate(parts), np.int32), off


def cpu_model_sample(config: int, spec, tensors, ids, offsets, budget_s: float = 20.0) -> dict:
    """The oracle (C restatement of the reference CPU integer path) on the
    host cores over the config's first requests until about budget_s of
    work. Config 4's 4096-token requests take minutes on the CPU, so there
    the sample is one request through the model's first 4 of 26 layers
    (the same weights), extrapolated per layer and labelled as such."""
    sys.path.insert(0, str(REPO / "tests"))
    import dataclasses
    import oracle
    from helpers import oracle_model
    threads = oracle.default_threads()
    if config == 4:
        part = dataclasses.replace(spec, n_layers=4)
        sub = {k: v for k, v in tensors.items()
               if not k.startswith("blk.") or int(k.split(".")[1]) < part.n_layers}
        om = oracle_model(part, sub)
        t0 = time.perf_counter()
        om.forward(ids[offsets[0]:offsets[1]], spec.verdict_ids, threads=threads)
        dt = (time.perf_counter() - t0) * spec.n_layers / part.n_layers
        n = int(offsets[1] - offsets[0])
        return {"value": n / dt, "unit": "tokens/s", "verdicts_per_s": 1.0 / dt, "cores": threads,
                "kind": "port", "host": host_cpu(),
                "sample": f"one 4096-token request through 4 of 26 layers ({dt * part.n_layers / spec.n_layers:.1f} s),"
                          f" extrapolated x{spec.n_layers / part.n_layers:.1f} per layer; oracle/ C restatement of"
                          f" the reference CPU integer path"}
    om = oracle_model(spec, tensors)
    t0 = time.perf_counter()
    tokens = reqs = 0
    for r in range(offsets.size - 1):
        om.forward(ids[offsets[r]:offsets[r + 1]], spec.verdict_ids, threads=threads)
        tokens += int(offsets[r + 1] - offsets[r])
        reqs += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": tokens / dt, "unit": "tokens/s", "verdicts_per_s": reqs / dt, "cores": threads,
            "kind": "port", "host": host_cpu(),
            "sample": f"first {reqs} requests of the config-{config} set ({tokens} tokens), oracle/ C restatement "
                      f"of the reference CPU integer path, {dt:.1f} s"}


# ------------------------------------------------------------ model configs

def init_dist(world: int):
    if world <= 1:
        return None
    import datetime
    import torch.distributed as dist
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    return dist


def gather_ranks(dist, values, world: int, device: str = "cuda") -> np.ndarray:
    """Every rank's row of float64 values, as a (world, len) array (one
    all_gather; rank order)."""
    import torch
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist is None:
        return t.cpu().numpy()[None, :]
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return torch.stack(out).cpu().numpy()


def model_from_gguf(spec, dist, local: int, wait_s: float = 900.0):
    """The config's model written once per node as a GGUF file (by local rank
    0, with every host core, in the temp directory; published by an atomic
    rename) and mapped back read-only by every rank, so the upload reads each
    tensor from the file's mapping as GgufFile.GetTensorPointer hands it over
    (Gguf/GgufFile.cs:195-199). The other ranks poll for the file (at most
    wait_s seconds) rather than wait in a collective with a short timeout.
    Returns (tensors, file, note)."""
    import tempfile
    from llm_shield_b200 import gguf_file, synth
    path = Path(tempfile.gettempdir()) / f"shield_bench_{spec.qtype}_{spec.n_layers}_{os.getppid()}.gguf"
    err = None
    if local == 0:
        part = path.with_suffix(".part")
        try:
            gguf_file.write_model(part, spec)
            os.replace(part, path)
        except OSError as e:
            err = str(e)
            part.unlink(missing_ok=True)
    else:
        t0 = time.monotonic()
        while not path.exists() and time.monotonic() - t0 < wait_s:
            time.sleep(0.5)
    if err is None and path.exists():
        g = gguf_file.GgufFile(path)
        return g.tensors(), g, f"mapped GGUF file {path.name} ({path.stat().st_size} bytes)"
    return synth.make_model(spec), None, f"in-memory tensors (the GGUF file is missing: {err or 'not written in time'})"


def run_model(args) -> int:
    rank, world, local, local_world = dist_env()
    import torch
    torch.cuda.set_device(local)
    dist = init_dist(world)
    from llm_shield_b200 import binding, synth

    # local rank 0 alone synthesizes the model (the others map its file)
    os.environ.setdefault("SHIELD_SYNTH_THREADS", str(len(os.sched_getaffinity(0))))
    spec = model_spec(args.config, args.layers)
    tensors, gfile, source = model_from_gguf(spec, dist, local)
    ids, offsets, lengths = request_set(args.config, spec.vocab, args.requests)

    ctx = binding.ShieldContext(1 << local)
    ctx.set_config(spec, max_positions=4096, max_batch_tokens=args.max_batch_tokens)
    t_up = time.perf_counter()
    ctx.upload_model(tensors)
    upload_s = time.perf_counter() - t_up
    upload_bytes = sum(int(t["data"].nbytes) for t in tensors.values())
    ctx.set_gemm_path(args.gemm_path)
    ctx.set_attention_rows(args.attention_rows)
    vid = np.asarray(spec.verdict_ids, np.int32)
    nyes = len(spec.yes_ids)
    stream = torch.cuda.ExternalStream(ctx.stream())
    peak8 = int8_peak()

    def one_step(s):
        sid, soff = pack(ids, offsets, rank_requests(args.config, s, rank, world, args.batch, lengths))
        ctx.score_packed(sid, soff, vid, nyes)
        return int(soff[-1]), soff.size - 1

    for s in range(args.warmup):
        one_step(s)
    ctx.read_timing(reset=True)
    ctx.set_timing(1)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    tokens = reqs = 0
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for s in range(args.warmup, args.warmup + args.steps):
            n_tok, n_req = one_step(s)
            tokens += n_tok
            reqs += n_req
        e1.record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e2e_ms = e0.elapsed_time(e1)
    tm = ctx.read_timing(reset=True)

    # one extra step with every GEMM launch and every layer's attention
    # bracketed by events: the roofline of the dominant kernels
    ctx.set_timing(2)
    one_step(args.warmup + args.steps)
    g = ctx.read_timing(reset=True)
    ctx.set_timing(0)

    per_rank = gather_ranks(dist, [tokens, reqs, tm["forward_ms"], e2e_ms, tm["kernel_launches"],
                                   tm["h2d_bytes"], tm["d2h_bytes"]], world)
    fwd_ms, e2e_max = float(per_rank[:, 2].max()), float(per_rank[:, 3].max())
    tokens_all, reqs_all = int(per_rank[:, 0].sum()), int(per_rank[:, 1].sum())
    line = model_line(args, world, spec, tokens_all, reqs_all, fwd_ms, e2e_max, per_rank, g, peak8)
    line["upload"] = {"seconds": upload_s, "bytes": upload_bytes, "gb_per_s": upload_bytes / upload_s / 1e9,
                      "what": "every GGUF tensor host->GPU, plus the derived planes built there",
                      "source": source}
    line["clocks"] = clocks.summary()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_model_sample(args.config, spec, tensors, ids, offsets)
    ctx.close()
    if dist:
        dist.barrier()  # every rank has uploaded before the file goes
        dist.destroy_process_group()
    if gfile is not None:
        path = gfile.path
        gfile.close()
        if local == 0:
            path.unlink(missing_ok=True)
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def fp32_simt_peak_tflops() -> float:
    """Nominal f32 CUDA-core rate of this GPU at its maximum SM clock: SMs x
    128 lanes x 2 flops per fused multiply-add (attention's roofline, since
    its exact order of arithmetic keeps it off the tensor cores)."""
    import torch
    p = torch.cuda.get_device_properties(torch.cuda.current_device())
    mhz = 1965.0
    try:
        out = subprocess.run(["nvidia-smi", "--query-gpu=clocks.max.sm", "--format=csv,noheader,nounits", "-i",
                              str(torch.cuda.current_device())], capture_output=True, text=True, timeout=10).stdout
        mhz = float(out.strip().splitlines()[0])
    except (OSError, ValueError, IndexError, subprocess.TimeoutExpired):
        pass
    return p.multi_processor_count * 128 * 2 * mhz * 1e6 / 1e12


def gemm_roofline(g: dict, peak8: float, sustained: bool) -> dict:
    pk = measured_peaks()
    peak = pk["bf16_sustained"] if sustained else pk["bf16"]
    achieved = g["gemm_ops"] / (g["gemm_ms"] * 1e-3) / 1e12 if g["gemm_ms"] > 0 else 0.0
    alg = g["gemm_bytes"] / max(1, g["gemm_launches"])
    tr = gemm_traffic()
    traffic = source = None
    if tr and tr.get("algorithmic_bytes"):
        ratio = tr["dram_bytes"] / tr["algorithmic_bytes"]
        traffic = ratio * alg
        source = (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch ({tr['launch']}): "
                  f"{tr['dram_bytes']:.4g} B = {ratio:.3f} x its algorithmic bytes, scaled to this line's "
                  f"mean launch; command: {tr['command']}")
    return {"bound": "tensor", "kernel": "quantized GEMM (k_gemm_tc and the few-token kernels)",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_source": f"{pk['source']} bf16_tflops{'_sustained' if sustained else ''} (the f16 MMA rate; "
                           f"of {pk['source']})",
            "frac_int8": achieved / peak8 if peak8 else None, "int8_peak_tops": peak8,
            "int8_peak_source": "torch._int_mm 8192^3 best of 10, measured in this run",
            "traffic": traffic, "traffic_source": source, "algorithmic_bytes_per_launch": alg,
            "gemm_launches_profiled": g["gemm_launches"],
            "gemm_share_of_forward": g["gemm_ms"] / g["forward_ms"] if g["forward_ms"] else None}


def model_line(args, world, spec, tokens, reqs, fwd_ms, e2e_ms, per_rank, g, peak8) -> dict:
    from llm_shield_b200 import synth
    attn_tf = g["attn_flops"] / (g["attn_ms"] * 1e-3) / 1e12 if g["attn_ms"] > 0 else 0.0
    simt = fp32_simt_peak_tflops()
    line = {
        "metric": METRIC, "value": tokens / (fwd_ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": e2e_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8+f32",
        "data": "synthetic (seeded N(0,0.02) weights quantized as gguf-py does; uniform non-special ids)",
        "verdicts_per_s": reqs / (fwd_ms * 1e-3),
        "config": {"workload": WORKLOAD[args.config] + (f", first {args.requests} requests" if args.requests else ""),
                   "model": MODEL_DESC + (f", first {spec.n_layers} layers only" if args.layers else ""),
                   "weights": synth.TYPE_NAMES[spec.qtype],
                   "per_rank_step": (f"{args.batch} requests of the set, LPT-balanced across ranks"
                                     if args.config == 5 else "the whole set"),
                   "tokens_per_step": tokens // args.steps,
                   "parallelism": f"request shards x{world}, full weight replicas, no collective",
                   "l2": "inputs larger than L2 (the weights stream through every layer)",
                   "gemm_path": args.gemm_path, "attention_rows": args.attention_rows},
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(per_rank[:, 5].sum()) // args.steps,
                "d2h_bytes_per_step": int(per_rank[:, 6].sum()) // args.steps},
        "gpu_launches": int(per_rank[:, 4].sum()),
        "roofline": gemm_roofline(g, peak8, sustained=True),
        "attention": {"achieved": attn_tf, "unit": "TFLOP/s", "peak": simt, "frac": attn_tf / simt if simt else None,
                      "peak_source": "nominal f32 CUDA-core rate at max SM clock (SMs x 128 x 2 x clock)",
                      "share_of_forward": g["attn_ms"] / g["forward_ms"] if g["forward_ms"] else None,
                      "flops": "4 * heads * head_dim per causal (query, key) pair"},
        "per_rank": [{"rank": i, "tokens": int(r[0]), "requests": int(r[1]), "forward_ms": round(float(r[2]), 2)}
                     for i, r in enumerate(per_rank)],
    }
    if args.config == 1:
        line["latency_ms_per_verdict"] = fwd_ms / max(1, reqs // world)
    return line


# ------------------------------------------------------------ config 2: GEMM sweep

def _csv(s: str, conv):
    return [conv(v) for v in s.split(",") if v.strip()]


def run_gemm_sweep(args) -> int:
    """QuantMatMul.ForwardAsync alone (Benchmark.cs:209-286): per weight type,
    shape and token count, the GEMM kernel's device time (library events
    around each launch) and the whole device call (activation quantization +
    GEMM, events around shield_qmatmul_device), L2 flushed before every call."""
    rank, world, local, _ = dist_env()
    import torch
    torch.cuda.set_device(local)
    dist = init_dist(world)
    from llm_shield_b200 import binding, synth
    types = [synth.TYPE_BY_NAME[t] for t in _csv(args.types, str)]
    shapes = [tuple(int(v) for v in s.split("x")) for s in _csv(args.shapes, str)] or SWEEP_SHAPES
    tokens = _csv(args.tokens, int) or SWEEP_TOKENS
    pk = measured_peaks()
    peak8 = int8_peak()
    ctx = binding.ShieldContext(1 << local)
    ctx.set_config(synth.small_spec())
    ctx.set_gemm_path(args.gemm_path)
    stream = torch.cuda.ExternalStream(ctx.stream())
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")  # 256 MB > L2
    name = "blk.0.ffn_gate.weight"
    sweep = []
    with ClockSampler(local) as clocks:
        for qt in types:
            for (N, K) in shapes:
                w = synth.tensor(qt, N, K, seed=SET_SEED, stream=N * 7 + K)
                ctx.upload(name, qt, N, K, w)
                gen = torch.Generator(device="cuda").manual_seed(K)
                x = torch.randn(max(tokens), K, device="cuda", generator=gen)
                y = torch.empty(max(tokens), N, device="cuda")
                for M in tokens:
                    for _ in range(args.warmup):
                        ctx.qmatmul_device(name, x.data_ptr(), M, y.data_ptr())
                    torch.cuda.synchronize()
                    ctx.read_timing(reset=True)
                    ctx.set_timing(2)
                    call_ms = 0.0
                    for _ in range(args.steps):
                        with torch.cuda.stream(stream):
                            flush.zero_()
                        e0 = torch.cuda.Event(enable_timing=True)
                        e1 = torch.cuda.Event(enable_timing=True)
                        e0.record(stream)
                        ctx.qmatmul_device(name, x.data_ptr(), M, y.data_ptr())
                        e1.record(stream)
                        e1.synchronize()
                        call_ms += e0.elapsed_time(e1)
                    t = ctx.read_timing(reset=True)
                    ctx.set_timing(0)
                    gemm_ms = t["gemm_ms"] / max(1, t["gemm_launches"])
                    call_ms /= args.steps
                    ops = 2.0 * M * N * K
                    io = N * K // 32 * synth.BLOCK_BYTES[qt] + 4 * M * K + 4 * M * N
                    sweep.append({"type": synth.TYPE_NAMES[qt], "N": N, "K": K, "M": M,
                                  "kernel": "few-token" if M <= 16 else "tensor cores",
                                  "gemm_us": round(gemm_ms * 1e3, 2), "call_us": round(call_ms * 1e3, 2),
                                  "gemm_tops": round(ops / gemm_ms / 1e9, 2),
                                  "frac_int8": round(ops / gemm_ms / 1e9 / peak8, 4),
                                  "frac_bf16": round(ops / gemm_ms / 1e9 / pk["bf16"], 4),
                                  "call_gbs": round(io / call_ms / 1e6, 1),
                                  "frac_hbm": round(io / call_ms / 1e6 / pk["hbm"], 4),
                                  "bound": "hbm" if M <= 64 else "tensor"})
                del x, y
    e2e = gemm_e2e(ctx, args) if synth.Q4_0 in types else None
    ctx.close()
    if dist:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(sweep_line(args, world, sweep, e2e, peak8, pk, clocks.summary())), flush=True)
    return 0


def projection_set(sweep, qtype_name="Q4_0", M=512):
    """(ops, device seconds) of one layer's seven projections at M tokens,
    from the sweep's kernel times."""
    by = {(e["N"], e["K"]): e for e in sweep if e["type"] == qtype_name and e["M"] == M}
    if not all(s in by for s in PROJECTIONS):
        return None
    ops = sum(2.0 * M * n * k for n, k in PROJECTIONS)
    sec = sum(by[s]["gemm_us"] * 1e-6 for s in PROJECTIONS)
    return ops, sec


def gemm_e2e(ctx, args, M: int = 512) -> dict:
    """The Q4_0 projection set at 512 tokens through shield_qmatmul with host
    buffers (host x in, host y out, copies inside the timed region)."""
    import torch
    from llm_shield_b200 import synth
    names = {}
    for i, (n, k) in enumerate(sorted(set(PROJECTIONS))):
        names[(n, k)] = f"blk.{i + 1}.attn_q.weight"
        ctx.upload(names[(n, k)], synth.Q4_0, n, k, synth.tensor(synth.Q4_0, n, k, seed=SET_SEED, stream=n * 7 + k))
    xs = {k: np.random.default_rng(k).standard_normal((M, k)).astype(np.float32) for _, k in PROJECTIONS}
    stream = torch.cuda.ExternalStream(ctx.stream())

    def one():
        for n, k in PROJECTIONS:
            ctx.qmatmul(names[(n, k)], xs[k], M, n)
    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        one()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ops = sum(2.0 * M * n * k for n, k in PROJECTIONS)
    return {"value": ops / (ms * 1e-3) / 1e12, "unit": "TOP/s",
            "h2d_bytes_per_step": sum(4 * M * k for _, k in PROJECTIONS),
            "d2h_bytes_per_step": sum(4 * M * n for n, _ in PROJECTIONS),
            "what": "one layer's seven Q4_0 projections at 512 tokens through shield_qmatmul, host f32 in and out"}


def cpu_gemm_sample(budget_s: float = 15.0, M: int = 512) -> dict:
    """The oracle's integer GEMM (IntegerGemm on the host cores) on the Q4_0
    projection set at 512 tokens, repeated until about budget_s."""
    import oracle
    from llm_shield_b200 import synth
    ws = {(n, k): synth.tensor(synth.Q4_0, n, k, seed=SET_SEED, stream=n * 7 + k) for n, k in set(PROJECTIONS)}
    xs = {k: np.random.default_rng(k).standard_normal((M, k)).astype(np.float32) for _, k in PROJECTIONS}
    threads = oracle.default_threads()
    t0 = time.perf_counter()
    sets = 0
    while True:
        for n, k in PROJECTIONS:
            oracle.qmatmul(synth.Q4_0, ws[(n, k)], n, k, xs[k], M, threads=threads)
        sets += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    ops = sets * sum(2.0 * M * n * k for n, k in PROJECTIONS)
    return {"value": ops / dt / 1e12, "unit": "TOP/s", "cores": threads, "kind": "port", "host": host_cpu(),
            "sample": f"{sets} passes over one layer's seven Q4_0 projections at 512 tokens, oracle/ C "
                      f"restatement of IntegerGemm, {dt:.1f} s"}


def sweep_line(args, world, sweep, e2e, peak8, pk, clocks) -> dict:
    ps = projection_set(sweep)
    value = ps[0] / ps[1] / 1e12 if ps else None
    line = {
        "metric": "quantized-GEMM throughput, config 2 sweep (value: one layer's seven Q4_0 projections at 512 tokens)",
        "value": value, "unit": "TOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ps[1] * 1e3 if ps else None, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8+f32", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "config": {"workload": "config 2: Q4_0/Q5_0/Q5_1/Q8_0 x 6 shapes x M in {1,64,512,4096}",
                   "l2": "flushed (256 MB written) before every timed call", "gemm_path": args.gemm_path},
        "roofline": {"bound": "tensor", "kernel": "k_gemm_tc, 512-token Q4_0 projections",
                     "achieved": value, "peak": pk["bf16"], "unit": "TFLOP/s",
                     "frac": value / pk["bf16"] if value else None,
                     "peak_source": f"{pk['source']} bf16_tflops burst (the f16 MMA rate; of {pk['source']})",
                     "frac_int8": value / peak8 if value else None, "int8_peak_tops": peak8,
                     "int8_peak_source": "torch._int_mm 8192^3 best of 10, measured in this run",
                     "traffic": None, "traffic_source": "see profiles/ for ncu captures of single launches"},
        "e2e": e2e, "gpu_launches": len(sweep) * args.steps * 2,  # quantize + GEMM per timed call
        "clocks": clocks, "sweep": sweep,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_gemm_sample()
    return line


# ------------------------------------------------------------ decode, reference arm

def run_decode(args) -> int:
    """Decode steps (Benchmark.cs:399-410): every sequence prefilled with a
    seeded 256-token prompt, then --steps greedy steps of one token per
    sequence on the full 131072-row head; one JSON line per sequence count."""
    import torch
    from llm_shield_b200 import binding, synth
    torch.cuda.set_device(dist_env()[2])
    spec = model_spec(5)
    tensors = synth.make_model(spec)
    ctx = binding.ShieldContext(1 << dist_env()[2])
    try:
        ctx.set_config(spec, max_positions=4096, max_batch_tokens=args.max_batch_tokens)
        ctx.upload_model(tensors)
        ctx.set_gemm_path(args.gemm_path)
        ctx.set_attention_rows(args.attention_rows)
        stream = torch.cuda.ExternalStream(ctx.stream())
        rng = np.random.default_rng(SET_SEED)
        for b in _csv(args.decode, int):
            seqs = [ctx.seq_create(256 + args.warmup + args.steps + 1) for _ in range(b)]
            try:
                logits = ctx.seq_forward(seqs, [rng.integers(1000, spec.vocab, size=256, dtype=np.int32)
                                                for _ in range(b)])

                def step(lg):
                    return ctx.seq_forward(seqs, [np.array([int(np.argmax(r))], np.int32) for r in lg])
                for _ in range(args.warmup):
                    logits = step(logits)
                torch.cuda.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(args.steps):
                    logits = step(logits)
                e1.record(stream)
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1) / args.steps
                print(json.dumps({"metric": "decode tokens/s (256-token context, full head to the host)",
                                  "sequences": b, "ms_per_step": round(ms, 3),
                                  "value": round(b * 1000.0 / ms, 1), "unit": "tokens/s"}), flush=True)
            finally:
                for s in seqs:
                    ctx.seq_release(s)
    finally:
        ctx.close()
    return 0


def run_reference(args) -> int:
    """The reference's CPU path (its C restatement, oracle/) on the host
    cores, rank 0 only, each step a bounded sample of the config's workload:
    one request of the set (config 4: one 4096-token request through 4 of 26
    layers, extrapolated per layer), or one pass over the Q4_0 projection set
    at 512 tokens (config 2)."""
    rank = dist_env()[0]
    if rank != 0:
        return 0
    if args.config == 2:
        times = [cpu_gemm_sample(budget_s=0.0) for _ in range(args.warmup + args.steps)][args.warmup:]
        value = statistics.mean(t["value"] for t in times)
        cpu = dict(times[-1], value=value, sample=f"{len(times)} passes over one layer's seven Q4_0 projections "
                                                   f"at 512 tokens, oracle/ C restatement of IntegerGemm")
        line = {"metric": "quantized-GEMM throughput, config 2 sweep (value: one layer's seven Q4_0 projections at 512 tokens)",
                "value": value, "unit": "TOP/s", "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "int8+f32", "data": "synthetic", "config": {"workload": "config 2 (Q4_0 projections, M=512)"},
                "cpu_baseline": cpu,
                "e2e": {"value": value, "unit": "TOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0
    from llm_shield_b200 import synth
    spec = model_spec(args.config)
    tensors = synth.make_model(spec)
    ids, offsets, lengths = request_set(args.config, spec.vocab)
    samples = []
    for s in range(args.warmup + args.steps):
        r = s % (offsets.size - 1)
        one = cpu_model_sample(args.config, spec, tensors, ids[offsets[r]:offsets[r + 1]],
                               np.array([0, offsets[r + 1] - offsets[r]], np.int64), budget_s=0.0)
        if s >= args.warmup:
            samples.append((int(offsets[r + 1] - offsets[r]) / one["value"], int(offsets[r + 1] - offsets[r]), one))
    total_t = sum(t for t, _, _ in samples)
    total_tok = sum(n for _, n, _ in samples)
    value = total_tok / total_t
    cpu = dict(samples[-1][2], value=value,
               sample=f"{len(samples)} requests ({total_tok} tokens), one per step; " + samples[-1][2]["sample"])
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total_t / len(samples),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8+f32",
            "data": "synthetic", "verdicts_per_s": len(samples) / total_t,
            "config": {"workload": WORKLOAD[args.config], "per_step": "one request of the set (bounded CPU sample)",
                       "model": MODEL_DESC},
            "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None) -> int:
    args = parse(argv)
    if args.impl == "reference":
        return run_reference(args)
    if args.int8_peak:
        import torch
        torch.cuda.set_device(dist_env()[2])
        print(json.dumps({"int8_dense": "torch._int_mm", "n": 8192, "tops": round(int8_peak(), 1),
                          "nominal_tops": 4500}), flush=True)
        return 0
    if args.decode:
        return run_decode(args)
    if args.config == 2:
        return run_gemm_sweep(args)
    return run_model(args)


if __name__ == "__main__":
    raise SystemExit(main())
