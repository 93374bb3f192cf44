"""The benchmark's multi-rank host logic on CPU: two and four gloo ranks split
every step's requests without overlap and with balanced device cost
(longest-processing-time first on S * (1 + S / 8192)), and the job's numbers
are built from every rank's row (the NCCL path does the same on GPUs)."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, out):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, str(REPO))
    import bench
    from llm_shield_b200 import synth
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        lengths = synth.lognormal_lengths(4096, seed=bench.SET_SEED)
        steps = [bench.rank_requests(5, s, rank, world, 96, lengths) for s in range(3)]
        rows = bench.gather_ranks(dist, [1000.0 * (rank + 1), 96, 10.0 + rank], world, device="cpu")
        out.put((rank, [st.tolist() for st in steps], rows.tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_split_requests_evenly_and_gather_numbers(world):
    torch = pytest.importorskip("torch")
    sys.path.insert(0, str(REPO))
    import bench
    from llm_shield_b200 import synth
    mp = torch.multiprocessing.get_context("spawn")
    q = mp.Queue()
    port = _free_port()
    procs = [mp.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict()
    for _ in procs:
        r, steps, rows = q.get(timeout=120)
        res[r] = (steps, rows)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    lengths = synth.lognormal_lengths(4096, seed=bench.SET_SEED)
    for s in range(3):
        parts = [set(res[r][0][s]) for r in range(world)]
        union = set().union(*parts)
        assert sum(len(p) for p in parts) == len(union) == world * 96  # disjoint, the whole window
        window = set(((np.arange(world * 96) + s * world * 96) % 4096).tolist())
        assert union == window
        loads = [sum(bench.cost(lengths[i]) for i in p) for p in parts]
        assert max(loads) / (sum(loads) / world) < 1.01  # within 1% of an even split
    for r in range(world):
        rows = np.array(res[r][1])
        assert rows.shape == (world, 3)
        np.testing.assert_array_equal(rows[:, 0], 1000.0 * (np.arange(world) + 1))
        assert rows[:, 2].max() == 10.0 + world - 1


def _gguf_rank(local: int, out):
    sys.path.insert(0, str(REPO))
    import bench
    from llm_shield_b200 import synth
    spec = synth.small_spec(qtype=synth.Q4_0, n_layers=2, seed=17)
    tensors, gfile, note = bench.model_from_gguf(spec, None, local, wait_s=120)
    digest = {k: (t["type"], t["rows"], t["cols"], int(np.asarray(t["data"], np.uint64).sum())) for k, t in tensors.items()}
    out.put((local, gfile is not None, note, digest))


def test_model_file_written_once_and_mapped_by_every_rank():
    """bench.py's per-node hand-off: local rank 0 writes the GGUF file
    (published by a rename), a rank that starts earlier waits for it, and
    both upload from a mapping of the same bytes."""
    torch = pytest.importorskip("torch")
    from llm_shield_b200 import synth
    mp = torch.multiprocessing.get_context("spawn")
    q = mp.Queue()
    procs = [mp.Process(target=_gguf_rank, args=(r, q)) for r in (1, 0)]  # the reader first
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, mapped, note, digest = q.get(timeout=300)
        res[r] = (mapped, note, digest)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    spec = synth.small_spec(qtype=synth.Q4_0, n_layers=2, seed=17)
    want = {k: (t["type"], t["rows"], t["cols"], int(np.asarray(t["data"], np.uint64).sum()))
            for k, t in synth.make_model(spec).items()}
    for r in (0, 1):
        assert res[r][0], res[r][1]
        assert res[r][2] == want
    import os
    import tempfile
    leftover = Path(tempfile.gettempdir()) / f"shield_bench_{spec.qtype}_{spec.n_layers}_{os.getpid()}.gguf"
    leftover.unlink(missing_ok=True)
