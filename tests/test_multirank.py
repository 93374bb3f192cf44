"""The benchmark's multi-rank host logic on CPU: two gloo ranks split every
step's requests without overlap, and the job's numbers are the slowest rank's
times and the summed counts (the NCCL path does the same on GPUs)."""
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
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        steps = [bench.step_slice(s, rank, world, 96) for s in range(3)]
        got = bench.combine_ranks(dist, 10.0 + rank, 20.0 - rank, 1000 * (rank + 1), 96, 7 + rank, "cpu")
        out.put((rank, [st.tolist() for st in steps], got))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_split_requests_and_combine_numbers():
    torch = pytest.importorskip("torch")
    mp = torch.multiprocessing.get_context("spawn")
    q = mp.Queue()
    port = _free_port()
    procs = [mp.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict()
    for _ in procs:
        r, steps, got = q.get(timeout=120)
        res[r] = (steps, got)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for s in range(3):
        a, b = set(res[0][0][s]), set(res[1][0][s])
        assert not a & b and len(a) == len(b) == 96
    for r in range(2):
        fwd, e2e, tokens, reqs, launches = res[r][1]
        assert (fwd, e2e) == (11.0, 20.0)  # max over ranks
        assert (tokens, reqs, launches) == (3000, 192, 15)  # sums
