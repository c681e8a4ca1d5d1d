"""The benchmark's multi-rank plumbing on two gloo ranks (no GPU): every rank
reaches the same collectives and rank 0 sees the max / sum over ranks."""
import os
import socket
import sys
from pathlib import Path

import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, str(REPO))
    import bench
    r, w, _ = bench.dist_setup(bench.parse_args([]))
    try:
        mx = bench.dist_max(float(rank + 1) * 10.0, w, "cpu")
        sm = bench.dist_sum(float(rank + 1), w, "cpu")
        bench.dist_barrier(w)
        q.put((r, mx, sm))
    finally:
        bench.dist_done(w)


def test_two_rank_max_and_sum():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    assert got == [(0, 20.0, 3.0), (1, 20.0, 3.0)]
