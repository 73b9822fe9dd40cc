"""The multi-rank plumbing of bench.py on CPU (gloo, world size 2): every
rank reports the slowest rank's time, and the barrier returns on all ranks.
bench.py runs one independent replica per GPU; these helpers are its only
cross-rank steps."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        bench.dist_barrier(world)
        out[rank] = bench.dist_max(1.5 + rank, world)
        bench.dist_barrier(world)
    finally:
        dist.destroy_process_group()


def test_dist_max_and_barrier_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs)
        assert dict(out) == {0: 2.5, 1: 2.5}
