"""The multi-rank plumbing of bench.py on CPU (gloo, world size 2): every
rank reports the slowest rank's time, the barrier returns on all ranks, and
the expert-parallel workload's communicator id reaches every rank with the
shard each rank then owns, and the batched-decode parity check's gather of
per-row digests reaches every rank.  The replica workloads have no other
cross-rank step; the expert-parallel exchange itself runs on GPUs
(tests/test_ep_gpu.py)."""
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
        sys.path.insert(0, os.path.join(ROOT, "qwen-mobile-agent_b200"))
        import qma_cuda as Q
        uid = bytes(range(128)) if rank == 0 else None
        got = bench.ep_share_uid(world)(uid)
        out[("uid", rank)] = got == bytes(range(128))
        out[("shard", rank)] = Q.ep_shard(rank, world)
        # the batched-decode parity check: per-row digests of every rank, in
        # rank order, and the AND of the ranks' verdicts
        import numpy as np
        rows = np.arange(6, dtype=np.float32).reshape(2, 3) + 10 * rank
        got = bench.dist_gather_i64(bench.logits_digest(rows), world)
        want = [bench.logits_digest(np.arange(6, dtype=np.float32).reshape(2, 3) + 10 * r) for r in range(world)]
        out[("gather", rank)] = all(np.array_equal(g, w) for g, w in zip(got, want))
        out[("min", rank)] = bench.dist_min(1.0 if rank == 0 else 0.0, world)
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
        assert dict(out) == {0: 2.5, 1: 2.5, ("uid", 0): True, ("uid", 1): True,
                             ("shard", 0): (0, 128), ("shard", 1): (128, 128),
                             ("gather", 0): True, ("gather", 1): True, ("min", 0): 0.0, ("min", 1): 0.0}


def test_logits_digest_tells_rows_apart_by_their_bits():
    """The parity check compares logits rows through 8-byte digests of their
    exact bytes: equal rows give equal digests, a one-ulp change or -0.0
    against +0.0 does not."""
    import numpy as np
    sys.path.insert(0, ROOT)
    import bench
    a = np.linspace(-3, 3, 64, dtype=np.float32).reshape(4, 16)
    b = a.copy()
    b[2, 5] = np.nextafter(b[2, 5], np.float32(np.inf))
    c = a.copy()
    c[1, 0] = -0.0 if c[1, 0] == 0 else c[1, 0]
    da, db = bench.logits_digest(a), bench.logits_digest(b)
    assert da.dtype == np.int64 and da.shape == (4,)
    assert np.array_equal(da, bench.logits_digest(a.copy()))
    assert (da != db).tolist() == [False, False, True, False]
    z = np.zeros((2, 8), np.float32)
    z[1, 3] = -0.0
    dz = bench.logits_digest(z)
    assert dz[0] != dz[1]
