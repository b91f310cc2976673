"""The multi-rank plumbing of bench.py on CPU: two gloo ranks, as torchrun
would start them, agree on the max over ranks, the whole-job rate and the
per-rank step times."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        t = 1.0 + rank  # rank 1 is the slower one
        m = bench.allmax(t, world)
        rate = bench.whole_job_rate(16384, t, world)
        per_rank = bench.allgather(t, world)
        bench.barrier(world)
        q.put((rank, m, rate, per_rank))
    finally:
        dist.destroy_process_group()


def test_two_ranks_max_and_rate():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    for rank, m, rate, per_rank in got:
        assert m == 2.0
        assert rate == pytest.approx(2 * 16384 / 2.0)
        assert per_rank == [1.0, 2.0]
