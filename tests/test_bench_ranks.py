"""Multi-rank logic of bench.py on CPU (gloo, world size 2): the timed region's
duration is the maximum over ranks, and only rank 0 runs and prints the CPU
reference arm."""

import os
import sys

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rank_main(rank, world, port, q):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    import bench
    try:
        got = bench.max_over_ranks_on(10.0 + rank * 5.0, world, "cpu")
        # a non-zero rank leaves the reference arm at once, printing nothing
        ref = None
        if rank == 1:
            class A:
                steps, gpus, warmup = 4, world, 3
            ref = bench.run_reference(A())
        q.put((rank, got, ref))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_reference_rank_gating():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 300
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][1] == res[1][1] == 15.0
    assert res[1][2] is None


def test_single_rank_is_identity():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks_on(3.5, 1, "cpu") == 3.5
