"""The one-shot NVLink sum and maximum of the KV-head-parallel decode
(qv_peer_sum_bf16, qv_peer_max_i64), on two and on eight GPUs (each skipped
with fewer), and its bounded wait when a rank never arrives.

Each rank sums seeded bf16 vectors of every rank; the result must equal, bit
for bit, the fp32 sum in rank order rounded once to bf16 (computed by each
rank from the regenerated inputs), on every rank: eagerly for several sizes
and rounds in a row, and replayed from a CUDA graph that holds three sums
(the epoch counter on the device advances with every replay); int64 maxima
equal torch's.  The error word stays 0.  When one rank skips a call, the
other's wait gives up after about 5 s, raises QV_DERR_TIMEOUT and returns: the
process and its GPU stay usable.  NVLS is off; the kernel uses plain peer
stores.
"""

import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _vec(rnd, rank, n):
    g = torch.Generator().manual_seed(7919 * rnd + 104729 * rank + n)
    return (torch.randn(n, generator=g) * 3).to(torch.bfloat16)


def _keys(rnd, rank, n):
    g = torch.Generator().manual_seed(31337 * rnd + 7 * rank + n)
    return torch.randint(-2 ** 62, 2 ** 62, (n,), generator=g, dtype=torch.int64)


def _ref(rnd, world, n):
    acc = torch.zeros(n, dtype=torch.float32)
    for r in range(world):
        acc += _vec(rnd, r, n).float()
    return acc.to(torch.bfloat16)


def _rank(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok, msg = True, ""
    ps = None
    try:
        from qevict_b200.peer_sum import PeerSum
        ps = PeerSum(rank, world, max_bytes=64 * 1024)
        rnd = 0
        for n in (4096, 8, 32768, 4096 * 3):
            for _ in range(3):
                t = _vec(rnd, rank, n).cuda()
                ps.sum_(t)
                if not torch.equal(t.cpu(), _ref(rnd, world, n)):
                    raise AssertionError(f"eager sum differs (n={n}, round {rnd})")
                rnd += 1
        # the int64 maximum (the greedy token's packed key), eagerly
        for n in (1, 8, 100):
            for _ in range(2):
                k = _keys(rnd, rank, n).cuda()
                ps.max_(k)
                want = torch.stack([_keys(rnd, r, n) for r in range(world)]).max(dim=0).values
                if not torch.equal(k.cpu(), want):
                    raise AssertionError(f"max differs (n={n}, round {rnd})")
                rnd += 1
        # three sums in one graph, replayed twice with new inputs
        n = 4096
        bufs = [torch.empty(n, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
        for b, r0 in zip(bufs, range(3)):
            b.copy_(_vec(100 + r0, rank, n))
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for b in bufs:
                ps.sum_(b)
        torch.cuda.current_stream().wait_stream(side)
        for b, r0 in zip(bufs, range(3)):
            if not torch.equal(b.cpu(), _ref(100 + r0, world, n)):
                raise AssertionError("warm-up sum differs")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for b in bufs:
                ps.sum_(b)
        for rep in range(2):
            base = 200 + 10 * rep
            for i, b in enumerate(bufs):
                b.copy_(_vec(base + i, rank, n))
            graph.replay()
            torch.cuda.synchronize()
            for i, b in enumerate(bufs):
                if not torch.equal(b.cpu(), _ref(base + i, world, n)):
                    raise AssertionError(f"graph replay {rep} sum {i} differs")
        del graph
        if ps.read_error() != 0:
            raise AssertionError("error word set")
    except Exception as e:  # reported to the parent
        ok, msg = False, repr(e)
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        if ps is not None:
            ps.close()
        dist.destroy_process_group()
    q.put((rank, ok, msg))


@pytest.mark.parametrize("world", [2, 8])
def test_peer_sum(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29400 + os.getpid() % 150 + world
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in procs])
    for p in procs:
        p.join(timeout=120)
    for rank, ok, msg in res:
        assert ok, f"rank {rank}: {msg}"


def _rank_timeout(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=90),
                            device_id=torch.device("cuda", rank))
    ok, msg = True, ""
    ps = None
    try:
        from qevict_b200._native import QV_DERR_TIMEOUT
        from qevict_b200.peer_sum import PeerSum
        ps = PeerSum(rank, world, max_bytes=64 * 1024)
        t = _vec(0, rank, 4096).cuda()
        ps.sum_(t)                            # both ranks: a normal call
        if not torch.equal(t.cpu(), _ref(0, world, 4096)):
            raise AssertionError("sum before the missed call differs")
        if rank == 0:
            ps.sum_(t)                        # rank 1 never makes this call
            err = ps.read_error()
            if not err & QV_DERR_TIMEOUT:
                raise AssertionError(f"error word {err}: the wait did not give up")
            x = torch.ones(1024, device="cuda") * 2
            if float(x.sum()) != 2048.0:      # the context is still usable
                raise AssertionError("GPU not usable after the timeout")
        elif ps.read_error() != 0:
            raise AssertionError("error word set on the rank that skipped")
    except Exception as e:  # reported to the parent
        ok, msg = False, repr(e)
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        if ps is not None:
            ps.close()
        dist.destroy_process_group()
    q.put((rank, ok, msg))


def test_peer_sum_missing_rank_times_out():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29380 + os.getpid() % 150
    procs = [ctx.Process(target=_rank_timeout, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in procs])
    for p in procs:
        p.join(timeout=120)
    for rank, ok, msg in res:
        assert ok, f"rank {rank}: {msg}"
