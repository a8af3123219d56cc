"""KV-head tensor parallelism over NCCL on two GPUs: rank r holds KV heads
[2r, 2r + 2) of a four-head layer; rank 0 also runs the unsplit layer and
checks the gathered attention outputs (bit for bit, fp32) and every rank's
window sets after several eviction cycles.  Needs two GPUs (skipped otherwise)."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _rank(rank, world, port, q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from qevict_b200.layer_state import StickyLayerState
    from qevict_b200.tp import KVHeadShardedLayer, TorchDistExchange
    ok, msg = True, ""
    try:
        B, H, G, D, om, sink, local, kw, qw = 2, 4, 2, 64, 16, 16, 32, 3, 4
        dt = torch.float32
        cpu = torch.Generator().manual_seed(5)
        S = sink + 12 * om
        K = torch.randn(B, H, S, D, generator=cpu).to(dt).cuda()
        V = torch.randn(B, H, S, D, generator=cpu).to(dt).cuda()
        cs = (torch.rand(B, H, S, generator=cpu) * 4).cuda()
        sh = KVHeadShardedLayer(rank, world, B, H, G, D, om, sink, local, kw, qw, 128, 8, dt)
        sl = sh.kv_slice()
        sh.prefill(K[:, sl].contiguous(), V[:, sl].contiguous(), cs[:, sl].contiguous())
        full = None
        if rank == 0:
            full = StickyLayerState(B, H, G, D, om, sink, local, kw, qw, 128, 8, dt)
            full.prefill(K, V, cs)
        ex = TorchDistExchange()
        out_t = torch.empty(B, H * G, D, dtype=dt, device="cuda")
        out_f = torch.empty_like(out_t)
        for i in range(80):
            qv = (torch.randn(B, H * G, D, generator=cpu) * 0.5).to(dt).cuda()
            kn = torch.randn(B, H, D, generator=cpu).to(dt).cuda()
            vn = torch.randn(B, H, D, generator=cpu).to(dt).cuda()
            sh.step(qv, kn, vn, out_t, ex)
            if full is not None:
                full.step(qv, kn, vn, out=out_f)
                if not torch.equal(out_t, out_f):
                    ok, msg = False, f"outputs differ at step {i}"
        for b in range(B):
            ids = sh.state.view_sticky(b)[0].cuda()
            parts = [torch.empty_like(ids) for _ in range(world)]
            dist.all_gather(parts, ids)
            if full is not None and not torch.equal(torch.cat(parts).cpu(), full.view_sticky(b)[0]):
                ok, msg = False, f"sticky windows differ (b={b})"
        torch.cuda.synchronize()
    except Exception as e:  # report, then leave the group in step with the other rank
        ok, msg = False, repr(e)
    finally:
        dist.destroy_process_group()
    q.put((rank, ok, msg))


def test_kv_head_split_over_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 150
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, ok, msg in res:
        assert ok, f"rank {rank}: {msg}"
