"""KV-head tensor parallelism: a layer split over ranks must behave exactly like
the unsplit layer.

* GPU, one device: two shards of two KV heads each (collectives done in-process,
  LocalExchange) against one four-head StickyLayerState driven with the same
  prompt and tokens through several eviction cycles: identical attention
  outputs (fp32: bit for bit; bf16: within the decode tolerance), identical
  sticky and Q-cache window sets.
* CPU, gloo, world size 2: the collectives of TorchDistExchange (head order of
  the all-gather, MIN of the loser counts).
"""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _run_split_vs_full(dtype, D, om, sink, local, kw, qw, steps, seed=1):
    from qevict_b200.layer_state import StickyLayerState
    from qevict_b200.tp import KVHeadShardedLayer, step_local
    B, H, G = 2, 4, 2
    g = torch.Generator(device="cuda").manual_seed(seed)
    S = sink + 12 * om
    K = torch.randn(B, H, S, D, generator=g, device="cuda").to(dtype)
    V = torch.randn(B, H, S, D, generator=g, device="cuda").to(dtype)
    cs = torch.rand(B, H, S, generator=g, device="cuda") * 4
    full = StickyLayerState(B, H, G, D, om, sink, local, kw, qw, 128, 8, dtype)
    full.prefill(K, V, cs)
    shards = [KVHeadShardedLayer(r, 2, B, H, G, D, om, sink, local, kw, qw, 128, 8, dtype) for r in range(2)]
    for sh in shards:
        sl = sh.kv_slice()
        sh.prefill(K[:, sl].contiguous(), V[:, sl].contiguous(), cs[:, sl].contiguous())
    out_f = torch.empty(B, H * G, D, dtype=dtype, device="cuda")
    out_t = torch.empty_like(out_f)
    cycles = 0
    for i in range(steps):
        q = (torch.randn(B, H * G, D, generator=g, device="cuda") * 0.5).to(dtype)
        kn = torch.randn(B, H, D, generator=g, device="cuda").to(dtype)
        vn = torch.randn(B, H, D, generator=g, device="cuda").to(dtype)
        # spikes on a few steps make windows change tier
        if i % 17 == 3:
            kn = kn * 4
        cyc = full.n_tokens + 1 > full.prompt_len and (full.n_tokens + 1 - full.prompt_len) % om == 0
        full.step(q, kn, vn, out=out_f)
        step_local(shards, q, kn, vn, out_t)
        cycles += cyc
        yield i, out_f, out_t
        if cyc:
            for b in range(B):
                ids_f, _ = full.view_sticky(b)
                ids_t = torch.cat([sh.state.view_sticky(b)[0] for sh in shards], dim=0)
                assert torch.equal(ids_f, ids_t), f"step {i} b {b}: sticky windows differ"
                qf = full.view_q(b)
                qt = [sh.state.view_q(b) for sh in shards]
                if qf is None:
                    assert all(x is None for x in qt)
                else:
                    assert torch.equal(qf["ids"], torch.cat([x["ids"] for x in qt], 0)), f"step {i}: Q windows differ"
                    assert torch.equal(qf["kq"], torch.cat([x["kq"] for x in qt], 0))
    assert cycles >= 3
    assert full.read_error() == 0 and all(sh.state.read_error() == 0 for sh in shards)


@pytest.mark.gpu
def test_split_layer_fp32_bit_exact():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    for _, of, ot in _run_split_vs_full(torch.float32, 64, 16, 16, 32, 3, 4, 80):
        assert torch.equal(of, ot)


@pytest.mark.gpu
def test_split_layer_bf16_tensor_core_path():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    for i, of, ot in _run_split_vs_full(torch.bfloat16, 128, 64, 64, 128, 3, 4, 200):
        err = (of.float() - ot.float()).abs()
        assert bool((err <= 2e-3 + 1e-2 * of.float().abs()).all()), f"step {i}"


# ----------------------------------------------------------------------------- CPU
def _gloo_rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from qevict_b200.tp import TorchDistExchange
    try:
        ex = TorchDistExchange()
        local = torch.full((2, 3, 4), float(rank))
        local[:, :, 0] = torch.arange(3, dtype=torch.float32) + 10 * rank
        out = torch.empty(2, 3 * world, 4)
        ex.gather_heads(local, out)
        counts = torch.tensor([5 + rank, 7 - 3 * rank], dtype=torch.int32)
        ex.min_(counts)
        q.put((rank, out.numpy().copy(), counts.numpy().copy()))
    finally:
        dist.destroy_process_group()


def test_exchange_collectives_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29900 + os.getpid() % 90
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=120) for _ in procs), key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, out, counts in res:
        # heads of rank 0 first, then rank 1
        np.testing.assert_array_equal(out[:, :3, 0], np.tile(np.arange(3), (2, 1)))
        np.testing.assert_array_equal(out[:, 3:, 0], np.tile(np.arange(3) + 10, (2, 1)))
        np.testing.assert_array_equal(out[:, 3:, 1], np.ones((2, 3)))
        np.testing.assert_array_equal(counts, [5, 4])
