"""The KV-head-parallel decoder (qevict_b200.tp_model).

* one GPU: the one-rank decoder's CUDA-graph decode matches its eager decode
  token for token (the cycle through qv_evict_cycle_count / _ext, the
  vocabulary-parallel greedy token, the graph-captured step);
* two GPUs (NCCL, skipped with fewer): both ranks produce the same tokens, the
  first tokens equal the one-rank decoder's on the same global weights, and
  every rank's window sets are those of the one-rank decoder's heads after
  the prompt (layer 0, whose inputs are the shared embeddings).
"""

import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPE = dict(vocab=1024, hidden=512, layers=2, heads=8, kv_heads=2, head_dim=64, ffn=1024)
STICKY = dict(omega=16, sink=16, local=32, k_windows=3, q_windows=4, bits=8)
PROMPT = 16 + 12 * 16


def _model(rank, world, seed=5):
    from qevict_b200.model import LlamaShape, StickyShape
    from qevict_b200.tp_model import TpStickyLlamaDecoder
    return TpStickyLlamaDecoder(LlamaShape(**SHAPE), StickyShape(**STICKY), rank, world, batch=1, max_pos=1024,
                                seed=seed, std=0.05)


def _ids():
    return torch.randint(0, SHAPE["vocab"], (1, PROMPT), generator=torch.Generator().manual_seed(3)).cuda()


def test_tp_decoder_one_rank_graph_matches_eager():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    toks = []
    for mode in ("eager", "graph"):
        m = _model(0, 1)
        m.prefill(_ids())
        seq = []
        if mode == "graph":
            m.capture()
        for _ in range(3 * 16 + 5):
            if mode == "eager":
                m.step_eager()
            else:
                m.step_graph()
            seq.append(int(m.tok[0]))
        toks.append(seq)
        assert all(st.read_error() == 0 for st in m.states)
        m.graphs.clear()
    assert toks[0] == toks[1]


def _rank(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok, msg, toks, ref = True, "", [], []
    try:
        m = _model(rank, world)
        m.prefill(_ids())
        toks.append(int(m.tok[0]))
        for _ in range(2 * 16 + 3):
            m.step_eager()
            toks.append(int(m.tok[0]))
        ids_tp = [m.states[0].view_sticky(0)[0]]
        if m.ps is not None:
            assert m.ps.read_error() == 0
        m.close()
        if rank == 0:
            one = _model(0, 1)
            one.prefill(_ids())
            ref.append(int(one.tok[0]))
            for _ in range(3):
                one.step_eager()
                ref.append(int(one.tok[0]))
            # layer 0's window sets of this rank's heads, after the prompt
            sl = slice(rank * m.hl, (rank + 1) * m.hl)
            full0 = _model(0, 1)
            full0.prefill(_ids())
            if not torch.equal(full0.states[0].view_sticky(0)[0][sl], ids_tp[0]):
                ok, msg = False, "layer-0 window sets differ from the one-rank decoder's"
        torch.cuda.synchronize()
    except Exception as e:
        ok, msg = False, repr(e)
    finally:
        dist.destroy_process_group()
    q.put((rank, ok, msg, toks, ref))


def test_tp_decoder_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 150
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=600) for _ in procs])
    for p in procs:
        p.join(timeout=120)
    for rank, ok, msg, _, _ in res:
        assert ok, f"rank {rank}: {msg}"
    assert res[0][3] == res[1][3], "ranks disagree on the generated tokens"
    assert res[0][3][:4] == res[0][4], (res[0][3][:4], res[0][4])
