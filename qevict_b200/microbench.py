"""Decode-attention microbenchmark at Llama-3-8B layer shape.

One Sticky-KV layer (8 KV heads, GQA group 4, head_dim 128, bf16) for B
sequences, state built from a random prompt through the prefill state builder,
then decode steps of RoPE + append, the fused attention with the ledger fold,
and the eviction cycle every omega tokens.  Inputs are random; per-step
device time is taken with CUDA events on the launching stream (the stream is
kept busy while the host issues each launch, so the events bracket device
time only).

Default sizes are the decode microbenchmark configuration: batch 64,
per-sequence cache of 64 sink + 512 local + 2048 sticky BF16 tokens and 4096
INT8 Q-cache tokens, 1000 steps.

    python -m qevict_b200.microbench [--batch 64] [--steps 1000] [--sticky 32] [--qwin 64]
    python -m qevict_b200.microbench --prefill 8192 [--steps 5]   (one layer's prefill lane)
    python -m qevict_b200.microbench --mha-spikes [--batch 16] [--steps 256]
        (Llama-2-7B MHA layer, fp16, 16384-token prompts, planted attention
        spikes that force promotions and demotions every cycle; under torchrun
        the batch is split over the ranks)
"""

import argparse
import json
import math

import torch

from .layer_state import StickyLayerState

H, G, D, OMEGA, SINK = 8, 4, 128, 64, 64


def algorithmic_bytes(batch, sticky, qwin, local, t, e=2, qbytes=128):
    """HBM bytes one attention launch must read: BF16 K+V of the live main zone,
    INT8 K+V codes + per-token V scale/zp + per-window K scale/zp of the Q-cache."""
    s_m = SINK + sticky * OMEGA + local + t
    s_q = qwin * OMEGA
    return batch * H * (s_m * 2 * D * e + s_q * (2 * qbytes + 2 * e) + qwin * 2 * D * e)


def build(batch, sticky, qwin, local, seed=0, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    st = StickyLayerState(batch, H, G, D, OMEGA, SINK, local, sticky, qwin, 4096, 8, dtype)
    prompt = SINK + (sticky + qwin) * OMEGA + local
    k = torch.randn(batch, H, prompt, D, generator=g, device="cuda").to(dtype)
    v = torch.randn(batch, H, prompt, D, generator=g, device="cuda").to(dtype)
    cs = torch.rand(batch, H, prompt, generator=g, device="cuda") * 4
    st.prefill(k, v, cs)
    del k, v, cs
    torch.cuda.synchronize()
    return st, g


def run(batch=64, steps=1000, warmup=8, sticky=32, qwin=64, local=512, quiet=False, fold=True):
    """fold=False times the attention without its vote-ledger fold
    (qv_decode_attention_nofold); the fold then runs after the timed span."""
    st, g = build(batch, sticky, qwin, local)
    q = torch.randn(batch, H * G, D, generator=g, device="cuda").to(st.dtype) * 0.3
    kn = torch.randn(batch, H, D, generator=g, device="cuda").to(st.dtype)
    vn = torch.randn(batch, H, D, generator=g, device="cuda").to(st.dtype)
    out = torch.empty(batch, H * G, D, dtype=st.dtype, device="cuda")
    # warm-up covers at least one eviction cycle, so first-launch costs of the
    # cycle kernels stay out of the timed steps
    for _ in range(max(warmup, st.omega + 1)):
        st.step(q, kn, vn, out=out)
    torch.cuda.synchronize()
    attn_t, cyc_t, step_t, tvals = [], [], [], []
    # a buffer larger than the 126 MB L2, rewritten before every step so that the
    # cache arrives cold, as it does in a model where the weights stream between
    # two launches of a layer
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    for _ in range(steps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        flush.zero_()
        torch.cuda._sleep(2000000)
        ev[0].record()
        qr = st.append(q, kn, vn)
        ev[1].record()
        st.attend(qr, out, fold=fold)
        ev[2].record()
        if not fold:
            st.fold()
        t = (st.n_tokens - st.prompt_len - 1) % st.omega + 1
        cyc = st.cycle_due()
        if cyc:
            st.evict_cycle()
        ev[3].record()
        tvals.append(t)
        step_t.append(ev)
    torch.cuda.synchronize()
    for ev, t in zip(step_t, tvals):
        attn_t.append(ev[1].elapsed_time(ev[2]) * 1e-3)
        cyc_t.append(ev[2].elapsed_time(ev[3]) * 1e-3)
    n_cyc = sum(1 for t in tvals if t == OMEGA)
    by = [algorithmic_bytes(batch, sticky, qwin, local, t) for t in tvals]
    avg_attn = sum(attn_t) / len(attn_t)
    res = {
        "batch": batch, "steps": steps, "avg_attention_us": avg_attn * 1e6,
        "attention_GBps": sum(by) / sum(attn_t) / 1e9,
        "avg_bytes_per_launch": sum(by) / len(by),
        "cycle_us_avg": (sum(c for c, t in zip(cyc_t, tvals) if t == OMEGA) / max(1, n_cyc)) * 1e6,
        "cycle_fraction_of_step": (sum(cyc_t) / max(1e-12, sum(attn_t) + sum(cyc_t))),
        "decode_path": st.decode_path, "error_word": st.read_error(), "ledger_fold_timed": fold,
    }
    if not quiet:
        print(json.dumps(res))
    return res


def run_prefill(S=8192, batch=1, steps=5, quiet=False, dtype=torch.bfloat16):
    """One layer's prefill lane (causal attention + column sums) at the Llama-3-8B
    layer shape; reports ms per layer and TFLOP/s of the minimal causal
    contraction count 2 * S^2 * D * Hq (Q.K^T and P.V over the lower triangle)."""
    from .model import prefill_attention
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    Hq = H * G
    q = torch.randn(batch, S, Hq, D, generator=g, device="cuda").to(dtype)
    k = torch.randn(batch, S, H, D, generator=g, device="cuda").to(dtype)
    v = torch.randn(batch, S, H, D, generator=g, device="cuda").to(dtype)
    prefill_attention(q, k, v)          # reads the device error word back
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        prefill_attention(q, k, v, check=False)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    flops = 2.0 * S * S * D * Hq * batch
    res = {"prefill_tokens": S, "batch": batch, "ms_per_layer": ms, "tflops_causal": flops / (ms * 1e-3) / 1e12}
    if not quiet:
        print(json.dumps(res))
    return res


def run_mha_spikes(batch=16, steps=256, warmup=8, prompt=16384, sticky=8, qwin=64, local=512, heads=32,
                   frac=0.05, n_dirs=4, seed=0, quiet=False):
    """The batch-sharded MHA workload on one layer: Llama-2-7B attention shape
    (32 heads, no GQA, head_dim 128), fp16, `batch` sequences of `prompt`
    tokens split over the ranks of a torch.distributed job (none: one GPU),
    sticky 8 windows (512 tokens) / Q-cache 64 windows (4096 tokens) of 64,
    sink 64, local 512.

    Planted spikes: n_dirs unit directions u_r per (sequence, head); for each,
    a random `frac` of the prompt's windows get keys 4 u_r (plus noise of 0.1):
    against a query of norm sqrt(D) along u_r their logit q.k / sqrt(D) is
    about 4, against about N(0, 1) for the random keys.  Decode queries point
    along u_r for the cycle r = (window index) mod n_dirs, so each eviction
    cycle the vote mass moves to another set of windows: windows are promoted
    out of the Q-cache and sticky windows demoted into it every cycle.

    Per step: RoPE-free append, the fused attention with the ledger fold, and
    the cycle every 64 tokens, device-timed with CUDA events (L2 flushed before
    every step).  Returns the rank's figures and, under torchrun, the job's
    (time = max over ranks, tokens summed)."""
    import os
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        if not dist.is_initialized():
            import datetime
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device("cuda", torch.cuda.current_device()))
    if batch % world:
        raise ValueError(f"batch {batch} does not split over {world} ranks")
    B = batch // world
    Hh, D, dt = heads, 128, torch.float16
    g = torch.Generator(device="cuda")
    g.manual_seed(seed + 1000 * rank)
    n_win = (prompt - SINK) // OMEGA
    st = StickyLayerState(B, Hh, 1, D, OMEGA, SINK, local, sticky, qwin, n_win + steps // OMEGA + 8, 8, dt)
    k = torch.randn(B, Hh, prompt, D, generator=g, device="cuda", dtype=dt)
    v = torch.randn(B, Hh, prompt, D, generator=g, device="cuda", dtype=dt)
    u = torch.nn.functional.normalize(torch.randn(n_dirs, B, Hh, D, generator=g, device="cuda"), dim=-1)
    # plant: for each direction, a random frac of the windows get keys 4 * u (+ small noise)
    kw = k[:, :, SINK:SINK + n_win * OMEGA].view(B, Hh, n_win, OMEGA, D)
    for r in range(n_dirs):
        sel = torch.rand(B, Hh, n_win, generator=g, device="cuda") < frac
        planted = (4.0 * u[r][:, :, None, None, :] + 0.1 * torch.randn(B, Hh, n_win, OMEGA, D, generator=g,
                                                                       device="cuda")).to(dt)
        kw.copy_(torch.where(sel[..., None, None], planted, kw))
    cs = torch.rand(B, Hh, prompt, generator=g, device="cuda") * 4
    st.prefill(k, v, cs)
    del k, v, kw, cs
    torch.cuda.synchronize()

    def query(step):
        r = ((st.n_tokens - st.prompt_len) // OMEGA) % n_dirs
        q = u[r] * math.sqrt(D) + 0.3 * torch.randn(B, Hh, D, generator=g, device="cuda")
        return q.to(dt)

    out = torch.empty(B, Hh, D, dtype=dt, device="cuda")
    kn = torch.randn(B, Hh, D, generator=g, device="cuda").to(dt)
    vn = torch.randn(B, Hh, D, generator=g, device="cuda").to(dt)
    for i in range(max(warmup, OMEGA + 1)):
        st.step(query(i), kn, vn, out=out)
    torch.cuda.synchronize()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    evs, tvals, moved = [], [], []
    for i in range(steps):
        q = query(i)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        flush.zero_()
        torch.cuda._sleep(2000000)
        ev[0].record()
        qr = st.append(q, kn, vn)
        ev[1].record()
        st.attend(qr, out)
        ev[2].record()
        t = (st.n_tokens - st.prompt_len - 1) % OMEGA + 1
        cyc = st.cycle_due()
        if cyc:
            before = st.sticky_wid.clone()
            st.evict_cycle()
        ev[3].record()
        if cyc:
            # windows that left the sticky slots (demoted or evicted) this cycle
            moved.append(int((st.sticky_wid != before).sum()))
        evs.append(ev)
        tvals.append(t)
    torch.cuda.synchronize()
    attn = [e[1].elapsed_time(e[2]) * 1e-3 for e in evs]
    cyc_t = [e[2].elapsed_time(e[3]) * 1e-3 for e, t in zip(evs, tvals) if t == OMEGA]
    app = [e[0].elapsed_time(e[1]) * 1e-3 for e in evs]
    by = [B * Hh * ((SINK + sticky * OMEGA + local + t) * 2 * D * 2 + qwin * OMEGA * (2 * D + 2 * 2)
                    + qwin * 2 * D * 2) for t in tvals]
    step_s = sum(attn) + sum(app) + sum(cyc_t)
    tot = {"attn_s": sum(attn), "step_s": step_s, "bytes": float(sum(by))}
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([tot["attn_s"], tot["step_s"]], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        b = torch.tensor([tot["bytes"]], dtype=torch.float64, device="cuda")
        dist.all_reduce(b, op=dist.ReduceOp.SUM)
        tot = {"attn_s": float(t[0]), "step_s": float(t[1]), "bytes": float(b[0])}
    res = {"workload": "Llama-2-7B MHA layer, fp16, 16384-token prompts, sticky 512 / Q-cache 4096, planted spikes",
           "batch": batch, "ranks": world, "batch_per_rank": B, "steps": steps,
           "avg_attention_us_rank": sum(attn) / steps * 1e6,
           "attention_GBps_job": tot["bytes"] / tot["attn_s"] / 1e9,
           "cycle_us_avg_rank": (sum(cyc_t) / max(1, len(cyc_t))) * 1e6,
           "cycle_fraction_of_step": sum(cyc_t) / max(1e-12, sum(attn) + sum(app) + sum(cyc_t)),
           "sticky_slots_changed_per_cycle": moved, "cycles": len(cyc_t),
           "tokens_per_s_job": batch * steps / tot["step_s"],
           "decode_path": st.decode_path, "error_word": st.read_error()}
    if not quiet and rank == 0:
        print(json.dumps(res))
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--sticky", type=int, default=32)
    ap.add_argument("--qwin", type=int, default=64)
    ap.add_argument("--local", type=int, default=512)
    ap.add_argument("--prefill", type=int, default=0, help="time one layer's prefill lane at this prompt length")
    ap.add_argument("--mha-spikes", action="store_true", help="the batch-sharded MHA workload with planted spikes")
    ap.add_argument("--nofold", action="store_true", help="time the attention without its vote-ledger fold")
    a = ap.parse_args()
    if a.mha_spikes:
        run_mha_spikes(batch=a.batch if a.batch != 64 else 16, steps=a.steps if a.steps != 1000 else 256,
                       warmup=a.warmup)
        return
    if a.prefill:
        run_prefill(a.prefill, steps=max(1, min(a.steps, 20)))
        return
    run(a.batch, a.steps, a.warmup, a.sticky, a.qwin, a.local, fold=not a.nofold)


if __name__ == "__main__":
    main()
