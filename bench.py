"""Benchmark: Sticky-KV decode at Llama-3-8B shape, 32k context.

Default workload (one GPU): a random-init Llama-3-8B-shaped decoder (32 layers,
hidden 4096, 32q/8kv heads, head_dim 128, FFN 14336, vocab 128256, bf16),
batch 1, a 32768-token prompt of uniform random token ids (prefill through the
Sticky-KV prefill lane), then greedy decode: at least W untimed warm-up steps
and K timed steps, each step = one token through all 32 layers.  Sticky-KV:
omega 64, sink 64, local 512, sticky 2048 tokens (32 windows), INT8 Q-cache
2048 tokens (32 windows).

The eviction cycle runs once per omega = 64 tokens.  The timed region starts
on a window boundary (the warm-up runs on to one, after timing a cycle step),
so K a multiple of 64 holds exactly K/64 cycles; for any other K the missing
share (K/64 minus the cycles timed) is added at the cycle step's measured
extra time, and the line says so (config.cycle_rate).

With --gpus N (torchrun) every rank decodes its own independent sequence (no
collective on the hot path): value = tokens/s summed over ranks, timed as the
max over ranks.

Prints one JSON line.  --impl reference runs the same decode on the host
cores: projections / MLP / LM head in torch, each layer's Sticky-KV attention,
ledger and eviction cycle in the oracle port of the reference (numpy), the
reference itself being Python that does not ship with this repository; the
port's speed relative to the reference's own code, measured where both run
(oracle/time_reference.py), is printed beside it.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s/GPU and fused-attn HBM GB/s (% of peak) at Llama-3-8B, 32k ctx"
WORKLOAD = ("Llama-3-8B-shaped full-model decode (32 layers, hidden 4096, 32q/8kv heads, head_dim 128, "
            "FFN 14336, vocab 128256), bf16 random init, batch 1 per GPU, 32768-token prompt + 512 decode "
            "steps; Sticky-KV omega 64, sink 64, local 512, sticky 2048, INT8 Q-cache 2048")
PROMPT = 32768


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------- CPU
PORT_VS_REF = os.path.join(ROOT, "oracle", "port_vs_reference.json")


def port_vs_reference():
    """The oracle port's speed against the reference's own decode step, measured
    where the reference is available (oracle/time_reference.py); None if absent."""
    if os.path.exists(PORT_VS_REF):
        with open(PORT_VS_REF) as f:
            return json.load(f)
    return None


class CpuPortDecoder:
    """The workload's decode on the host cores: a Llama-3-8B-shaped decoder whose
    projections, MLP and LM head run in torch (bf16, every host thread) and whose
    Sticky-KV attention, vote ledger and eviction cycle per layer run in the
    oracle port (numpy), the KV heads of a layer spread over a thread pool.

    Random-init weights (uniform, std 0.02), batch 1.  Each layer's cache state
    is built by the port's own prefill from a random rotated prompt of exactly
    sink + (sticky + Q) windows + local tokens with random per-key column scores
    (the decode-time state of the 32k-token workload: the same zone sizes)."""

    def __init__(self, n_layers=32, seed=0, threads=None):
        import concurrent.futures
        import numpy as np
        import torch

        from oracle.numerics import rnd
        from oracle.sticky_state import OracleStickyLayer
        self.np, self.torch = np, torch
        self.threads = threads or os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.pool = concurrent.futures.ThreadPoolExecutor(max_workers=min(self.threads, 8))
        self.L = n_layers
        hid, Hq, H, D, ffn, V = 4096, 32, 8, 128, 14336, 128256
        self.hid, self.Hq, self.H, self.D, self.G = hid, Hq, H, D, Hq // H
        g = torch.Generator().manual_seed(seed)
        pool = torch.empty(1 << 27, dtype=torch.bfloat16).uniform_(-0.0346, 0.0346, generator=g)

        def w(*shape):
            n = 1
            for x in shape:
                n *= x
            t = torch.empty(n, dtype=torch.bfloat16)
            off = int(torch.randint(0, pool.numel(), (1,), generator=g))
            done = 0
            while done < n:
                k = min(n - done, pool.numel() - off)
                t[done:done + k].copy_(pool[off:off + k])
                done += k
                off = 0
            return t.view(*shape)

        self.layers = [dict(wqkv=w((Hq + 2 * H) * D, hid), wo=w(hid, Hq * D), wgu=w(2 * ffn, hid), wd=w(hid, ffn))
                       for _ in range(n_layers)]
        self.embed = w(V, hid)
        self.lm_head = w(V, hid)
        self.ffn = ffn
        rng = np.random.default_rng(seed)
        om, sink, local, kw, qw = 64, 64, 512, 32, 32
        self.omega = om
        prompt = sink + (kw + qw) * om + local
        Kp = rnd(rng.standard_normal((H, prompt, D), dtype=np.float32), "bf16")
        Vp = rnd(rng.standard_normal((H, prompt, D), dtype=np.float32), "bf16")
        self.states, self.K, self.V = [], [], []
        for _ in range(n_layers):
            st = OracleStickyLayer(H, D, om, sink, local, kw, qw, "bf16", 8, max_windows=(40960 - sink) // om,
                                   max_context=8192, window_sum="sequential")
            cs = rng.random((H, 1, prompt), dtype=np.float32) * 4
            K, V = st.prefill(Kp, Vp, cs, "fp32")
            self.states.append(st)
            self.K.append(K)
            self.V.append(V)
        self.pos = 32768
        self.tok = 0

    def _attention(self, li, q, kn, vn):
        """One layer's Sticky-KV decode in the port: append, attention (heads in
        parallel), ledger tally, eviction cycle when due.  q [Hq, D], kn/vn [H, D]."""
        from oracle.attention import decode_attention
        np = self.np
        st = self.states[li]
        K = np.concatenate([self.K[li], kn[:, None]], 1)
        V = np.concatenate([self.V[li], vn[:, None]], 1)
        qc = None if st.q is None else {k: st.q[k] for k in ("kq", "ks", "kz", "vq", "vs", "vz")}
        G = self.G

        def head(h):
            qh = None if qc is None else {k: v[h:h + 1] for k, v in qc.items()}
            return decode_attention(q[h * G:(h + 1) * G], K[h:h + 1], V[h:h + 1], "bf16", qh)

        res = list(self.pool.map(head, range(self.H)))
        out = np.concatenate([r[0] for r in res], 0)
        sc = np.concatenate([r[1] for r in res], 0)
        qsc = None if qc is None else np.concatenate([r[2] for r in res], 0)
        self.K[li], self.V[li] = st.decode(K, V, sc, qsc, "bf16")
        return out

    def step(self, layers=None):
        """One decode token through `layers` layers (default all) and the LM head."""
        from oracle.numerics import rnd
        from oracle.sticky_state import apply_rope, rope_cos_sin
        np, torch = self.np, self.torch
        F = torch.nn.functional
        Hq, H, D = self.Hq, self.H, self.D
        cos, sin = rope_cos_sin(np.array([self.pos]), D, 500000.0, "bf16")
        x = self.embed[self.tok][None]
        for li in range(self.L if layers is None else layers):
            Lw = self.layers[li]
            h = F.rms_norm(x, (self.hid,), None, 1e-5)
            qkv = (h @ Lw["wqkv"].t())[0].float().numpy()
            q = apply_rope(qkv[:Hq * D].reshape(Hq, 1, D), cos, sin, "bf16")[:, 0]
            k = apply_rope(qkv[Hq * D:(Hq + H) * D].reshape(H, 1, D), cos, sin, "bf16")[:, 0]
            v = rnd(qkv[(Hq + H) * D:].reshape(H, D), "bf16")
            a = self._attention(li, q, k, v)
            x = x + torch.from_numpy(np.ascontiguousarray(a.reshape(1, Hq * D))).to(torch.bfloat16) @ Lw["wo"].t()
            h = F.rms_norm(x, (self.hid,), None, 1e-5)
            gu = h @ Lw["wgu"].t()
            x = x + (F.silu(gu[:, :self.ffn]) * gu[:, self.ffn:]) @ Lw["wd"].t()
        h = F.rms_norm(x, (self.hid,), None, 1e-5)
        self.tok = int(torch.argmax(h @ self.lm_head.t(), dim=-1))
        self.pos += 1

    def cycle_extra_s(self):
        """Host time one eviction cycle adds to a token (all layers): the port's
        cycle timed on a copy of layer 0's state, times the layer count."""
        import copy
        np = self.np
        st = copy.deepcopy(self.states[0])
        K, V = self.K[0], self.V[0]
        rng = np.random.default_rng(5)
        while st.tokens_since + 1 < st.omega:
            K = np.concatenate([K, K[:, -1:]], 1)
            V = np.concatenate([V, V[:, -1:]], 1)
            st.tally(K, rng.random((self.H, K.shape[1]), dtype=np.float32) * 1e-3, None, "bf16")
        K = np.concatenate([K, K[:, -1:]], 1)
        V = np.concatenate([V, V[:, -1:]], 1)
        st.tally(K, rng.random((self.H, K.shape[1]), dtype=np.float32) * 1e-3, None, "bf16")
        t0 = time.perf_counter()
        st.cycle(K, V)
        return (time.perf_counter() - t0) * self.L


def cpu_port_run(steps, warmup, budget_s=150.0, layers=32):
    """Time the port decoder: `warmup` untimed then `steps` timed tokens.  If the
    full tokens would not fit `budget_s`, each timed step runs a bounded sample
    of the layers (the same per-layer work) and the token time is scaled to all
    32 layers.  The eviction cycle enters at its true rate (one per 64 tokens):
    cycles inside the timed steps are replaced by steps/64 cycles of measured
    cost.  Returns a dict of the measurement."""
    dec = CpuPortDecoder(n_layers=layers)
    t0 = time.perf_counter()
    dec.step()
    t_tok = time.perf_counter() - t0
    n_sample = layers
    if (steps + warmup) * t_tok > budget_s:
        n_sample = max(1, min(layers, int(layers * budget_s / ((steps + warmup) * t_tok))))
    for _ in range(max(0, warmup - 1)):
        dec.step(n_sample)
    cycles, times = 0, []
    for _ in range(steps):
        c0 = sum(1 for st in dec.states[:n_sample] if st.tokens_since + 1 == st.omega)
        t0 = time.perf_counter()
        dec.step(n_sample)
        times.append(time.perf_counter() - t0)
        cycles += 1 if c0 else 0
    c_extra = dec.cycle_extra_s() * n_sample / layers
    total = sum(times) + (steps / dec.omega - cycles) * c_extra
    per_tok = total / steps * layers / n_sample
    return {"s_per_token": per_tok, "timed_s": sum(times), "layers_per_step": n_sample, "cycles_timed": cycles,
            "cycle_extra_s": c_extra * layers / n_sample, "threads": dec.threads, "steps": steps, "warmup": warmup}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    r = cpu_port_run(args.steps, args.warmup)
    tps = 1.0 / r["s_per_token"]
    pvr = port_vs_reference()
    sample = (f"oracle port of the reference's decode path: Llama-3-8B-shaped decoder on the host, projections / "
              f"MLP / LM head in torch bf16 on {r['threads']} threads, each layer's Sticky-KV attention + ledger + "
              f"eviction cycle in numpy (KV heads over a thread pool), one sequence; "
              f"{r['layers_per_step']} of 32 layers per timed step"
              + (" (all of them)" if r["layers_per_step"] == 32 else ", token time scaled to 32 layers")
              + f"; {r['cycles_timed']} eviction cycles in the timed steps, cycles counted at 1 per 64 tokens "
              f"({r['cycle_extra_s'] * 1e3:.0f} ms each)")
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["s_per_token"] * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: random-init weights, random rotated K/V prompt state, random per-key column scores",
            "config": {"workload": WORKLOAD, "timed_s": round(r["timed_s"], 2)},
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": r["threads"], "kind": "port",
                             "sample": sample, "port_vs_reference": pvr},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU
def max_over_ranks_on(x, world, device):
    """Maximum of a per-rank number over all ranks (the job's time is its slowest rank's)."""
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args):
    import torch
    import torch.distributed as dist

    from qevict_b200.model import LlamaShape, StickyLlamaDecoder, StickyShape

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        return max_over_ranks_on(x, world, dev)

    torch.backends.cuda.matmul.allow_tf32 = False
    model = StickyLlamaDecoder(LlamaShape(), StickyShape(), batch=1, max_pos=PROMPT + 4096, device=dev,
                               seed=1234 + rank)
    g = torch.Generator(device=dev)
    g.manual_seed(99 + rank)
    ids = torch.randint(0, model.s.vocab, (1, PROMPT), generator=g, device=dev)
    t0 = time.perf_counter()
    model.prefill(ids)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    del ids

    W, K = args.warmup, args.steps
    om = model.k.omega
    # per layer: gemv_kernel x4 (qkv, output, gate/up, down), rope_append_kernel,
    # decode_mma_kernel, decode_combine_kernel, add_rmsnorm_kernel x2,
    # silu_mul_kernel; per step: the first add_rmsnorm_kernel, the LM head's
    # gemv_kernel and argmax_kernel
    launches_per_step = 10 * model.s.layers + 3
    # warm-up: eager first (allocator / cuBLAS), then graph capture, then graph
    # replays; the replays continue past W until (a) a step that ends a window
    # (and runs the eviction cycle of every layer) has been timed and (b) the
    # next step starts a window, so the timed region starts on a window
    # boundary and holds the cycle at its true rate, one per omega steps
    n_eager = min(3, W)
    for _ in range(n_eager):
        model.step_eager()
    torch.cuda.synchronize()
    model.capture()
    plain_ms, cycle_ms = [], []
    n_warm = n_eager
    st0 = model.states[0]
    while n_warm < W or not cycle_ms or (st0.n_tokens - st0.prompt_len) % om != 0:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        cyc = model.step_graph()
        b.record()
        b.synchronize()
        (cycle_ms if cyc else plain_ms).append(a.elapsed_time(b))
        n_warm += 1
    plain_med = statistics.median(plain_ms[-32:]) if plain_ms else 0.0
    # all ranks agree on the cycle's extra time (the slowest rank's)
    cycle_extra_ms = max_over_ranks(max(0.0, statistics.median(cycle_ms) - plain_med))

    # ---- timed region: K graph-replayed steps, inputs resident on the device.
    # The clock sampler runs over the timed steps and over whole windows of
    # identical steps just before them (>= ~1 s under load, so that nvidia-smi
    # takes several samples even when K steps last only tens of ms)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cycles = 0
    with ClockSampler(torch.cuda.current_device()) as clk:
        pre = max(1, int(math.ceil(1200.0 / max(1e-3, om * plain_med))))
        for _ in range(pre * om):
            model.step_graph()
        barrier()
        torch.cuda.synchronize()
        # a profiler started with profiling off (ncu --profile-from-start off)
        # records exactly the timed steps; without a profiler these are no-ops
        torch.cuda.profiler.start()
        start.record()
        for _ in range(K):
            cycles += model.step_graph()
        end.record()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        barrier()
    raw_ms = max_over_ranks(start.elapsed_time(end))
    # the cycle at its true rate: K/omega cycles (a timed region shorter than a
    # window holds none; one of whole windows holds exactly K/omega)
    added_ms = (K / om - cycles) * cycle_extra_ms
    ms = raw_ms + added_ms
    # an eviction cycle adds cycle_select, up_gather, demote and up_scatter per layer
    gpu_launches = K * launches_per_step + cycles * 4 * model.s.layers
    tok_s = world * K / (ms / 1e3)

    # ---- end to end through the public API: pinned host token in, next token out, every step
    Ke = min(K, 128)
    h_in = torch.zeros(1, dtype=torch.long, pin_memory=True)
    h_out = torch.zeros(1, dtype=torch.long, pin_memory=True)
    h_in.copy_(model.tok.cpu())
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e_cycles = 0
    e0.record()
    for _ in range(Ke):
        model.tok.copy_(h_in, non_blocking=True)
        e_cycles += model.step_graph()
        h_out.copy_(model.next_tok, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        h_in.copy_(h_out)
    e1.record()
    torch.cuda.synchronize()
    e_ms = max_over_ranks(e0.elapsed_time(e1)) + (Ke / om - e_cycles) * cycle_extra_ms
    e2e = {"value": world * Ke / (e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 8,
           "d2h_bytes_per_step": 8, "steps": Ke, "eviction_cycles": e_cycles,
           "cycle_rate": "as the device-timed value: cycles counted at one per omega steps"}

    # ---- live roofline of the fused attention kernel: CUDA events around every launch
    n_inst = min(64, K)
    evs = []
    for _ in range(n_inst):
        cyc = model.cycle_next()
        x = model.embed[model.tok]
        for li in range(model.s.layers):
            L, st = model.layers[li], model.states[li]
            s = model.s
            h = torch.nn.functional.rms_norm(x, (s.hidden,), L["ln1"], s.rms_eps)
            qkv = h @ L["wqkv"].t()
            Hq, H, D = s.heads, s.kv_heads, s.head_dim
            qr = st.append(qkv[:, :Hq * D].reshape(1, Hq, D), qkv[:, Hq * D:(Hq + H) * D].reshape(1, H, D),
                           qkv[:, (Hq + H) * D:].reshape(1, H, D), model.cos, model.sin)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            # keep the stream busy while the host issues the launch, so the two
            # events bracket device time only
            torch.cuda._sleep(1000000)
            a.record()
            st.attend(qr, model.attn_out)
            b.record()
            evs.append((a, b, (st.n_tokens - 1 - st.prompt_len) % st.omega + 1))
            x = x + model.attn_out.reshape(1, Hq * D) @ L["wo"].t()
            x = model._mlp(x, L)
            if cyc:
                st.evict_cycle()
        hh = torch.nn.functional.rms_norm(x, (model.s.hidden,), model.norm, model.s.rms_eps)
        model.tok.copy_(torch.argmax(hh @ model.lm_head.t(), dim=-1))
    torch.cuda.synchronize()
    durs = [a.elapsed_time(b) * 1e-3 for a, b, _ in evs]
    bytes_ = [model.attention_bytes_per_layer(t) for _, _, t in evs]
    avg_dur = sum(durs) / len(durs)
    achieved = (sum(bytes_) / len(bytes_)) / avg_dur / 1e9
    peak, peak_kind = peaks()
    traffic = None
    tf = os.path.join(ROOT, "profiles", "decode_attention_traffic.txt")
    if os.path.exists(tf):
        with open(tf) as f:
            for ln in f:
                if ln.startswith("bytes_per_launch"):
                    traffic = int(ln.split("=")[1])

    # ---- the whole step against HBM: bytes a decode step must read (every
    # weight once + the live KV of every layer) / device time per step
    wbytes = sum(L[k].numel() * L[k].element_size() for L in model.layers for k in ("wqkv", "wo", "wgu", "wd"))
    wbytes += model.lm_head.numel() * model.lm_head.element_size() + model.s.hidden * 2
    kvbytes = model.s.layers * model.attention_bytes_per_layer((model.k.omega + 1) / 2)
    step_gbs = (wbytes + kvbytes) / (ms / K * 1e-3) / 1e9

    # ---- decode-attention microbenchmark at batch 64 (one Llama-3-8B layer, 64 sink
    # + 512 local + 2048 sticky bf16 tokens and 4096 INT8 Q-cache tokens per
    # sequence, eviction cycle every 64 steps, L2 flushed before every step)
    attn_b64 = None
    if rank == 0:
        try:
            from qevict_b200 import microbench
            r = microbench.run(batch=64, steps=200, warmup=8, quiet=True)
            attn_b64 = {"batch": 64, "steps": 200, "avg_launch_us": r["avg_attention_us"],
                        "bytes_per_launch": r["avg_bytes_per_launch"], "achieved": r["attention_GBps"],
                        "unit": "GB/s", "peak": peak, "frac": r["attention_GBps"] / peak,
                        "cycle_fraction_of_step": r["cycle_fraction_of_step"], "cycle_us_avg": r["cycle_us_avg"],
                        "l2": "flushed before every step"}
        except Exception as exc:   # the headline line must still print
            attn_b64 = {"error": str(exc)[:200]}

    if rank == 0:
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: random-init weights N(0,0.02), uniform random prompt token ids",
            "config": {"workload": WORKLOAD, "prompt_tokens": PROMPT, "batch_per_gpu": 1,
                       "parallelism": f"{world} independent sequence(s), one per GPU",
                       "l2": "no flush needed: each step streams ~15 GB of weights, far above the 126 MB L2",
                       "prefill_s": round(prefill_s, 2), "warmup_steps_run": n_warm,
                       "eviction_cycles_timed": cycles,
                       "cycle_rate": {"method": ("timed region starts on a window boundary; K/omega cycles "
                                                 "counted: (K/omega - cycles timed) x the measured extra time "
                                                 "of a cycle step added to the device time"),
                                      "cycles_at_true_rate": K / om, "cycle_step_extra_ms": cycle_extra_ms,
                                      "plain_step_ms": plain_med, "added_ms": added_ms,
                                      "device_timed_ms": raw_ms}},
            "roofline": {"bound": "hbm", "kernel": "qv_decode_attention (decode_mma_kernel + decode_combine_kernel)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": peak_kind, "traffic": traffic,
                         "avg_launch_us": avg_dur * 1e6, "bytes_per_launch": sum(bytes_) / len(bytes_)},
            "step_roofline": {"bound": "hbm", "bytes_per_step": wbytes + kvbytes, "weight_bytes": wbytes,
                              "kv_bytes": kvbytes, "achieved": step_gbs, "peak": peak, "unit": "GB/s",
                              "frac": step_gbs / peak},
            "attention_microbench": attn_b64,
            "e2e": e2e,
            "gpu_launches": gpu_launches,
            "clocks": dict(clk.summary(), window=f"the timed steps and {pre * om} identical steps just before them"),
        }
        if world == 1:
            r = cpu_port_run(steps=args.cpu_steps, warmup=1)
            line["cpu_baseline"] = {
                "value": 1.0 / r["s_per_token"], "unit": "tokens/s", "cores": r["threads"], "kind": "port",
                "sample": (f"{r['steps']} tokens of the same workload on the host: projections / MLP / LM head in "
                           f"torch bf16 ({r['threads']} threads), Sticky-KV attention + ledger + cycle of each "
                           f"layer in the oracle port (numpy, KV heads over a thread pool), "
                           f"{r['layers_per_step']} of 32 layers per token"
                           + ("" if r["layers_per_step"] == 32 else " scaled to 32")
                           + ", eviction cycles at 1 per 64 tokens"),
                "port_vs_reference": port_vs_reference()}
        print(json.dumps(line), flush=True)
    model.graphs.clear()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


TP_PROMPT = 131072
TP_WORKLOAD = ("Llama-3-8B-shaped full-model decode with KV-head tensor parallelism over the job's GPUs (q/k/v and "
               "gate/up column-parallel, o_proj and down row-parallel with one all-reduce each -- in decode the "
               "library's NVLink peer-store sum, NCCL with --tp-nccl and in prefill -- vocab-parallel "
               "LM head), bf16 random init, batch 1, 131072-token prompt (prefill lane: causal attention + per-key "
               "column sums seeding the ledger), then decode; Sticky-KV omega 64, sink 64, local 512, sticky 4096, "
               "INT8 Q-cache 8192")


def run_tp(args):
    """The long-context workload split by KV head over the job's ranks (strong scaling)."""
    import datetime

    import torch
    import torch.distributed as dist

    from qevict_b200.model import LlamaShape, StickyShape
    from qevict_b200.tp_model import TpStickyLlamaDecoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev,
                            rank=rank, world_size=world) if world > 1 else None
    torch.backends.cuda.matmul.allow_tf32 = False
    prompt = args.tp_prompt
    sticky = StickyShape(k_windows=64, q_windows=128)
    model = TpStickyLlamaDecoder(LlamaShape(), sticky, rank, world, batch=1, max_pos=prompt + 4096, device=dev,
                                 seed=1234, peer_sum=not args.tp_nccl)
    g = torch.Generator(device=dev)
    g.manual_seed(99)
    ids = torch.randint(0, model.s.vocab, (1, prompt), generator=g, device=dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    model.prefill(ids)
    torch.cuda.synchronize()
    prefill_s = max_over_ranks_on(time.perf_counter() - t0, world, dev)
    del ids
    W, K = args.warmup, args.steps
    om = sticky.omega
    for _ in range(min(3, W)):
        model.step_eager()
    torch.cuda.synchronize()
    model.capture()
    plain_ms, cycle_ms = [], []
    n_warm = min(3, W)
    st0 = model.states[0]
    while n_warm < W or not cycle_ms or (st0.n_tokens - st0.prompt_len) % om != 0:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        cyc = model.step_graph()
        b.record()
        b.synchronize()
        (cycle_ms if cyc else plain_ms).append(a.elapsed_time(b))
        n_warm += 1
    plain_med = statistics.median(plain_ms[-32:]) if plain_ms else 0.0
    cycle_extra_ms = max_over_ranks_on(max(0.0, statistics.median(cycle_ms) - plain_med), world, dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cycles = 0
    with ClockSampler(torch.cuda.current_device()) as clk:
        for _ in range(max(1, int(math.ceil(1200.0 / max(1e-3, om * plain_med)))) * om):
            model.step_graph()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(K):
            cycles += model.step_graph()
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    raw_ms = max_over_ranks_on(start.elapsed_time(end), world, dev)
    added_ms = (K / om - cycles) * cycle_extra_ms
    ms = raw_ms + added_ms
    # the collectives of one plain step alone (same sizes, same group), captured
    # in a graph and replayed: the latency floor the exchange puts under a token
    coll_ms = coll_nccl_ms = None
    if world > 1:
        xs = torch.zeros(1, model.s.hidden, dtype=torch.bfloat16, device=dev)
        key = torch.zeros(1, dtype=torch.int64, device=dev)

        def time_collectives(nccl_only):
            def collectives():
                for _ in range(2 * model.s.layers):
                    if nccl_only:
                        dist.all_reduce(xs, op=dist.ReduceOp.SUM, group=model.group)
                    else:
                        model._sum(xs)
                if nccl_only or model.ps is None:
                    dist.all_reduce(key, op=dist.ReduceOp.MAX, group=model.group)
                else:
                    model.ps.max_(key)

            side = torch.cuda.Stream(device=dev)
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                collectives()
            torch.cuda.current_stream().wait_stream(side)
            cg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(cg):
                collectives()
            for _ in range(3):
                cg.replay()
            dist.barrier()
            torch.cuda.synchronize()
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n_rep = 20
            c0.record()
            for _ in range(n_rep):
                cg.replay()
            c1.record()
            torch.cuda.synchronize()
            t = max_over_ranks_on(c0.elapsed_time(c1) / n_rep, world, dev)
            del cg
            dist.barrier()
            return t

        coll_ms = time_collectives(False)
        coll_nccl_ms = time_collectives(True)
    # per layer: gemv x4, rope_append, decode_mma, fold, add_rmsnorm x2, silu_mul (+ torch's
    # argmax pieces per step); per cycle and layer: count + ext
    launches = K * (10 * model.s.layers + 3) + cycles * 2 * model.s.layers
    kv = model.s.layers * model.attention_bytes_per_layer((om + 1) / 2)
    step_bytes = model.weight_bytes() + kv
    peak, peak_kind = peaks()
    if rank == 0:
        line = {"metric": METRIC, "value": K / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": K,
                "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic: random-init weights N(0,0.02), uniform random prompt token ids",
                "config": {"workload": TP_WORKLOAD, "prompt_tokens": prompt, "batch": 1,
                           "parallelism": f"kv-head tensor parallel x{world} ({model.hl} KV head(s) per GPU)",
                           "prefill_s": round(prefill_s, 2), "eviction_cycles_timed": cycles,
                           "cycle_rate": {"cycles_at_true_rate": K / om, "cycle_step_extra_ms": cycle_extra_ms,
                                          "added_ms": added_ms, "device_timed_ms": raw_ms},
                           "collectives_per_step": {"all_reduce_sum_bf16_hidden": 2 * model.s.layers,
                                                    "all_reduce_max_int64": 1,
                                                    "all_reduce_min_int32_per_cycle": model.s.layers},
                           "collectives_alone_ms_per_step": coll_ms,
                           "collectives_alone_all_nccl_ms_per_step": coll_nccl_ms,
                           "decode_collectives": ("qv_peer_sum / qv_peer_max_i64 (NVLink peer stores)"
                                                  if model.ps is not None else "NCCL"),
                           "collectives_share_of_step": None if coll_ms is None else coll_ms / (ms / K)},
                "step_roofline": {"bound": "hbm", "bytes_per_step_per_gpu": step_bytes,
                                  "achieved": step_bytes / (ms / K * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                                  "frac": step_bytes / (ms / K * 1e-3) / 1e9 / peak, "peak_source": peak_kind},
                "gpu_launches": launches, "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=448)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-steps", type=int, default=8, help="tokens the host baseline times (rank 0, N=1)")
    ap.add_argument("--tp", action="store_true", help="the long-context workload, KV heads split over the ranks")
    ap.add_argument("--tp-prompt", type=int, default=TP_PROMPT)
    ap.add_argument("--tp-nccl", action="store_true", help="--tp with NCCL for the decode sums (no qv_peer_sum)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.tp:
        run_tp(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
