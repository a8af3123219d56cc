"""Host-side timing of the reference's own decode step against this oracle port.

Test/bench infrastructure, not product code.  The reference is Python and
cannot be shipped with this repository, so the benchmark's CPU arm times the
oracle port (oracle/) instead; this script measures, on one machine, how the
port's speed compares with the reference's own code on the same work, and
writes the result to oracle/port_vs_reference.json, which bench.py prints
beside its CPU numbers.

Work timed (one layer of the full-model workload's decode, bf16, 8 KV heads,
group 4, head_dim 128, omega 64, sink 64, local 512, 32 sticky + 32 INT8 Q
windows), per decode token:
  * reference: the torch.cat append (module.py:198-200), compute_main_logits
    (ops.py:23-46), compute_qcache_joint_softmax (ops.py:74-169) and
    STICKYKVCache_LayerWise.__call__ (cache.py:234-427, an eviction cycle
    every 64 tokens), on all host threads (torch);
  * port: the same steps in oracle.attention.decode_attention and
    OracleStickyLayer.decode (numpy), on one thread and with the KV heads of
    the attention spread over a thread pool (as bench.py's host arm runs it).

    python oracle/time_reference.py <reference checkout> [--steps 128]
"""

import argparse
import json
import os
import platform
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
H, G, D, OMEGA, SINK, LOCAL, KW, QW = 8, 4, 128, 64, 64, 512, 32, 32


def time_reference(ref, steps, seed=0):
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref)
    sys.path.insert(0, os.path.join(ref, "src"))
    import torch
    import src.sticky_config as sticky_config
    import src.models.kv_cache.cache as ref_cache_mod
    from src.models.kv_cache.allocator import BudgetResult
    from src.models.kv_cache.cache import STICKYKVCache_LayerWise
    from src.models.attention import ops as ref_ops
    from src.models.configuration_sticky_llama import LlamaConfig
    torch.set_num_threads(os.cpu_count() or 1)
    sticky_config.OMEGA, sticky_config.SINK_TOKENS = OMEGA, SINK
    sticky_config.QUANTIZATION_BIT_WIDTH, sticky_config.LOCAL_NUM_TOKENS = 8, LOCAL
    ref_cache_mod.compute_budget = lambda **kw: BudgetResult(local_num=LOCAL, k_windows=KW, q_windows_count=QW,
                                                             q_num=0, quant_bytes_len=D)
    cfg = LlamaConfig(hidden_size=H * G * D, num_attention_heads=H * G, num_key_value_heads=H,
                      max_position_embeddings=8192, intermediate_size=8192, num_hidden_layers=2)
    cfg.rope_parameters = {"rope_type": "default", "rope_theta": 500000.0}
    cache = STICKYKVCache_LayerWise(p_ratio=50, r_ratio=20, start_idx=0, num_heads=H, layer_idx=1, config=cfg)
    g = torch.Generator().manual_seed(seed)
    prompt = SINK + (KW + QW) * OMEGA + LOCAL
    K = torch.randn(1, H, prompt, D, generator=g).to(torch.bfloat16)
    V = torch.randn(1, H, prompt, D, generator=g).to(torch.bfloat16)
    attn = torch.rand(1, H, 1, prompt, generator=g) * 4.0
    kv = cache((K, V), attn, q_len=prompt)
    times = []
    for _ in range(steps):
        q = (torch.randn(1, H * G, 1, D, generator=g) * 0.3).to(torch.bfloat16)
        kn = torch.randn(1, H, 1, D, generator=g).to(torch.bfloat16)
        vn = torch.randn(1, H, 1, D, generator=g).to(torch.bfloat16)
        t0 = time.perf_counter()
        Kc = torch.cat([kv[0], kn], dim=2)
        Vc = torch.cat([kv[1], vn], dim=2)
        S = Kc.shape[2]
        lg = ref_ops.compute_main_logits(q, Kc, 1, H * G, H, G, 1, D)
        lg = lg + torch.zeros(1, 1, 1, S, dtype=torch.bfloat16)
        _, sc, qs, _ = ref_ops.compute_qcache_joint_softmax(q, lg, Vc, cache, 1, H * G, H, G, 1, D)
        kv = cache((Kc, Vc), sc, q_len=1, q_attn_scores=qs)
        times.append(time.perf_counter() - t0)
    return float(np.mean(times)), torch.get_num_threads()


def time_port(steps, seed=0, threads=1):
    """The port on the same work; threads > 1 spreads the KV heads of the
    attention over a thread pool, as the benchmark's host arm runs it."""
    import concurrent.futures
    sys.path.insert(0, os.path.dirname(HERE))
    from oracle.attention import decode_attention
    from oracle.numerics import rnd
    from oracle.sticky_state import OracleStickyLayer
    rng = np.random.default_rng(seed)
    prompt = SINK + (KW + QW) * OMEGA + LOCAL
    st = OracleStickyLayer(H, D, OMEGA, SINK, LOCAL, KW, QW, "bf16", 8, max_windows=640, max_context=8192)
    Kp = rnd(rng.standard_normal((H, prompt, D), dtype=np.float32), "bf16")
    Vp = rnd(rng.standard_normal((H, prompt, D), dtype=np.float32), "bf16")
    cs = rng.random((H, 1, prompt), dtype=np.float32) * 4
    K, V = st.prefill(Kp, Vp, cs, "fp32")
    pool = concurrent.futures.ThreadPoolExecutor(max_workers=threads) if threads > 1 else None
    times = []
    for _ in range(steps):
        q = rnd(rng.standard_normal((H * G, D), dtype=np.float32) * 0.3, "bf16")
        kn = rnd(rng.standard_normal((H, D), dtype=np.float32), "bf16")
        vn = rnd(rng.standard_normal((H, D), dtype=np.float32), "bf16")
        t0 = time.perf_counter()
        K = np.concatenate([K, kn[:, None]], 1)
        V = np.concatenate([V, vn[:, None]], 1)
        qc = None if st.q is None else {k: st.q[k] for k in ("kq", "ks", "kz", "vq", "vs", "vz")}
        if pool is None:
            _, sc, qsc = decode_attention(q, K, V, "bf16", qc)
        else:
            def head(h):
                qh = None if qc is None else {k: v[h:h + 1] for k, v in qc.items()}
                return decode_attention(q[h * G:(h + 1) * G], K[h:h + 1], V[h:h + 1], "bf16", qh)
            res = list(pool.map(head, range(H)))
            sc = np.concatenate([r[1] for r in res], 0)
            qsc = None if qc is None else np.concatenate([r[2] for r in res], 0)
        K, V = st.decode(K, V, sc, qsc, "bf16")
        times.append(time.perf_counter() - t0)
    return float(np.mean(times))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("reference")
    ap.add_argument("--steps", type=int, default=128)
    a = ap.parse_args()
    ref_s, threads = time_reference(a.reference, a.steps)
    port1_s = time_port(a.steps)
    portn_s = time_port(a.steps, threads=min(8, os.cpu_count() or 1))
    res = {"work": (f"one decode token of one layer at the full-model workload's shape (bf16, {H} KV heads, group "
                    f"{G}, head_dim {D}, omega {OMEGA}, sink {SINK}, local {LOCAL}, {KW} sticky + {QW} INT8 Q "
                    f"windows), append + logits + joint softmax + ledger + an eviction cycle every {OMEGA} tokens, "
                    f"mean over {a.steps} tokens"),
           "reference_ms_per_layer_step": ref_s * 1e3, "reference_threads": threads,
           "port_ms_per_layer_step": port1_s * 1e3, "port_threads": 1,
           "port_heads_threaded_ms_per_layer_step": portn_s * 1e3,
           "port_heads_threaded_threads": min(8, os.cpu_count() or 1),
           "port_over_reference": portn_s / ref_s,
           "port_over_reference_note": "threaded port (as the benchmark's host arm runs it) / reference",
           "host": f"{platform.processor() or platform.machine()}, {os.cpu_count()} cores"}
    with open(os.path.join(HERE, "port_vs_reference.json"), "w") as f:
        json.dump(res, f, indent=1)
    print(json.dumps(res))


if __name__ == "__main__":
    main()
