"""Generate golden vectors by running the reference implementation itself.

Run where a checkout of the reference is available; its path is the first
argument or the QEVICT_REFERENCE environment variable (there is no default).
The reference is imported read-only, with the harness patches it needs on
current libraries:

  * ``sticky_config`` knobs (OMEGA, SINK_TOKENS, QUANTIZATION_BIT_WIDTH,
    LOCAL_NUM_TOKENS) set before construction (read at cache.py:66-119);
  * ``compute_budget`` replaced by a fixed BudgetResult so the window counts
    are exact (called at cache.py:274-287);
  * ``config.rope_parameters`` set for transformers 5.x (rope.py:223-237);
  * ``layer_idx != 0`` so the layer-0 debug prints stay silent.

Each scenario records its seeded inputs and the reference's outputs into
``tests/golden/<name>.npz``; ``tests/test_oracle_golden.py`` replays the inputs
through the oracle and compares.  Fixtures are small (sub-MB).

    python tests/golden/make_golden.py <reference checkout> [scenario ...]

Scenarios: codec attention state module prefill budget tracking module_c1
(default: all but module_c1, which takes about a minute and ~10 GB of RAM).
"""

import os
import sys

import numpy as np

_ARGS = [a for a in sys.argv[1:] if not a.startswith("-")]
REF = _ARGS.pop(0) if _ARGS and os.path.isdir(_ARGS[0]) else os.environ.get("QEVICT_REFERENCE")
if not REF or not os.path.isdir(REF):
    sys.exit("usage: make_golden.py <reference checkout> [scenario ...]  (or set QEVICT_REFERENCE)")
OUT = os.path.dirname(os.path.abspath(__file__))
sys.dont_write_bytecode = True
sys.path.insert(0, OUT)
sys.path.insert(0, REF)
sys.path.insert(0, os.path.join(REF, "src"))

import torch  # noqa: E402

import src.sticky_config as sticky_config  # noqa: E402
import src.models.kv_cache.cache as ref_cache_mod  # noqa: E402
from src.models.kv_cache.allocator import BudgetResult  # noqa: E402
from src.models.kv_cache import quantize as ref_q  # noqa: E402
from src.models.attention import ops as ref_ops  # noqa: E402
from c1_inputs import C1, c1_inputs  # noqa: E402

TD = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def f32(t):
    return t.detach().to(torch.float32).cpu().numpy()


def save(name, **arrays):
    path = os.path.join(OUT, name + ".npz")
    np.savez_compressed(path, **arrays)
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.1f} KiB)")


def configure(omega, sink, local, k_windows, q_windows, bits=8):
    sticky_config.OMEGA = omega
    sticky_config.SINK_TOKENS = sink
    sticky_config.QUANTIZATION_BIT_WIDTH = bits
    sticky_config.LOCAL_NUM_TOKENS = local
    qbl = 0  # unused by the coordinator beyond storage

    def fixed_budget(**kw):
        return BudgetResult(local_num=local, k_windows=k_windows, q_windows_count=q_windows,
                            q_num=qbl, quant_bytes_len=kw.get("head_dim", 0))

    ref_cache_mod.compute_budget = fixed_budget


def make_config(hidden, heads, kv_heads, max_pos=4096):
    from src.models.configuration_sticky_llama import LlamaConfig
    cfg = LlamaConfig(hidden_size=hidden, num_attention_heads=heads, num_key_value_heads=kv_heads,
                      max_position_embeddings=max_pos, intermediate_size=2 * hidden,
                      num_hidden_layers=2)
    cfg.rope_parameters = {"rope_type": "default", "rope_theta": 500000.0}
    return cfg


# ---------------------------------------------------------------------------
# 1. codec
# ---------------------------------------------------------------------------
def gen_codec():
    g = torch.Generator().manual_seed(1)
    out = {}
    for dt in ("fp32", "bf16", "fp16"):
        x = torch.randn(2, 3, 16, 32, generator=g) * 2.0
        x[0, 1] = 0.0          # all-zero window (the zero-filled challenger case)
        x[1, 2] = 0.75         # constant window
        x[1, 0, :, 5] = 3.0    # constant channel
        x = x.to(TD[dt])
        for bits in (8, 4):
            kq, ks, kz = ref_q.quantize_k_per_window(x, bits)
            vq, vs, vz = ref_q.quantize_v_per_window(x, bits)
            kd = ref_q.dequantize_from_quant(kq, ks, kz, bits)
            vd = ref_q.dequantize_from_quant(vq, vs, vz, bits)
            p = f"{dt}_b{bits}_"
            out[p + "x"] = f32(x)
            out[p + "kq"], out[p + "ks"], out[p + "kz"] = kq.numpy(), f32(ks), f32(kz)
            out[p + "vq"], out[p + "vs"], out[p + "vz"] = vq.numpy(), f32(vs), f32(vz)
            out[p + "kd"], out[p + "vd"] = f32(kd), f32(vd)
    # one full-width window at the production head_dim
    x = (torch.randn(1, 1, 64, 128, generator=g) * 1.5).to(torch.bfloat16)
    kq, ks, kz = ref_q.quantize_k_per_window(x, 8)
    vq, vs, vz = ref_q.quantize_v_per_window(x, 8)
    out["d128_x"], out["d128_kq"], out["d128_ks"], out["d128_kz"] = f32(x), kq.numpy(), f32(ks), f32(kz)
    out["d128_vq"], out["d128_vs"], out["d128_vz"] = vq.numpy(), f32(vs), f32(vz)
    save("codec", **out)


# ---------------------------------------------------------------------------
# 2. decode attention ops
# ---------------------------------------------------------------------------
class _QView:
    """Duck-typed stand-in for the cache object that ops.py reads (ops.py:99-110)."""

    def __init__(self, kq, ks, kz, vq, vs, vz, bits):
        self.q_cache_k_quant, self.q_cache_k_scale, self.q_cache_k_zp = kq, ks, kz
        self.q_cache_v_quant, self.q_cache_v_scale, self.q_cache_v_zp = vq, vs, vz
        self.quant_bit_width = bits

    @staticmethod
    def _dequantize_from_quant(q, s, z, bits=8):
        return ref_q.dequantize_from_quant(q, s, z, bits)


def gen_attention():
    g = torch.Generator().manual_seed(2)
    out = {}
    H, G, D, S, W, om = 2, 4, 32, 80, 3, 16
    for dt in ("fp32", "bf16", "fp16"):
        td = TD[dt]
        q = (torch.randn(1, H * G, 1, D, generator=g)).to(td)
        k = (torch.randn(1, H, S, D, generator=g)).to(td)
        v = (torch.randn(1, H, S, D, generator=g)).to(td)
        kw = (torch.randn(H, W, om, D, generator=g)).to(td)
        vw = (torch.randn(H, W, om, D, generator=g)).to(td)
        kq, ks, kz = ref_q.quantize_k_per_window(kw, 8)
        vq, vs, vz = ref_q.quantize_v_per_window(vw, 8)
        kvc = _QView(kq, ks, kz, vq, vs, vz, 8)
        logits = ref_ops.compute_main_logits(q, k, 1, H * G, H, G, 1, D)
        mask = torch.zeros(1, 1, 1, S, dtype=td)
        logits = logits + mask
        o, sc, qs, _ = ref_ops.compute_qcache_joint_softmax(q, logits, v, kvc, 1, H * G, H, G, 1, D)
        o2, sc2, _ = ref_ops.compute_standard_softmax(q, logits, v, 1, H * G, H, G, 1, D)
        p = dt + "_"
        out[p + "q"], out[p + "k"], out[p + "v"] = f32(q), f32(k), f32(v)
        out[p + "kq"], out[p + "ks"], out[p + "kz"] = kq.numpy(), f32(ks), f32(kz)
        out[p + "vq"], out[p + "vs"], out[p + "vz"] = vq.numpy(), f32(vs), f32(vz)
        out[p + "out"], out[p + "scores"], out[p + "qscores"] = f32(o), f32(sc), f32(qs)
        out[p + "out_noq"], out[p + "scores_noq"] = f32(o2), f32(sc2)
    save("attention", **out)


# ---------------------------------------------------------------------------
# 3. cache state machine driven with explicit scores (forced churn)
# ---------------------------------------------------------------------------
def gen_state(name, dt, attn_kind, seed, H=2, D=16, omega=16, sink=8, local=32,
              k_windows=3, q_windows=4, prompt=200, steps=96, bits=8, tracking=False):
    configure(omega, sink, local, k_windows, q_windows, bits)
    cfg = make_config(hidden=4 * D, heads=4, kv_heads=H)
    from src.models.kv_cache.cache import STICKYKVCache_LayerWise
    # the research token ledger is on when sticky_config.tracking_flag == 1 (cache.py:112-119)
    sticky_config.tracking_flag = 1 if tracking else 0
    cache = STICKYKVCache_LayerWise(p_ratio=50, r_ratio=20, start_idx=0, num_heads=H,
                                    layer_idx=1, config=cfg)
    sticky_config.tracking_flag = 0
    rows = prompt + steps + 8

    def track(rec, p):
        if tracking:
            rec[p + "trk_ledger"] = cache.token_ledger[:rows].numpy().copy()
            rec[p + "trk_hist"] = cache.global_score_history[:rows].numpy().copy()
            rec[p + "trk_counter"] = np.array(int(cache.global_token_counter))
    td = TD[dt]
    g = torch.Generator().manual_seed(seed)
    K = torch.randn(1, H, prompt, D, generator=g).to(td)
    V = torch.randn(1, H, prompt, D, generator=g).to(td)
    if attn_kind == "sdpa":
        a = torch.rand(1, H, prompt, prompt, generator=g)
        a = torch.tril(a)
        attn = (a / a.sum(-1, keepdim=True)).to(td)
        attn_dt = dt
    else:
        attn = torch.rand(1, H, 1, prompt, generator=g) * 10.0
        attn_dt = "fp32"
    rec = dict(K0=f32(K), V0=f32(V), attn=f32(attn), attn_dt=np.array(attn_dt),
               dt=np.array(dt), params=np.array([H, D, omega, sink, local, k_windows, q_windows,
                                                   prompt, steps, bits, cache.eviction_manager.window_scores.shape[1]]))
    kv = cache((K, V), attn, q_len=prompt)
    rec["pre_K"], rec["pre_V"] = f32(kv[0]), f32(kv[1])
    track(rec, "pre_")
    ws0 = cache.window_scores[:, :, 0]
    big = float(torch.nan_to_num(ws0, nan=0.0).max())
    rec["pre_ws"] = cache.window_scores.numpy().copy()
    rec["pre_lh"] = cache.eviction_manager.local_history.numpy().copy()
    rec["pre_lid"] = cache.eviction_manager.logical_id_map.numpy().copy()
    if cache.q_cache_ids is not None:
        rec["pre_qids"] = cache.q_cache_ids.numpy().copy()
        rec["pre_qkq"] = cache.q_cache_k_quant.numpy().copy()
        rec["pre_qks"] = f32(cache.q_cache_k_scale)
        rec["pre_qvs"] = f32(cache.q_cache_v_scale)
    cyc = 0
    newk, newv, scs, qss, qsn = [], [], [], [], []
    for step in range(steps):
        kn = torch.randn(1, H, 1, D, generator=g).to(td)
        vn = torch.randn(1, H, 1, D, generator=g).to(td)
        Kc = torch.cat([kv[0], kn], dim=2)
        Vc = torch.cat([kv[1], vn], dim=2)
        S = Kc.shape[2]
        sc = torch.rand(1, H, 1, S, generator=g) * 1e-3
        qids = cache.q_cache_ids
        # planted churn: once per cycle each head gets a large vote on a random
        # main-zone token (sticky or local window) and on a random Q-cache token,
        # sized like the prefill window scores, so windows are promoted/demoted
        if step % omega == omega // 2:
            for h in range(H):
                hot = int(torch.randint(sink, S, (1,), generator=g))
                sc[0, h, 0, hot] += float(torch.rand(1, generator=g)) * 2.0 * big
        sc = sc.to(td)
        if qids is not None:
            qsc = torch.rand(1, H, 1, qids.shape[1] * omega, generator=g) * 1e-3
            if step % omega == omega // 2:
                for h in range(H):
                    j = int(torch.randint(0, qids.shape[1] * omega, (1,), generator=g))
                    qsc[0, h, 0, j] += float(torch.rand(1, generator=g)) * 2.0 * big
            qsc = qsc.to(td)
            qss.append(np.pad(f32(qsc)[0, :, 0], ((0, 0), (0, q_windows * omega - qsc.shape[-1]))))
            qsn.append(qsc.shape[-1])
        else:
            qsc = None
            qss.append(np.zeros((H, q_windows * omega), np.float32))
            qsn.append(-1)
        newk.append(f32(kn)[0, :, 0]); newv.append(f32(vn)[0, :, 0])
        scs.append(np.pad(f32(sc)[0, :, 0], ((0, 0), (0, 1024 - S))))
        kv = cache((Kc, Vc), sc, q_len=1, q_attn_scores=qsc)
        if cache.eviction_manager.tokens_since_last_review == 0:
            p = f"c{cyc}_"
            rec[p + "step"] = np.array(step)
            rec[p + "K"], rec[p + "V"] = f32(kv[0]), f32(kv[1])
            rec[p + "ws"] = cache.window_scores.numpy()[:, :k_windows].copy()
            rec[p + "lh"] = cache.eviction_manager.local_history.numpy().copy()
            rec[p + "lid"] = cache.eviction_manager.logical_id_map.numpy().copy()
            if cache.q_cache_ids is not None:
                rec[p + "qids"] = cache.q_cache_ids.numpy().copy()
                rec[p + "qsc"] = cache.q_cache_scores.numpy().copy()
                rec[p + "qkq"] = cache.q_cache_k_quant.numpy().copy()
                rec[p + "qvq"] = cache.q_cache_v_quant.numpy().copy()
                rec[p + "qks"], rec[p + "qkz"] = f32(cache.q_cache_k_scale), f32(cache.q_cache_k_zp)
                rec[p + "qvs"], rec[p + "qvz"] = f32(cache.q_cache_v_scale), f32(cache.q_cache_v_zp)
            rec[p + "meta"] = np.array(sorted([list(k) for k in cache.quantization_manager.q_retired_meta.keys()]) or np.zeros((0, 2)), dtype=np.int64)
            track(rec, p)
            cyc += 1
    rec["newk"], rec["newv"] = np.stack(newk), np.stack(newv)
    rec["scores"], rec["qscores"], rec["qscores_n"] = np.stack(scs), np.stack(qss), np.array(qsn)
    rec["n_cycles"] = np.array(cyc)
    rec["final_K"], rec["final_V"] = f32(kv[0]), f32(kv[1])
    track(rec, "final_")
    save(name, **rec)


# ---------------------------------------------------------------------------
# 4. whole attention module (prefill + decode), fp32 and bf16
# ---------------------------------------------------------------------------
def gen_module(name, dt, seed, prompt=200, steps=40):
    configure(16, 8, 32, 3, 4, 8)
    cfg = make_config(hidden=64, heads=4, kv_heads=2)
    from src.models.attention.module import STICKYLlamaAttention
    from transformers import DynamicCache
    torch.manual_seed(seed)
    m = STICKYLlamaAttention(cfg, 1)
    with torch.no_grad():
        for lin in (m.q_proj, m.k_proj, m.v_proj, m.o_proj):
            lin.weight.normal_(0.0, 0.2)
    m = m.to(TD[dt])
    g = torch.Generator().manual_seed(seed + 1)
    hs = torch.randn(1, prompt, 64, generator=g).to(TD[dt])
    dec = torch.randn(steps, 1, 1, 64, generator=g).to(TD[dt])
    c = DynamicCache()
    with torch.no_grad():
        o_pre, _ = m(hs, past_key_values=c, use_cache=True)
        outs = []
        for i in range(steps):
            o, _ = m(dec[i], past_key_values=c, use_cache=True)
            outs.append(f32(o)[0, 0])
    save(name, wq=f32(m.q_proj.weight), wk=f32(m.k_proj.weight), wv=f32(m.v_proj.weight),
         wo=f32(m.o_proj.weight), hs=f32(hs), dec=f32(dec), out_pre=f32(o_pre), outs=np.stack(outs),
         dt=np.array(dt), final_K=f32(c.layers[1].keys), final_V=f32(c.layers[1].values),
         qids=m.kv_cache.q_cache_ids.numpy() if m.kv_cache.q_cache_ids is not None else np.zeros((0,)),
         ws=m.kv_cache.window_scores.numpy()[:, :3].copy())


# ---------------------------------------------------------------------------
# 5. prefill lane: chunked column sums (FA path) and SDPA causal output
# ---------------------------------------------------------------------------
def gen_prefill():
    sys.modules.setdefault("flash_attn", type(sys)("flash_attn"))
    if not hasattr(sys.modules["flash_attn"], "flash_attn_func"):
        sys.modules["flash_attn"].flash_attn_func = None  # only the pure-torch scorer is used
    from src.models.attention.ops_flash import compute_chunked_prefill_scores
    g = torch.Generator().manual_seed(5)
    out = {}
    Hq, H, S, D = 8, 2, 530, 16
    for dt in ("fp32", "bf16"):
        td = TD[dt]
        q = torch.randn(1, Hq, S, D, generator=g).to(td)
        k = torch.randn(1, H, S, D, generator=g).to(td)
        v = torch.randn(1, H, S, D, generator=g).to(td)
        cs = compute_chunked_prefill_scores(q, k, S, 0, H, Hq, Hq // H, D)
        lg = ref_ops.compute_main_logits(q, k, 1, Hq, H, Hq // H, S, D)
        ref_ops.apply_prefill_causal_mask(lg, S, 0)
        o, _, _ = ref_ops.compute_standard_softmax(q, lg, v, 1, Hq, H, Hq // H, S, D)
        p = dt + "_"
        out[p + "q"], out[p + "k"], out[p + "v"] = f32(q), f32(k), f32(v)
        out[p + "colsum"], out[p + "out"] = f32(cs), f32(o)
    save("prefill", **out)


# ---------------------------------------------------------------------------
# 6. budget allocator over a grid of prompt lengths and ratios
# ---------------------------------------------------------------------------
def gen_budget():
    import contextlib
    import io
    from src.models.kv_cache.allocator import compute_budget as ref_budget
    rows, outs = [], []
    for new_tokens in (100, 1000, 4096, 32768, 131072):
        for r in (5, 20, 50, 100):
            for fixed, local in ((True, 512), (True, 256), (False, 0)):
                for q_ratio in (0, 10, 50):
                    for bits in (8, 4):
                        for omega in (16, 64):
                            args = dict(total_cache_ratio=r, sink_tokens=64, use_fixed_local_tokens=fixed,
                                        local_num_tokens=local, local_cache_ratio=50, q_ratio=q_ratio,
                                        quant_bit_width=bits, head_dim=128, omega=omega,
                                        new_tokens=new_tokens, max_tokens=512, layer_idx=1)
                            with contextlib.redirect_stdout(io.StringIO()):
                                res = ref_budget(**args)
                            rows.append([new_tokens, r, int(fixed), local, q_ratio, bits, omega])
                            outs.append([res.local_num, res.k_windows, res.q_windows_count, res.q_num,
                                         res.quant_bytes_len])
    save("budget", inputs=np.array(rows, np.int64), outputs=np.array(outs, np.int64))


# ---------------------------------------------------------------------------
# 7. research token ledger, operation by operation (tracking_manager.py:27-204)
# ---------------------------------------------------------------------------
def gen_tracking_ops(H=3, C=64, prompt=40, keep=28, steps=30, cycles=(10, 20), layer_idx=5):
    """TrackingManager driven directly, with the edge cases its callers can
    produce: score rows shorter than the physical cache (positions out of
    range), evicted tokens (votes added once more), and a ledger smaller than
    the token count (rows past max_context are dropped)."""
    from src.models.kv_cache.tracking_manager import TrackingManager
    g = torch.Generator().manual_seed(41)
    tm = TrackingManager(C, H, torch.device("cpu"))
    rec = {"params": np.array([H, C, prompt, keep, steps, layer_idx])}
    snaps_l, snaps_h = [], []

    def snap():
        snaps_l.append(tm.token_ledger.numpy().copy())
        snaps_h.append(tm._global_score_history.numpy().copy())

    attn = torch.rand(1, H, 1, prompt, generator=g) * 5.0
    surv = torch.stack([torch.sort(torch.randperm(prompt, generator=g)[:keep]).values for _ in range(H)])
    tm.increment(n=prompt)
    tm.record_prefill(seq_len=prompt, q_len=prompt, layer_idx=layer_idx, attn_score_cache=attn,
                      survivor_ids=surv, full_attn_scores=None, global_start=0, num_new_tokens=prompt)
    snap()
    rec["attn"], rec["surv"] = f32(attn), surv.numpy()
    phys_len = keep
    scs, kvs, lens, maps, votes = [], [], [], [], []
    for step in range(steps):
        gs = int(tm.global_token_counter)
        tm.increment(n=1)
        phys_len += 1
        kv = phys_len - 2 if step % 7 == 3 else phys_len
        sc = torch.rand(1, H, 1, kv, generator=g)
        tm.record_decode(sc, phys_len, layer_idx, gs)
        snap()
        scs.append(np.pad(f32(sc)[0, :, 0], ((0, 0), (0, 128 - kv))))
        kvs.append(kv)
        lens.append(phys_len)
        if step in cycles:
            kept = torch.rand(H, phys_len, generator=g) < 0.7
            mp = torch.full((H, phys_len), -1.0)
            n_new = int(kept.sum(dim=1).min())
            for h in range(H):
                idx = torch.nonzero(kept[h]).flatten()[:n_new]
                mp[h, idx] = torch.randperm(n_new, generator=g).float()
            vt = torch.rand(H, C, generator=g) * 3.0
            tm.update_physical_positions(mp, phys_len, vt)
            snap()
            maps.append(np.pad(mp.numpy(), ((0, 0), (0, 128 - phys_len)), constant_values=-1.0))
            votes.append(vt.numpy())
            phys_len = n_new
    rec["scores"], rec["kv"], rec["seq_len"] = np.stack(scs), np.array(kvs), np.array(lens)
    rec["cycles"], rec["mapping"], rec["votes"] = np.array(cycles), np.stack(maps), np.stack(votes)
    rec["ledger"], rec["hist"] = np.stack(snaps_l), np.stack(snaps_h)
    rec["counter"] = np.array(int(tm.global_token_counter))
    save("tracking_ops", **rec)




# ---------------------------------------------------------------------------
# 8. the single-layer fp32 workload at full shape (one Llama attention layer)
# ---------------------------------------------------------------------------
def gen_module_c1(c=C1):
    """The reference's STICKYLlamaAttention at the fp32 single-layer workload's
    full shape: 32 query / 8 KV heads, head_dim 128, RoPE theta 500000, a
    4096-token prompt and 256 decode steps, omega 64, sink 64, local 256, 16
    sticky + 16 INT8 Q windows (SDPA path, sticky_config.USE_FLASH_ATTENTION=0).
    Records the prefill output at every 128th position, every decode output's
    first 1024 elements (and whole-vector sums), the window sets after the
    prefill and after each of the four eviction cycles, and the final Q-cache
    scales / zero points and code checksums."""
    configure(c["omega"], c["sink"], c["local"], c["k_windows"], c["q_windows"], 8)
    cfg = make_config(hidden=c["hidden"], heads=c["heads"], kv_heads=c["kv_heads"],
                      max_pos=c["prompt"] + c["steps"] + 64)
    from src.models.attention.module import STICKYLlamaAttention
    from transformers import DynamicCache
    w, hs, dec = c1_inputs(c)
    m = STICKYLlamaAttention(cfg, 1)
    with torch.no_grad():
        for lin, name in ((m.q_proj, "q"), (m.k_proj, "k"), (m.v_proj, "v"), (m.o_proj, "o")):
            lin.weight.copy_(torch.from_numpy(w[name]))
    cache = DynamicCache()
    kc = m.kv_cache
    em = kc.eviction_manager
    kw = c["k_windows"]

    def windows():
        ids = em.window_scores[:, :kw, 1].numpy().copy()
        qids = kc.q_cache_ids.numpy().copy() if kc.q_cache_ids is not None else np.zeros((0,), np.float32)
        return ids, qids

    rec = {}
    with torch.no_grad():
        o_pre, _ = m(torch.from_numpy(hs)[None], past_key_values=cache, use_cache=True)
        o_pre = f32(o_pre)[0]
        rec["pre_rows"] = np.arange(0, c["prompt"], 128)
        rec["out_pre"] = o_pre[rec["pre_rows"]]
        rec["out_pre_rowsum"] = o_pre.astype(np.float64).sum(axis=1)
        ids, qids = windows()
        sticky, qsets, cyc_steps = [ids], [qids], [-1]
        outs = []
        for i in range(c["steps"]):
            o, _ = m(torch.from_numpy(dec[i])[None, None], past_key_values=cache, use_cache=True)
            outs.append(f32(o)[0, 0])
            if em.tokens_since_last_review == 0:
                ids, qids = windows()
                sticky.append(ids)
                qsets.append(qids)
                cyc_steps.append(i)
    outs = np.stack(outs)
    rec["out_dec"] = outs[:, :1024]
    rec["out_dec_sum"] = outs.astype(np.float64).sum(axis=1)
    rec["out_dec_abssum"] = np.abs(outs.astype(np.float64)).sum(axis=1)
    rec["sticky_ids"] = np.stack(sticky)
    rec["q_ids"] = np.stack(qsets)
    rec["cycle_steps"] = np.array(cyc_steps)
    rec["q_ks"], rec["q_kz"] = f32(kc.q_cache_k_scale), f32(kc.q_cache_k_zp)
    rec["q_vs"], rec["q_vz"] = f32(kc.q_cache_v_scale), f32(kc.q_cache_v_zp)
    kq, vq = kc.q_cache_k_quant.numpy(), kc.q_cache_v_quant.numpy()
    rec["q_kq_sum"] = kq.astype(np.int64).sum(axis=(2, 3))
    rec["q_vq_sum"] = vq.astype(np.int64).sum(axis=(2, 3))
    rec["q_kq_w0"], rec["q_vq_w0"] = kq[:, 0].copy(), vq[:, 0].copy()
    rec["global_token_counter"] = np.array(int(kc.global_token_counter))
    rec["config"] = np.array([c[k] for k in ("hidden", "heads", "kv_heads", "omega", "sink", "local",
                                             "k_windows", "q_windows", "prompt", "steps", "seed")])
    save("module_c1_fp32", **rec)


SCENARIOS = {
    "codec": lambda: gen_codec(),
    "attention": lambda: gen_attention(),
    "state": lambda: (gen_state("state_bf16_sdpa", "bf16", "sdpa", seed=11),
                      gen_state("state_fp32_fa", "fp32", "fa", seed=12),
                      gen_state("state_fp16_fa", "fp16", "fa", seed=13)),
    "module": lambda: (gen_module("module_fp32", "fp32", seed=21), gen_module("module_bf16", "bf16", seed=22)),
    "prefill": lambda: gen_prefill(),
    "budget": lambda: gen_budget(),
    "tracking": lambda: (gen_state("tracking_fp32_fa", "fp32", "fa", seed=31, tracking=True), gen_tracking_ops()),
    "module_c1": lambda: gen_module_c1(),
}


if __name__ == "__main__":
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    for name in (_ARGS or [k for k in SCENARIOS if k != "module_c1"]):
        SCENARIOS[name]()
