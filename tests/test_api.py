"""The reference-facing API: compute_budget, STICKYKVCache_LayerWise, STICKYLlamaAttention.

* ``compute_budget`` against the reference's own allocator outputs
  (tests/golden/budget.npz, made by tests/golden/make_golden.py) -- CPU.
* ``STICKYKVCache_LayerWise`` driven the way the reference's attention module
  drives it (the caller computes attention and passes the probabilities):
  every returned physical cache, window set and Q-cache must equal the
  oracle's bit for bit, fed the same probabilities -- GPU.
* ``STICKYLlamaAttention`` (fused kernels) against the oracle replaying the
  same module: prefill and decode outputs within tolerance, the same windows.
"""

import os
from types import SimpleNamespace

import numpy as np
import pytest

from qevict_b200.allocator import compute_budget

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_compute_budget_matches_reference():
    z = np.load(os.path.join(GOLDEN, "budget.npz"))
    for row, out in zip(z["inputs"], z["outputs"]):
        new_tokens, r, fixed, local, q_ratio, bits, omega = (int(x) for x in row)
        res = compute_budget(total_cache_ratio=r, sink_tokens=64, use_fixed_local_tokens=bool(fixed),
                             local_num_tokens=local, local_cache_ratio=50, q_ratio=q_ratio, quant_bit_width=bits,
                             head_dim=128, omega=omega, new_tokens=new_tokens, max_tokens=512, layer_idx=1)
        assert list(res) == [int(x) for x in out], (row, res, out)


def test_compute_budget_warns_without_sticky_windows(capsys):
    res = compute_budget(5, 64, True, 512, 50, 10, 8, 128, 64, 100, 512, 3)
    assert res.k_windows == 0
    assert "k_windows=0" in capsys.readouterr().out


# ----------------------------------------------------------------------------- GPU
@pytest.fixture()
def knobs():
    """Set the sticky_config knobs for one test and restore them afterwards."""
    from qevict_b200 import sticky_config as sc
    saved = {k: getattr(sc, k) for k in ("OMEGA", "SINK_TOKENS", "LOCAL_NUM_TOKENS", "Q_RATIO",
                                         "QUANTIZATION_BIT_WIDTH", "GENERATION_CONFIG", "P_RATIO")}

    def set_(**kw):
        for k, v in kw.items():
            setattr(sc, k, v)
    yield set_
    for k, v in saved.items():
        setattr(sc, k, v)


def _cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch


@pytest.mark.gpu
def test_cache_object_with_caller_scores_matches_oracle(knobs):
    torch = _cuda()
    from oracle.attention import decode_attention
    from oracle.sticky_state import OracleStickyLayer
    from qevict_b200.kv_cache import STICKYKVCache_LayerWise
    H, G, D, om, sink, local, steps = 2, 2, 64, 16, 16, 32, 100
    knobs(OMEGA=om, SINK_TOKENS=sink, LOCAL_NUM_TOKENS=local, Q_RATIO=40, QUANTIZATION_BIT_WIDTH=8,
          GENERATION_CONFIG={"max_new_tokens": steps})
    cfg = SimpleNamespace(hidden_size=H * G * D, num_attention_heads=H * G, num_key_value_heads=H,
                          max_position_embeddings=4096)
    cache = STICKYKVCache_LayerWise(50, 30, 0, H, 1, cfg)
    rng = np.random.default_rng(7)
    S = sink + 20 * om
    K = rng.standard_normal((1, H, S, D)).astype(np.float32)
    V = rng.standard_normal((1, H, S, D)).astype(np.float32)
    cs = (rng.random((1, H, 1, S)) * 3).astype(np.float32)
    dev = torch.device("cuda")
    Kg, Vg = cache((torch.tensor(K, device=dev), torch.tensor(V, device=dev)), torch.tensor(cs, device=dev))
    o = OracleStickyLayer(H, D, om, sink, cache.local_num, cache.k_windows, cache.q_windows_count, "fp32", 8,
                          max_windows=cache.max_windows, max_context=4096, r_ratio=30, window_sum="tree")
    Ko, Vo = o.prefill(K[0], V[0], cs[0], "fp32")
    assert cache.k_windows > 0 and cache.q_windows_count > 0
    np.testing.assert_array_equal(Kg[0].cpu().numpy(), Ko)
    np.testing.assert_array_equal(Vg[0].cpu().numpy(), Vo)
    cycles = 0
    for step in range(steps):
        q = (rng.standard_normal((H * G, D)) * 0.5).astype(np.float32)
        kn = rng.standard_normal((H, 1, D)).astype(np.float32)
        vn = rng.standard_normal((H, 1, D)).astype(np.float32)
        Kc, Vc = np.concatenate([Ko, kn], 1), np.concatenate([Vo, vn], 1)
        qc = None if o.q is None else {k: o.q[k] for k in ("kq", "ks", "kz", "vq", "vs", "vz")}
        _, scm, scq = decode_attention(q, Kc, Vc, "fp32", qc)
        sc_t = torch.tensor(scm[None, :, None, :], device=dev)
        qs_t = None if scq is None else torch.tensor(scq[None, :, None, :], device=dev)
        Kg, Vg = cache((torch.cat([Kg, torch.tensor(kn[None], device=dev)], 2),
                        torch.cat([Vg, torch.tensor(vn[None], device=dev)], 2)), sc_t, q_attn_scores=qs_t)
        due = o.tokens_since + 1 == om
        Ko, Vo = o.decode(Kc, Vc, scm, scq, "fp32")
        np.testing.assert_array_equal(Kg[0].cpu().numpy(), Ko, err_msg=f"step {step}")
        np.testing.assert_array_equal(Vg[0].cpu().numpy(), Vo, err_msg=f"step {step}")
        if due:
            cycles += 1
            ws = cache.window_scores
            np.testing.assert_array_equal(ws[:, :cache.k_windows, 1].numpy(), o.window_scores[:, :cache.k_windows, 1])
            np.testing.assert_array_equal(cache.q_cache_ids.numpy(), o.q["ids"])
            np.testing.assert_array_equal(cache.q_cache_k_quant.numpy(), o.q["kq"])
            np.testing.assert_array_equal(cache.q_cache_v_quant.numpy(), o.q["vq"])
    assert cycles == steps // om
    assert int(cache.global_token_counter) == S + steps
    assert cache.state.read_error() == 0


@pytest.mark.gpu
def test_attention_module_matches_oracle(knobs):
    torch = _cuda()
    from oracle.attention import decode_attention
    from oracle.prefill import causal_attention, chunked_prefill_scores
    from oracle.sticky_state import OracleStickyLayer, apply_rope, rope_cos_sin
    from qevict_b200.attention import STICKYLlamaAttention
    Hq, H, D, om, sink, local, steps = 4, 2, 64, 16, 16, 32, 70
    knobs(OMEGA=om, SINK_TOKENS=sink, LOCAL_NUM_TOKENS=local, Q_RATIO=40, QUANTIZATION_BIT_WIDTH=8,
          GENERATION_CONFIG={"max_new_tokens": steps})
    cfg = SimpleNamespace(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=H,
                          max_position_embeddings=2048, rope_theta=500000.0, r_ratio=30, p_ratio=50, start_idx=0)
    torch.manual_seed(3)
    m = STICKYLlamaAttention(cfg, 1).cuda()
    with torch.no_grad():
        for lin in (m.q_proj, m.k_proj, m.v_proj, m.o_proj):
            lin.weight.normal_(0.0, 0.06)
    S = sink + 20 * om
    g = torch.Generator(device="cuda").manual_seed(4)
    hs = torch.randn(1, S, Hq * D, generator=g, device="cuda")
    dec = torch.randn(steps, 1, 1, Hq * D, generator=g, device="cuda")
    with torch.no_grad():
        out_pre, _ = m(hs, use_cache=True)
        # the oracle sees the module's own projections (same cuBLAS calls)
        W = {n: getattr(m, n).weight for n in ("q_proj", "k_proj", "v_proj", "o_proj")}

        def proj(x, n):
            return (x @ W[n].t()).double().cpu().numpy().astype(np.float32)
        q = proj(hs[0], "q_proj").reshape(S, Hq, D).transpose(1, 0, 2)
        k = proj(hs[0], "k_proj").reshape(S, H, D).transpose(1, 0, 2)
        v = proj(hs[0], "v_proj").reshape(S, H, D).transpose(1, 0, 2)
        cos, sin = rope_cos_sin(np.arange(S), D, 500000.0, "fp32")
        q, k = apply_rope(q, cos, sin, "fp32"), apply_rope(k, cos, sin, "fp32")
        o_att = causal_attention(q, k, v, "fp32")
        ref_pre = o_att.transpose(1, 0, 2).reshape(S, Hq * D) @ W["o_proj"].double().cpu().numpy().T
        np.testing.assert_allclose(out_pre[0].double().cpu().numpy(), ref_pre, atol=2e-4, rtol=1e-3)
        cs = chunked_prefill_scores(q, k, "fp32")
        kc = m.kv_cache
        o = OracleStickyLayer(H, D, om, sink, kc.local_num, kc.k_windows, kc.q_windows_count, "fp32", 8,
                              max_windows=kc.max_windows, max_context=2048, r_ratio=30, window_sum="tree")
        Kc, Vc = o.prefill(k, v, cs[:, None, :] if cs.ndim == 2 else cs, "fp32")
        wo = W["o_proj"].double().cpu().numpy()
        for i in range(steps):
            res, _ = m(dec[i], use_cache=True)
            x = dec[i, 0]
            pos = S + i
            cq, sq = rope_cos_sin(np.array([pos]), D, 500000.0, "fp32")
            qn = apply_rope(proj(x, "q_proj").reshape(1, Hq, D).transpose(1, 0, 2), cq, sq, "fp32")[:, 0]
            kn = apply_rope(proj(x, "k_proj").reshape(1, H, D).transpose(1, 0, 2), cq, sq, "fp32")
            vn = proj(x, "v_proj").reshape(1, H, D).transpose(1, 0, 2)
            Kc, Vc = np.concatenate([Kc, kn], 1), np.concatenate([Vc, vn], 1)
            qc = None if o.q is None else {k2: o.q[k2] for k2 in ("kq", "ks", "kz", "vq", "vs", "vz")}
            out, scm, scq = decode_attention(qn, Kc, Vc, "fp32", qc)
            ref = out.reshape(-1).astype(np.float64) @ wo.T
            np.testing.assert_allclose(res[0, 0].double().cpu().numpy(), ref, atol=2e-4, rtol=1e-3,
                                       err_msg=f"decode step {i}")
            Kc, Vc = o.decode(Kc, Vc, scm, scq, "fp32")
        ids, _ = kc.state.view_sticky(0)
        np.testing.assert_array_equal(ids.numpy(), o.window_scores[:, :ids.shape[1], 1])
        assert kc.state.read_error() == 0
        assert int(kc.global_token_counter) == S + steps


def _c1_inputs():
    import importlib.util
    path = os.path.join(GOLDEN, "c1_inputs.py")
    spec = importlib.util.spec_from_file_location("c1_inputs", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.C1, mod.c1_inputs


@pytest.mark.gpu
def test_attention_module_c1_matches_reference_golden(knobs, monkeypatch):
    """STICKYLlamaAttention (fp32) at the single-layer workload's full shape against
    outputs of the reference's own STICKYLlamaAttention on the same seeded inputs
    (tests/golden/module_c1_fp32.npz, written by make_golden.py module_c1): a
    4096-token prompt and 256 decode steps, free running on both sides (each
    side's own projections, logits, ledger and cycles).  Window sets after the
    prefill and after each of the four cycles: equal (and the Q-cache's top-k
    order); prefill outputs: max-abs <= 4e-5 (outputs up to ~6.4, fp32 sums
    over 4096 positions); final Q-cache scales within fp32 rounding of the
    inputs.

    Decode outputs: max-abs <= 1e-3.  Both sides' fp32 projections of the same
    inputs differ by ~1e-6, and the INT8 codes are a step function of K and V:
    a value on a rounding boundary of (x - zp) / scale takes the neighbouring
    code on one side, one quantisation step (scale ~ 0.03 here) apart, which
    the attention then weights by that token's probability.  The test counts
    those code flips (a few per window at most) and checks each side's code
    sums against the other's."""
    torch = _cuda()
    import qevict_b200.kv_cache as kvmod
    from qevict_b200.allocator import BudgetResult
    from qevict_b200.attention import STICKYLlamaAttention
    C1, c1_inputs = _c1_inputs()
    z = np.load(os.path.join(GOLDEN, "module_c1_fp32.npz"))
    assert [int(x) for x in z["config"]] == [C1[k] for k in ("hidden", "heads", "kv_heads", "omega", "sink", "local",
                                                             "k_windows", "q_windows", "prompt", "steps", "seed")]
    knobs(OMEGA=C1["omega"], SINK_TOKENS=C1["sink"], LOCAL_NUM_TOKENS=C1["local"], Q_RATIO=10,
          QUANTIZATION_BIT_WIDTH=8, GENERATION_CONFIG={"max_new_tokens": C1["steps"]})
    # the same fixed window budget the golden's generator gave the reference
    monkeypatch.setattr(kvmod, "compute_budget", lambda **kw: BudgetResult(
        C1["local"], C1["k_windows"], C1["q_windows"], 0, kw.get("head_dim", 0)))
    old_prec = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        cfg = SimpleNamespace(hidden_size=C1["hidden"], num_attention_heads=C1["heads"],
                              num_key_value_heads=C1["kv_heads"], max_position_embeddings=C1["prompt"] + C1["steps"] + 64,
                              rope_theta=500000.0, r_ratio=20, p_ratio=50, start_idx=0)
        w, hs, dec = c1_inputs(C1)
        m = STICKYLlamaAttention(cfg, 1).cuda()
        with torch.no_grad():
            for lin, name in ((m.q_proj, "q"), (m.k_proj, "k"), (m.v_proj, "v"), (m.o_proj, "o")):
                lin.weight.copy_(torch.from_numpy(w[name]))
            out_pre, _ = m(torch.from_numpy(hs).cuda()[None], use_cache=True)
            out_pre = out_pre[0].double().cpu().numpy()
            st = m.kv_cache.state
            kw = C1["k_windows"]

            def windows():
                ids, _ = st.view_sticky(0)
                q = st.view_q(0)
                return ids.numpy().astype(np.float32), q["ids"].numpy()

            pre_err = float(np.abs(out_pre[z["pre_rows"]] - z["out_pre"]).max())
            sticky, qsets = [], []
            ids, qids = windows()
            sticky.append(ids)
            qsets.append(qids)
            outs = []
            for i in range(C1["steps"]):
                o, _ = m(torch.from_numpy(dec[i]).cuda()[None, None], use_cache=True)
                outs.append(o[0, 0].double().cpu().numpy())
                if st.last_compaction == st.n_tokens:
                    ids, qids = windows()
                    sticky.append(ids)
                    qsets.append(qids)
        outs = np.stack(outs)
        dec_err = float(np.abs(outs[:, :1024] - z["out_dec"]).max())
        sum_err = float(np.abs(outs.sum(axis=1) - z["out_dec_sum"]).max())
        print(f"\n[C1 module vs reference golden] prefill rows max-abs {pre_err:.3e}, decode max-abs {dec_err:.3e}, "
              f"decode row-sum max-abs {sum_err:.3e}")
        assert len(sticky) == len(z["sticky_ids"]) == 5
        for c in range(5):
            np.testing.assert_array_equal(sticky[c], z["sticky_ids"][c][:, :kw], err_msg=f"sticky ids, cycle {c}")
            for h in range(C1["kv_heads"]):
                assert sorted(qsets[c][h].tolist()) == sorted(z["q_ids"][c][h].tolist()), f"Q window set, cycle {c}"
        order_same = np.mean([np.array_equal(a, b) for a, b in zip(qsets, z["q_ids"])])
        print(f"[C1] Q-cache top-k order identical after {order_same * 100:.0f} % of the cycles")
        assert dec_err <= 1e-3, dec_err
        assert pre_err <= 4e-5, pre_err
        q = st.view_q(0)
        # order the final Q windows like the reference's before comparing per window
        perm = [[list(q["ids"][h].numpy()).index(x) for x in z["q_ids"][-1][h]] for h in range(C1["kv_heads"])]
        hh = np.arange(C1["kv_heads"])[:, None]
        for key, ref in (("ks", z["q_ks"]), ("kz", z["q_kz"]), ("vs", z["q_vs"]), ("vz", z["q_vz"])):
            np.testing.assert_allclose(q[key].numpy()[hh, perm], ref, rtol=1e-5, atol=1e-6, err_msg=key)
        ksum = q["kq"].numpy().astype(np.int64).sum(axis=(2, 3))[hh, perm]
        vsum = q["vq"].numpy().astype(np.int64).sum(axis=(2, 3))[hh, perm]
        # a code can sit on a rounding boundary of (x - zp) / scale: at most a
        # handful of +-1 flips per window of 8192 codes
        kq0 = q["kq"].numpy()[hh, perm][:, 0].astype(np.int64)
        vq0 = q["vq"].numpy()[hh, perm][:, 0].astype(np.int64)
        flips = int((kq0 != z["q_kq_w0"]).sum() + (vq0 != z["q_vq_w0"]).sum())
        print(f"[C1] code flips in the first Q window of every head: {flips} of {kq0.size * 2}; "
              f"code-sum differences K {int(np.abs(ksum - z['q_kq_sum']).max())}, "
              f"V {int(np.abs(vsum - z['q_vq_sum']).max())}")
        assert int(np.abs(kq0 - z["q_kq_w0"]).max()) <= 1 and int(np.abs(vq0 - z["q_vq_w0"]).max()) <= 1
        assert flips <= 0.001 * kq0.size * 2
        assert np.abs(ksum - z["q_kq_sum"]).max() <= 16 and np.abs(vsum - z["q_vq_sum"]).max() <= 16
        assert int(m.kv_cache.global_token_counter) == int(z["global_token_counter"])
        assert st.read_error() == 0
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old_prec


def test_full_cache_bypass_r_ratio_100(knobs):
    """R_RATIO >= 100 with Q_RATIO == 0 keeps the prompt KV untouched and never
    evicts (cache.py:302-304: the prefill returns past_key_values as given;
    the decode branch then returns early, as logical_id_map stays None,
    cache.py:364-365); the counter still advances.  The oracle's state after
    its own prefill at R_RATIO 100 / no Q-cache is the same identity.  No
    device state is built, so this runs on the host."""
    import torch
    from qevict_b200.kv_cache import STICKYKVCache_LayerWise
    H, G, D, om, sink, local = 2, 2, 64, 16, 16, 32
    knobs(OMEGA=om, SINK_TOKENS=sink, LOCAL_NUM_TOKENS=local, Q_RATIO=0, QUANTIZATION_BIT_WIDTH=8,
          GENERATION_CONFIG={"max_new_tokens": 40})
    cfg = SimpleNamespace(hidden_size=H * G * D, num_attention_heads=H * G, num_key_value_heads=H,
                          max_position_embeddings=1024)
    cache = STICKYKVCache_LayerWise(50, 100, 0, H, 1, cfg)
    dev = torch.device("cpu")
    S = sink + 7 * om + 5          # any length: nothing is cut into windows
    K = torch.randn(1, H, S, D, device=dev)
    V = torch.randn(1, H, S, D, device=dev)
    cs = torch.rand(1, H, 1, S, device=dev)
    Kg, Vg = cache((K, V), cs, q_len=S)
    assert Kg is K and Vg is V
    assert cache.state is None
    for i in range(2 * om + 3):
        K = torch.cat([K, torch.randn(1, H, 1, D, device=dev)], 2)
        V = torch.cat([V, torch.randn(1, H, 1, D, device=dev)], 2)
        sc = torch.rand(1, H, 1, K.shape[2], device=dev)
        Kg, Vg = cache((K, V), sc, q_len=1)
        assert Kg is K and Vg is V
    assert cache.state is None
    # the counter counts the prompt and every decode token (cache.py:251-260)
    assert int(cache.global_token_counter) == S + 2 * om + 3


def test_full_cache_with_q_cache_rejected(knobs):
    """R_RATIO == 100 with a Q-cache (Q_RATIO > 0): the reference evicts at the
    prefill and then stops compacting (cache.py:391-397, the physical cache
    grows by torch.cat without bound).  The fixed slot layout cannot hold an
    unbounded cache, so this combination is refused with a clear error."""
    from qevict_b200 import QevictError
    from qevict_b200.kv_cache import STICKYKVCache_LayerWise
    import torch
    knobs(OMEGA=16, SINK_TOKENS=16, LOCAL_NUM_TOKENS=32, Q_RATIO=10, QUANTIZATION_BIT_WIDTH=8,
          GENERATION_CONFIG={"max_new_tokens": 40})
    cfg = SimpleNamespace(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=1024)
    cache = STICKYKVCache_LayerWise(50, 100, 0, 2, 1, cfg)
    K = torch.zeros(1, 2, 16 + 16 * 6, 64)
    with pytest.raises(QevictError, match="R_RATIO"):
        cache((K, K), torch.zeros(1, 2, 1, K.shape[2]))
