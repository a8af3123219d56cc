"""Pin the oracle against golden vectors recorded from the reference itself.

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py,
which imports the reference's own modules (quantize.py, ops.py,
STICKYKVCache_LayerWise, STICKYLlamaAttention, ops_flash.py) and records their
outputs on seeded inputs.  Integer / index outputs must match exactly; float
outputs within the tolerances stated in each test.
"""

import os

import numpy as np
import pytest

from oracle import codec
from oracle.attention import decode_attention
from oracle.prefill import causal_attention, chunked_prefill_scores, sdpa_causal_attention
from oracle.sticky_state import OracleStickyLayer, apply_rope, rope_cos_sin

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name + ".npz"))


@pytest.mark.parametrize("dt", ["fp32", "bf16", "fp16"])
@pytest.mark.parametrize("bits", [8, 4])
def test_codec_bit_exact(dt, bits):
    z = load("codec")
    p = f"{dt}_b{bits}_"
    x = z[p + "x"]
    kq, ks, kz = codec.quantize_k_per_window(x, dt, bits)
    vq, vs, vz = codec.quantize_v_per_window(x, dt, bits)
    np.testing.assert_array_equal(kq, z[p + "kq"])
    np.testing.assert_array_equal(vq, z[p + "vq"])
    np.testing.assert_array_equal(ks, z[p + "ks"])
    np.testing.assert_array_equal(kz, z[p + "kz"])
    np.testing.assert_array_equal(vs, z[p + "vs"])
    np.testing.assert_array_equal(vz, z[p + "vz"])
    kd = codec.dequantize_from_quant(kq, ks, kz, dt, bits)
    vd = codec.dequantize_from_quant(vq, vs, vz, dt, bits)
    np.testing.assert_array_equal(kd, z[p + "kd"])
    np.testing.assert_array_equal(vd, z[p + "vd"])


def test_codec_d128_bit_exact():
    z = load("codec")
    kq, ks, kz = codec.quantize_k_per_window(z["d128_x"], "bf16")
    vq, vs, vz = codec.quantize_v_per_window(z["d128_x"], "bf16")
    for a, b in ((kq, "kq"), (ks, "ks"), (kz, "kz"), (vq, "vq"), (vs, "vs"), (vz, "vz")):
        np.testing.assert_array_equal(a, z["d128_" + b])


# bf16 / fp16 outputs may differ by one ulp of the KV dtype at a logit rounding
# boundary (the oracle accumulates matmuls in float64, torch in fp32).
ATOL = {"fp32": 1e-5, "bf16": 2e-3, "fp16": 5e-4}


@pytest.mark.parametrize("dt", ["fp32", "bf16", "fp16"])
def test_decode_attention(dt):
    z = load("attention")
    p = dt + "_"
    H = z[p + "k"].shape[1]
    qc = dict(kq=z[p + "kq"], ks=z[p + "ks"], kz=z[p + "kz"], vq=z[p + "vq"], vs=z[p + "vs"], vz=z[p + "vz"])
    q = z[p + "q"][0, :, 0]
    out, sc, qs = decode_attention(q, z[p + "k"][0], z[p + "v"][0], dt, qc)
    np.testing.assert_allclose(out, z[p + "out"][0, :, 0], atol=ATOL[dt], rtol=0)
    np.testing.assert_allclose(sc, z[p + "scores"][0, :, 0], atol=ATOL[dt] / 10, rtol=0)
    np.testing.assert_allclose(qs, z[p + "qscores"][0, :, 0], atol=ATOL[dt] / 10, rtol=0)
    out2, sc2, _ = decode_attention(q, z[p + "k"][0], z[p + "v"][0], dt, None)
    np.testing.assert_allclose(out2, z[p + "out_noq"][0, :, 0], atol=ATOL[dt], rtol=0)
    np.testing.assert_allclose(sc2, z[p + "scores_noq"][0, :, 0], atol=ATOL[dt] / 10, rtol=0)
    assert sc.shape == (H, z[p + "k"].shape[2])


@pytest.mark.parametrize("name", ["state_bf16_sdpa", "state_fp32_fa", "state_fp16_fa"])
def test_state_machine_replay(name):
    """Replay the reference's prefill + 96 decode steps with forced churn.

    Window sets, Q-cache ids, INT8 codes and scales, logical id maps and the
    physical cache must all match exactly; window/Q scores and local history
    (fp32 sums) within 1e-5 relative.
    """
    z = load(name)
    H, D, om, sink, local, kw, qw, prompt, steps, bits, maxW = [int(v) for v in z["params"]]
    dt = str(z["dt"])
    st = OracleStickyLayer(H, D, om, sink, local, kw, qw, dt, bits, max_windows=maxW,
                           max_context=4096, window_sum="sequential")
    attn = z["attn"][0]
    K, V = st.prefill(z["K0"][0], z["V0"][0], attn, str(z["attn_dt"]))
    np.testing.assert_array_equal(K, z["pre_K"][0])
    np.testing.assert_array_equal(V, z["pre_V"][0])
    np.testing.assert_array_equal(st.lid, z["pre_lid"])
    ws = z["pre_ws"]
    np.testing.assert_array_equal(np.isnan(st.window_scores), np.isnan(ws))
    np.testing.assert_allclose(np.nan_to_num(st.window_scores), np.nan_to_num(ws), rtol=1e-6)
    np.testing.assert_allclose(st.local_history, z["pre_lh"], rtol=1e-6)
    np.testing.assert_array_equal(st.q["ids"], z["pre_qids"])
    np.testing.assert_array_equal(st.q["kq"], z["pre_qkq"])
    cyc = 0
    for step in range(steps):
        kn, vn = z["newk"][step], z["newv"][step]
        Kc = np.concatenate([K, kn[:, None]], axis=1)
        Vc = np.concatenate([V, vn[:, None]], axis=1)
        S = Kc.shape[1]
        sc = z["scores"][step][:, :S]
        qn = int(z["qscores_n"][step])
        qs = z["qscores"][step][:, :qn] if qn >= 0 else None
        K, V = st.decode(Kc, Vc, sc, qs, dt)
        if st.tokens_since == 0:
            p = f"c{cyc}_"
            assert int(z[p + "step"]) == step
            np.testing.assert_array_equal(st.window_scores[:, :kw, 1], z[p + "ws"][:, :, 1])
            np.testing.assert_allclose(st.window_scores[:, :kw, 0], z[p + "ws"][:, :, 0], rtol=1e-5)
            np.testing.assert_array_equal(st.lid, z[p + "lid"])
            np.testing.assert_array_equal(K, z[p + "K"][0])
            np.testing.assert_array_equal(V, z[p + "V"][0])
            np.testing.assert_allclose(st.local_history, z[p + "lh"], rtol=1e-5, atol=1e-7)
            if p + "qids" in z:
                np.testing.assert_array_equal(st.q["ids"], z[p + "qids"])
                np.testing.assert_allclose(st.q["scores"], z[p + "qsc"], rtol=1e-5)
                np.testing.assert_array_equal(st.q["kq"], z[p + "qkq"])
                np.testing.assert_array_equal(st.q["vq"], z[p + "qvq"])
                for key in ("ks", "kz", "vs", "vz"):
                    np.testing.assert_array_equal(st.q[key], z[p + "q" + key])
            else:
                assert st.q is None
            meta = sorted([list(k) for k in st.meta.keys()])
            np.testing.assert_array_equal(np.array(meta, dtype=np.int64).reshape(-1, 2), z[p + "meta"].reshape(-1, 2))
            cyc += 1
    assert cyc == int(z["n_cycles"])
    np.testing.assert_array_equal(K, z["final_K"][0])


@pytest.mark.parametrize("name", ["module_fp32", "module_bf16"])
def test_module_end_to_end(name):
    """Whole STICKYLlamaAttention (projections, RoPE, attention, cache) vs the reference."""
    from oracle.numerics import rnd
    z = load(name)
    dt = str(z["dt"])
    wq, wk, wv, wo = z["wq"], z["wk"], z["wv"], z["wo"]
    Hq, H, D = 4, 2, 16
    st = OracleStickyLayer(H, D, 16, 8, 32, 3, 4, dt, 8, max_windows=255, max_context=4096)

    def proj(x, w):
        return rnd(np.asarray(x, np.float64) @ np.asarray(w, np.float64).T, dt)

    hs = z["hs"][0]
    S = hs.shape[0]
    q = proj(hs, wq).reshape(S, Hq, D).transpose(1, 0, 2)
    k = proj(hs, wk).reshape(S, H, D).transpose(1, 0, 2)
    v = proj(hs, wv).reshape(S, H, D).transpose(1, 0, 2)
    cos, sin = rope_cos_sin(np.arange(S), D, 500000.0, dt, inv_freq_dt=dt)
    q = apply_rope(q, cos, sin, dt)
    k = apply_rope(k, cos, sin, dt)
    o, attn = sdpa_causal_attention(q, k, v, dt)
    out_pre = proj(o.transpose(1, 0, 2).reshape(S, Hq * D), wo)
    tol = 1e-5 if dt == "fp32" else 2e-2
    np.testing.assert_allclose(out_pre, z["out_pre"][0], atol=tol, rtol=0)
    Kc, Vc = st.prefill(k, v, attn, dt)
    for i in range(z["dec"].shape[0]):
        x = z["dec"][i, 0]
        pos = st.global_counter
        cq, sq = rope_cos_sin(np.array([pos]), D, 500000.0, dt, inv_freq_dt=dt)
        qn = apply_rope(proj(x, wq).reshape(1, Hq, D).transpose(1, 0, 2), cq, sq, dt)[:, 0]
        kn = apply_rope(proj(x, wk).reshape(1, H, D).transpose(1, 0, 2), cq, sq, dt)
        vn = proj(x, wv).reshape(1, H, D).transpose(1, 0, 2)
        Kc = np.concatenate([Kc, kn], axis=1)
        Vc = np.concatenate([Vc, vn], axis=1)
        qcache = None
        if st.q is not None:
            qcache = {k2: st.q[k2] for k2 in ("kq", "ks", "kz", "vq", "vs", "vz")}
        out, scm, scq = decode_attention(qn, Kc, Vc, dt, qcache)
        res = proj(out.reshape(-1), wo)
        np.testing.assert_allclose(res, z["outs"][i], atol=tol, rtol=0)
        Kc, Vc = st.decode(Kc, Vc, scm, scq, dt)
    np.testing.assert_array_equal(st.window_scores[:, :3, 1], z["ws"][:, :, 1])


@pytest.mark.parametrize("dt", ["fp32", "bf16"])
def test_prefill_lane(dt):
    z = load("prefill")
    p = dt + "_"
    q, k, v = z[p + "q"][0], z[p + "k"][0], z[p + "v"][0]
    cs = chunked_prefill_scores(q, k, dt)
    rtol = 1e-5 if dt == "fp32" else 2e-2
    np.testing.assert_allclose(cs, z[p + "colsum"][0, :, 0], rtol=rtol, atol=1e-5)
    out = causal_attention(q, k, v, dt)
    atol = 1e-5 if dt == "fp32" else 2e-2
    np.testing.assert_allclose(out, z[p + "out"][0], atol=atol, rtol=0)
    out2, _ = sdpa_causal_attention(q, k, v, dt)
    np.testing.assert_allclose(out2, z[p + "out"][0], atol=atol / 4 if dt != "fp32" else atol, rtol=0)


# ----------------------------------------------------------------------------- token ledger
def _ledger_eq(tr, ledger, hist, what):
    R = ledger.shape[0]
    np.testing.assert_array_equal(tr.ledger[:R], ledger, err_msg=what)
    np.testing.assert_array_equal(tr.history[:R], hist, err_msg=what)
    assert (tr.ledger[R:] == -1).all() and (tr.history[R:] == -1).all(), what


def test_tracking_ops_replay():
    """TrackingManager operation by operation: every ledger and history
    snapshot bit for bit (float32 adds in the reference's order)."""
    from oracle.tracking import OracleTracker
    z = load("tracking_ops")
    H, C, prompt, keep, steps, layer = (int(v) for v in z["params"])
    tr = OracleTracker(C, H)
    tr.increment(prompt)
    tr.record_prefill(prompt, prompt, layer, z["attn"], z["surv"], None, 0, prompt)
    k = 0
    _ledger_eq(tr, z["ledger"][k], z["hist"][k], "prefill")
    cycles = list(z["cycles"])
    for step in range(steps):
        gs = tr.counter
        tr.increment(1)
        kv, S = int(z["kv"][step]), int(z["seq_len"][step])
        tr.record_decode(z["scores"][step][None, :, None, :kv], S, layer, gs)
        k += 1
        _ledger_eq(tr, z["ledger"][k], z["hist"][k], f"decode {step}")
        if step in cycles:
            ci = cycles.index(step)
            tr.update_physical_positions(z["mapping"][ci][:, :S], S, z["votes"][ci])
            k += 1
            _ledger_eq(tr, z["ledger"][k], z["hist"][k], f"positions {step}")
    assert tr.counter == int(z["counter"]) and k + 1 == z["ledger"].shape[0]


def test_tracking_state_replay():
    """The cache object with tracking on (prefill + 96 decode steps with churn):
    the oracle's old->new position mapping and ledger reproduce the
    reference's token ledger and score history bit for bit at every cycle."""
    from oracle.tracking import OracleTracker, tracked_decode, tracked_prefill
    z = load("tracking_fp32_fa")
    H, D, om, sink, local, kw, qw, prompt, steps, bits, maxW = [int(v) for v in z["params"]]
    dt = str(z["dt"])
    st = OracleStickyLayer(H, D, om, sink, local, kw, qw, dt, bits, max_windows=maxW,
                           max_context=4096, window_sum="sequential")
    tr = OracleTracker(4096, H)
    K, V = tracked_prefill(st, tr, z["K0"][0], z["V0"][0], z["attn"][0], str(z["attn_dt"]), 1)
    _ledger_eq(tr, z["pre_trk_ledger"], z["pre_trk_hist"], "prefill")
    cyc = 0
    for step in range(steps):
        Kc = np.concatenate([K, z["newk"][step][:, None]], axis=1)
        Vc = np.concatenate([V, z["newv"][step][:, None]], axis=1)
        S = Kc.shape[1]
        qn = int(z["qscores_n"][step])
        qs = z["qscores"][step][:, :qn] if qn >= 0 else None
        K, V = tracked_decode(st, tr, Kc, Vc, z["scores"][step][:, :S], qs, dt, 1)
        if st.tokens_since == 0:
            p = f"c{cyc}_"
            np.testing.assert_array_equal(K, z[p + "K"][0])
            _ledger_eq(tr, z[p + "trk_ledger"], z[p + "trk_hist"], p)
            assert tr.counter == int(z[p + "trk_counter"])
            cyc += 1
    assert cyc == int(z["n_cycles"]) and cyc >= 5
    _ledger_eq(tr, z["final_trk_ledger"], z["final_trk_hist"], "final")
