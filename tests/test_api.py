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
