"""Research token ledger (TrackingManager) on the device.

* CPU: the oracle's ledger accessor and the no-op manager's API.
* GPU: the native updates replay the reference's own TrackingManager
  operation by operation (tests/golden/tracking_ops.npz, made by
  tests/golden/make_golden.py) bit for bit; and the cache object with
  ``tracking_flag = 1`` keeps the same ledger and score history as the oracle
  (whose cycle mapping and ledger reproduce the reference's, see
  test_oracle_golden.py) over a prefill and decode steps with planted churn.
"""

import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_noop_manager_api():
    from qevict_b200.tracking import NoOpTrackingManager
    m = NoOpTrackingManager(torch.device("cpu"))
    m.increment(5)
    m.record_prefill(4, 4, 0, None, None, None, 0, 4)
    m.record_decode(None, 5, 0, 4)
    m.update_physical_positions(None, 5, None)
    assert int(m.global_token_counter) == 5
    assert tuple(m.token_ledger.shape) == (1, 2)
    assert set(m.get_ledger_data()) == {"global_id", "layer_id", "physical_id", "attention_score"}
    m.reset()
    assert int(m.global_token_counter) == 0


def test_ledger_accessor_matches_oracle():
    from oracle.tracking import OracleTracker
    from qevict_b200.ledger import get_ledger_data
    z = np.load(os.path.join(GOLD, "tracking_ops.npz"))
    H = int(z["params"][0])
    tr = OracleTracker(z["ledger"].shape[1], H)
    tr.ledger[:] = z["ledger"][-1]
    tr.counter = int(z["counter"])
    want = tr.get_ledger_data()
    got = get_ledger_data(torch.tensor(tr.counter), torch.tensor(z["ledger"][-1]), H)
    for k in want:
        np.testing.assert_array_equal(got[k].numpy(), want[k])


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


@pytest.mark.gpu
def test_native_ledger_replays_reference_ops():
    """qv_track_prefill / qv_track_decode / qv_track_positions against the
    reference's TrackingManager: every snapshot of the ledger and the score
    history equal (float32 adds in the same order), including positions past
    the score row, evicted tokens and tokens past max_context."""
    _cuda()
    from qevict_b200.tracking import TrackingManager
    z = np.load(os.path.join(GOLD, "tracking_ops.npz"))
    H, C, prompt, keep, steps, layer = (int(v) for v in z["params"])
    dev = torch.device("cuda")
    tm = TrackingManager(C, H, dev)
    snaps = iter(range(z["ledger"].shape[0]))

    def check(what):
        k = next(snaps)
        np.testing.assert_array_equal(tm.token_ledger.cpu().numpy(), z["ledger"][k], err_msg=what)
        np.testing.assert_array_equal(tm._global_score_history.cpu().numpy(), z["hist"][k], err_msg=what)

    tm.increment(prompt)
    tm.record_prefill(prompt, prompt, layer, torch.tensor(z["attn"], device=dev), torch.tensor(z["surv"]), None,
                      0, prompt)
    check("prefill")
    cycles = list(z["cycles"])
    for step in range(steps):
        gs = int(tm.global_token_counter)
        tm.increment(1)
        kv, S = int(z["kv"][step]), int(z["seq_len"][step])
        tm.record_decode(torch.tensor(z["scores"][step][None, :, None, :kv], device=dev), S, layer, gs)
        check(f"decode {step}")
        if step in cycles:
            ci = cycles.index(step)
            tm.update_physical_positions(torch.tensor(z["mapping"][ci][:, :S], device=dev), S,
                                         torch.tensor(z["votes"][ci], device=dev))
            check(f"positions {step}")
    assert int(tm.global_token_counter) == int(z["counter"])
    data = tm.get_ledger_data()
    assert data["global_id"].shape[0] == min(int(z["counter"]), C)


@pytest.mark.gpu
def test_cache_object_ledger_matches_oracle():
    _cuda()
    from oracle.attention import decode_attention
    from oracle.sticky_state import OracleStickyLayer
    from oracle.tracking import OracleTracker, tracked_decode, tracked_prefill
    from qevict_b200 import sticky_config as sc
    from qevict_b200.kv_cache import STICKYKVCache_LayerWise
    keys = ("OMEGA", "SINK_TOKENS", "LOCAL_NUM_TOKENS", "Q_RATIO", "QUANTIZATION_BIT_WIDTH", "GENERATION_CONFIG",
            "tracking_flag")
    saved = {k: getattr(sc, k) for k in keys}
    H, G, D, om, sink, local, steps = 2, 2, 64, 16, 16, 32, 100
    try:
        for k, v in dict(OMEGA=om, SINK_TOKENS=sink, LOCAL_NUM_TOKENS=local, Q_RATIO=40, QUANTIZATION_BIT_WIDTH=8,
                         GENERATION_CONFIG={"max_new_tokens": steps}, tracking_flag=1).items():
            setattr(sc, k, v)
        cfg = SimpleNamespace(hidden_size=H * G * D, num_attention_heads=H * G, num_key_value_heads=H,
                              max_position_embeddings=1024)
        cache = STICKYKVCache_LayerWise(50, 30, 0, H, 3, cfg)
    finally:
        for k, v in saved.items():
            setattr(sc, k, v)
    rng = np.random.default_rng(17)
    S = sink + 20 * om
    K = rng.standard_normal((1, H, S, D)).astype(np.float32)
    V = rng.standard_normal((1, H, S, D)).astype(np.float32)
    cs = (rng.random((1, H, 1, S)) * 3).astype(np.float32)
    dev = torch.device("cuda")
    Kg, Vg = cache((torch.tensor(K, device=dev), torch.tensor(V, device=dev)), torch.tensor(cs, device=dev),
                   q_len=S)
    o = OracleStickyLayer(H, D, om, sink, cache.local_num, cache.k_windows, cache.q_windows_count, "fp32", 8,
                          max_windows=cache.max_windows, max_context=1024, r_ratio=30, window_sum="tree")
    tr = OracleTracker(1024, H)
    Ko, Vo = tracked_prefill(o, tr, K[0], V[0], cs[0], "fp32", 3)

    def same(what):
        np.testing.assert_array_equal(cache.token_ledger.cpu().numpy(), tr.ledger, err_msg=what)
        np.testing.assert_array_equal(cache.global_score_history.cpu().numpy(), tr.history, err_msg=what)

    same("prefill")
    np.testing.assert_array_equal(cache.prefill_attention_matrix.numpy(), tr.prefill_attention_matrix)
    for step in range(steps):
        q = (rng.standard_normal((H * G, D)) * 0.5).astype(np.float32)
        kn = rng.standard_normal((H, 1, D)).astype(np.float32)
        vn = rng.standard_normal((H, 1, D)).astype(np.float32)
        Kc, Vc = np.concatenate([Ko, kn], 1), np.concatenate([Vo, vn], 1)
        qc = None if o.q is None else {k: o.q[k] for k in ("kq", "ks", "kz", "vq", "vs", "vz")}
        _, scm, scq = decode_attention(q, Kc, Vc, "fp32", qc)
        if step % om == om // 2:       # planted churn: a large vote on a random main-zone token
            for h in range(H):
                scm[h, rng.integers(sink, Kc.shape[1])] += np.float32(40.0)
        sc_t = torch.tensor(scm[None, :, None, :], device=dev)
        qs_t = None if scq is None else torch.tensor(scq[None, :, None, :], device=dev)
        Kg, Vg = cache((torch.cat([Kg, torch.tensor(kn[None], device=dev)], 2),
                        torch.cat([Vg, torch.tensor(vn[None], device=dev)], 2)), sc_t, q_attn_scores=qs_t)
        Ko, Vo = tracked_decode(o, tr, Kc, Vc, scm, scq, "fp32", 3)
        np.testing.assert_array_equal(Kg[0].cpu().numpy(), Ko, err_msg=f"step {step}")
        same(f"step {step}")
    led = tr.ledger[:tr.counter]
    left = (led[:, 0] >= 0) & (led[:, 2:2 + H] < 0).all(axis=1)
    assert left.sum() >= om, "no token left the cache"
    assert int(cache.get_ledger_data()["global_id"].shape[0]) == S + steps
