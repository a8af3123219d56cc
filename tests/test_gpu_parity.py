"""CUDA path vs the oracle (which is pinned to the reference's golden vectors).

Integer / index state (window ids, Q-cache codes, scales, zero points, the
physical cache after every compaction) must match bit-for-bit whenever both
sides consume the same score ledger; attention outputs and ledger values match
within the stated tolerances.
"""

import numpy as np
import pytest
import torch

from oracle import codec as ocodec
from oracle.attention import decode_attention
from oracle.numerics import rnd
from oracle.sticky_state import OracleStickyLayer

pytestmark = pytest.mark.gpu

TD = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}
# Attention-output tolerance per KV dtype, given the same logits:
#   |gpu - ref| <= atol + rtol * |ref| + ulp(out_main) + ulp(out_q).
# The reference rounds the softmax probabilities to the KV dtype before P.V
# (src/models/attention/ops.py:132), which the kernel does not (rtol: about two
# ulps of the dtype), and rounds out_main and out_q separately before adding
# them (ops.py:150), so either may land one ulp apart (the two ulp terms).
TOL_OUT = {"fp32": (1e-5, 1e-5), "bf16": (2e-3, 1e-2), "fp16": (1e-3, 2e-3)}
# Vote-ledger tolerance (rtol, atol), given the same logits: the kernel and the
# oracle round the same probabilities; only the fp32 normaliser's summation
# order differs, which can flip a rounding tie by one ulp of the KV dtype.
TOL_LEDGER = {"fp32": (1e-5, 1e-7), "bf16": (8e-3, 1e-6), "fp16": (2e-3, 1e-7)}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    torch.manual_seed(0)


def to_dev(x, dt):
    return torch.tensor(np.ascontiguousarray(x), dtype=torch.float32).to(TD[dt]).cuda()


@pytest.mark.parametrize("dt", ["fp32", "bf16", "fp16"])
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("D", [128, 64])
def test_codec_kernels_bit_exact(dt, bits, D):
    from qevict_b200 import codec
    rng = np.random.default_rng(1)
    x = rnd(rng.standard_normal((2, 3, 64, D)).astype(np.float32) * 2.0, dt)
    x[0, 1] = 0.0
    x[1, 2] = 0.625
    x[1, 0, :, 5] = 1.5
    xt = to_dev(x, dt)
    kq, ks, kz = codec.quantize_k_per_window(xt, bits)
    vq, vs, vz = codec.quantize_v_per_window(xt, bits)
    okq, oks, okz = ocodec.quantize_k_per_window(x, dt, bits)
    ovq, ovs, ovz = ocodec.quantize_v_per_window(x, dt, bits)
    np.testing.assert_array_equal(kq.cpu().numpy(), okq)
    np.testing.assert_array_equal(vq.cpu().numpy(), ovq)
    for a, b in ((ks, oks), (kz, okz), (vs, ovs), (vz, ovz)):
        np.testing.assert_array_equal(a.float().cpu().numpy(), b)
    kd = codec.dequantize_from_quant(kq, ks, kz, bits)
    vd = codec.dequantize_from_quant(vq, vs, vz, bits)
    np.testing.assert_array_equal(kd.float().cpu().numpy(), ocodec.dequantize_from_quant(okq, oks, okz, dt, bits))
    np.testing.assert_array_equal(vd.float().cpu().numpy(), ocodec.dequantize_from_quant(ovq, ovs, ovz, dt, bits))


def _check_state(st, oracles, Kref, Vref, where):
    ck, qc = st.counts()
    for b, o in enumerate(oracles):
        ids, sc = st.view_sticky(b)
        oids, osc = o.sticky_ids()
        assert ck[b] == oids.shape[1], where
        np.testing.assert_array_equal(ids.numpy(), oids, err_msg=f"{where} b={b} sticky ids")
        np.testing.assert_array_equal(sc.numpy(), osc, err_msg=f"{where} b={b} sticky scores")
        q = st.view_q(b)
        if o.q is None:
            assert q is None, where
        else:
            assert qc[b] == o.q["ids"].shape[1], where
            for key in ("ids", "scores", "kq", "vq", "ks", "kz", "vs", "vz"):
                np.testing.assert_array_equal(q[key].numpy(), o.q[key], err_msg=f"{where} b={b} q.{key}")
        K, V = st.view_kv(b)
        np.testing.assert_array_equal(K.numpy(), Kref[b], err_msg=f"{where} b={b} K")
        np.testing.assert_array_equal(V.numpy(), Vref[b], err_msg=f"{where} b={b} V")
        np.testing.assert_array_equal(st.local_hist[b].cpu().numpy(), o.local_history, err_msg=f"{where} b={b} local_history")
        arch = st.arch_valid[b].cpu().numpy()
        got = sorted((int(w), int(h)) for h, w in zip(*np.nonzero(arch)))
        assert got == sorted(o.meta.keys()), f"{where} b={b} archive"


def run_parity(dt, bits=8, B=2, H=2, G=4, D=128, om=64, sink=64, local=128, kw=3, qw=4,
               n_prompt_windows=10, steps=256, seed=0, churn=True, maxW=64, reference_rounding=False,
               max_context=4096):
    """Prefill + decode + eviction cycles on the GPU and in the oracle, step by step.

    The tensor-core decode path dequantises the Q-cache exactly (code*scale + zp
    in fp32); the oracle then runs with dequant="exact".  The CUDA-core path
    (reference_rounding=True, and every shape the tensor-core kernel does not
    take) reproduces the reference's rounding; the oracle runs with
    dequant="reference".
    """
    from qevict_b200 import StickyLayerState
    rng = np.random.default_rng(seed)
    prompt = sink + n_prompt_windows * om
    st = StickyLayerState(B, H, G, D, om, sink, local, kw, qw, maxW, bits, TD[dt],
                          reference_rounding=reference_rounding)
    dq_mode = "exact" if st.decode_path == 1 else "reference"
    Kp = rnd(rng.standard_normal((B, H, prompt, D)), dt)
    Vp = rnd(rng.standard_normal((B, H, prompt, D)), dt)
    colsum = (rng.random((B, H, prompt)) * 4.0).astype(np.float32)
    st.prefill(to_dev(Kp, dt), to_dev(Vp, dt), torch.tensor(colsum).cuda())
    oracles, Kref, Vref = [], [], []
    for b in range(B):
        o = OracleStickyLayer(H, D, om, sink, local, kw, qw, dt, bits, max_windows=maxW,
                              max_context=max_context, window_sum="tree")
        K, V = o.prefill(Kp[b], Vp[b], colsum[b][:, None, :], "fp32")
        oracles.append(o)
        Kref.append(K)
        Vref.append(V)
    _check_state(st, oracles, Kref, Vref, "prefill")
    n_cycles = 0
    for step in range(steps):
        q = rnd(rng.standard_normal((B, H * G, D)) * 0.3, dt)
        if churn and step % om in (10, 40):
            # plant attention spikes on a random cached token (main zone or Q-cache)
            for b in range(B):
                for h in range(H):
                    o = oracles[b]
                    if o.q is not None and rng.random() < 0.5:
                        qd = ocodec.dequantize_from_quant(o.q["kq"], o.q["ks"], o.q["kz"], dt, bits)
                        j = rng.integers(qd.shape[1])
                        t = rng.integers(om)
                        key = qd[h, j, t]
                    else:
                        key = Kref[b][h, rng.integers(Kref[b].shape[1])]
                    q[b, h * G:(h + 1) * G] = rnd(key * rng.uniform(0.4, 0.9), dt)
        kn = rnd(rng.standard_normal((B, H, D)), dt)
        vn = rnd(rng.standard_normal((B, H, D)), dt)
        qr = st.append(to_dev(q, dt), to_dev(kn, dt), to_dev(vn, dt))
        out = torch.empty(B, H * G, D, dtype=TD[dt], device="cuda")
        st.attend(qr, out)
        out_h = out.float().cpu().numpy()
        due = False
        for b in range(B):
            o = oracles[b]
            Kc = np.concatenate([Kref[b], kn[b][:, None]], axis=1)
            Vc = np.concatenate([Vref[b], vn[b][:, None]], axis=1)
            qc = None
            if o.q is not None:
                qc = {k2: o.q[k2] for k2 in ("kq", "ks", "kz", "vq", "vs", "vz")}
            oo, sc, qsc, ex = decode_attention(q[b], Kc, Vc, dt, qc, bits, dequant=dq_mode, return_extras=True)
            # (1) the kernel's rounded logits equal the oracle's up to the accumulation-
            #     order bound: one ulp of the KV dtype at the raw dot product (/ sqrt D)
            #     plus one at the logit (plus the fp16 scale folding for Q tokens)
            gl = st.view_logits(b).numpy()
            assert gl.shape == ex["logits"].shape, (gl.shape, ex["logits"].shape)
            dl = np.abs(gl.astype(np.float64) - ex["logits"])
            bad = dl > ex["bound"]
            assert not bad.any(), f"step {step} b={b}: {int(bad.sum())} logits beyond bound, worst {float((dl - ex['bound']).max())}"
            # (2) everything downstream of the logits, driven by the kernel's logits
            oo, sc, qsc, ex2 = decode_attention(q[b], Kc, Vc, dt, qc, bits, dequant=dq_mode,
                                                logits_override=gl, return_extras=True)
            tol = TOL_OUT[dt][0] + TOL_OUT[dt][1] * np.abs(oo) + ex2["out_ulps"]
            err = np.abs(out_h[b] - oo)
            assert (err <= tol).all(), (f"step {step} b={b} out: {int((err > tol).sum())} beyond tolerance, "
                                        f"worst excess {float((err - tol).max())}")
            due = o.tally(Kc, sc, qsc, dt)
            S = Kc.shape[1]
            rt, at = TOL_LEDGER[dt]
            gv = st.view_votes(b).numpy()
            np.testing.assert_allclose(gv, o.votes[:, :S], rtol=rt, atol=at, err_msg=f"step {step} b={b} votes")
            gq = st.view_q(b)
            if o.q is not None:
                np.testing.assert_allclose(gq["scores"].numpy(), o.q["scores"], rtol=rt, atol=at,
                                           err_msg=f"step {step} b={b} q scores")
            if due:
                # same ledger on both sides before the cycle
                o.votes[:, :S] = gv
                if o.q is not None:
                    o.q["scores"] = gq["scores"].numpy().copy()
            Kref[b], Vref[b] = Kc, Vc
        assert due == st.cycle_due()
        if due:
            st.evict_cycle()
            for b in range(B):
                Kref[b], Vref[b] = oracles[b].cycle(Kref[b], Vref[b])
            n_cycles += 1
            _check_state(st, oracles, Kref, Vref, f"cycle {n_cycles}")
    assert st.read_error() == 0
    return n_cycles, oracles


@pytest.mark.parametrize("dt", ["bf16", "fp32", "fp16"])
def test_decode_and_cycles_vs_oracle(dt):
    n, oracles = run_parity(dt)
    assert n == 4
    # the planted spikes must have exercised promotion (archive) and Q churn
    assert any(len(o.meta) > 0 for o in oracles)


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
def test_decode_reference_rounding_mode(dt):
    """The CUDA-core kernel with the reference's Q-cache dequantisation rounding."""
    n, oracles = run_parity(dt, reference_rounding=True)
    assert n == 4
    # the planted spikes must have exercised promotion (archive) and Q churn
    assert any(len(o.meta) > 0 for o in oracles)


def test_decode_int4_qcache():
    n, _ = run_parity("bf16", bits=4, steps=128)
    assert n == 2


def test_decode_many_items_per_cta():
    """The full-model layer shape at batch 4: 4 x 8 (sequence, head) pairs of 116
    items (84 main-zone tiles of 32 tokens + 32 Q windows) = 3712 items over 148
    CTAs, 26 per CTA -- enough that the tensor-core kernel runs with ten consumer
    warps instead of eight.  Attention outputs, logits and ledger against the
    oracle for a few steps (the cycle does not depend on the warp count)."""
    n, _ = run_parity("bf16", B=4, H=8, local=512, kw=32, qw=32, n_prompt_windows=72, steps=6,
                      churn=False, maxW=128, max_context=8192)
    assert n == 0


def test_decode_mha_and_small_budget():
    # G = 1 (MHA), sticky capacity larger than the prompt offers (growing phase)
    n, _ = run_parity("fp16", G=1, kw=6, qw=2, n_prompt_windows=5, steps=192)
    assert n == 3


def test_misaligned_prompt_rejected():
    from qevict_b200 import QevictError, StickyLayerState
    st = StickyLayerState(1, 2, 4, 128, 64, 64, 128, 3, 4, 64, 8, torch.bfloat16)
    k = torch.zeros(1, 2, 64 + 64 * 5 + 7, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(QevictError):
        st.prefill(k, k, torch.zeros(1, 2, k.shape[2], device="cuda"))
