"""The prefill lane at the full-model workload's prompt length (32768 tokens).

The numpy oracle cannot run a 32k-token causal attention in test time, so the
checker here is a plain PyTorch fp32 restatement on the GPU (matmuls without
TF32), chunked over queries, with the reference's rounding points:

* output: causal softmax(q k^T / sqrt(D)) v in fp32, rounded once to the KV
  dtype (the exact causal attention of oracle.prefill.causal_attention);
* column sums: the chunked scorer of src/models/attention/ops_flash.py:56-141
  (oracle.prefill.chunked_prefill_scores): per 512-query chunk the logits are
  rounded to the KV dtype and divided by sqrt(D) (rounded), the softmax is
  fp32, probabilities are rounded to the KV dtype, the GQA group mean is
  rounded, the chunk's sum over queries is rounded to the KV dtype, and chunk
  sums are accumulated in fp32.

Bounds, each from a rounding point:
* output, per element: u * sum_k p_qk |v_k| + one ulp of the output (u = unit
  roundoff of the KV dtype): the tensor-core lane rounds the probabilities to
  the KV dtype before P.V, as the reference's flash-attention path does, and
  both sides round the result once;
* column sums, relative: 2^-7 (bf16) / 2^-10 (fp16) -- a chunk sum rounded to
  the KV dtype can land one ulp apart when one of its probabilities rounds the
  other way (fp32 normaliser summed in another order), and the accumulation of
  positive chunk sums keeps that relative bound.
The plain maximum absolute error of the output is reported.  The window sets
the prefill state builder selects from the lane's sums must equal the
oracle's, given the same sums (bit-exact).
"""

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TD = {"bf16": torch.bfloat16, "fp16": torch.float16}
UNIT = {"bf16": 2.0 ** -8, "fp16": 2.0 ** -11}
CS_RTOL = {"bf16": 2.0 ** -7, "fp16": 2.0 ** -10}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _ulp(x, dt):
    bits = {"bf16": 7, "fp16": 10}[dt]
    ax = x.abs().clamp_min(1e-30)
    return torch.exp2(torch.floor(torch.log2(ax)) - bits)


def reference(q, k, v, dt, chunk=512):
    """q [S, Hq, D], k/v [S, H, D] (KV dtype, on the GPU) -> (out [S, Hq, D] fp32
    rounded to dt, abs-weighted sums [S, Hq, D], column sums [H, S] fp32)."""
    S, Hq, D = q.shape
    H = k.shape[1]
    G = Hq // H
    td = TD[dt]
    out = torch.empty(S, Hq, D, device=q.device)
    aw = torch.empty(S, Hq, D, device=q.device)
    cs = torch.zeros(H, S, device=q.device)
    sd = torch.tensor(math.sqrt(D), dtype=torch.float32)
    for h in range(H):
        kh = k[:, h].float()                 # [S, D]
        vh = v[:, h].float()
        for i in range(0, S, chunk):
            c = min(chunk, S - i)
            n = i + c                         # keys a causal chunk can see
            qc = q[i:i + c, h * G:(h + 1) * G].float().permute(1, 0, 2)   # [G, c, D]
            raw = qc @ kh[:n].t()                                         # [G, c, n]
            causal = torch.arange(n, device=q.device)[None, :] <= torch.arange(i, i + c, device=q.device)[:, None]
            # exact causal output (rounded once at the end)
            x = torch.where(causal, raw / sd, torch.tensor(-math.inf, device=q.device))
            p = torch.softmax(x, dim=-1)
            out[i:i + c, h * G:(h + 1) * G] = (p @ vh[:n]).permute(1, 0, 2)
            aw[i:i + c, h * G:(h + 1) * G] = (p @ vh[:n].abs()).permute(1, 0, 2)
            # the chunked scorer's rounding points
            lg = (raw.to(td).float() / sd).to(td).float()
            minv = torch.finfo(td).min
            lg = torch.where(causal, lg, torch.tensor(minv, device=q.device)).to(td).float()
            pr = torch.softmax(lg, dim=-1).to(td).float()
            gm = pr.mean(dim=0).to(td).float() if G > 1 else pr[0]
            cs[h, :n] += gm.sum(dim=0).to(td).float()
    return out.to(td).float(), aw, cs


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
def test_prefill_lane_32k(dt):
    from oracle.sticky_state import OracleStickyLayer
    from qevict_b200 import StickyLayerState
    from qevict_b200.model import prefill_attention
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        S, Hq, H, D = 32768, 32, 8, 128
        g = torch.Generator(device="cuda").manual_seed(31)
        q = torch.randn(1, S, Hq, D, generator=g, device="cuda").to(TD[dt])
        k = torch.randn(1, S, H, D, generator=g, device="cuda").to(TD[dt])
        v = torch.randn(1, S, H, D, generator=g, device="cuda").to(TD[dt])
        out, cs = prefill_attention(q, k, v)
        ref_out, aw, ref_cs = reference(q[0], k[0], v[0], dt)
        got = out[0].float()
        err = (got - ref_out).abs()
        tol = 1.01 * UNIT[dt] * aw + _ulp(ref_out, dt) + 1e-30
        ratio = float((err / tol).max())
        mx = float(err.max())
        late = float(err[512:].max())
        cs_rel = float(((cs[0] - ref_cs).abs() / ref_cs.abs().clamp_min(1e-30)).max())
        print(f"\n[prefill {dt} S={S}] output max-abs {mx:.3e} (queries >= 512: {late:.3e}), max err/bound "
              f"{ratio:.3f}; column sums max relative difference {cs_rel:.3e} (bound {CS_RTOL[dt]:.2e})")
        assert ratio <= 1.0
        assert cs_rel <= CS_RTOL[dt]
        # the prompt state built from the lane's column sums: window sets,
        # Q-cache codes and the physical cache equal the oracle's given the same sums
        om, sink, local, kw, qw = 64, 64, 512, 32, 32
        st = StickyLayerState(1, H, Hq // H, D, om, sink, local, kw, qw, (S - sink) // om + 8, 8, TD[dt])
        kt = k.transpose(1, 2).contiguous()
        vt = v.transpose(1, 2).contiguous()
        st.prefill(kt, vt, cs)
        o = OracleStickyLayer(H, D, om, sink, local, kw, qw, dt, 8, max_windows=(S - sink) // om + 8,
                              max_context=S + 1024, window_sum="tree")
        Kr, Vr = o.prefill(kt[0].float().cpu().numpy(), vt[0].float().cpu().numpy(),
                           cs[0].cpu().numpy()[:, None, :], "fp32")
        ids, _ = st.view_sticky(0)
        np.testing.assert_array_equal(ids.numpy(), o.sticky_ids()[0])
        qv = st.view_q(0)
        for key in ("ids", "kq", "vq", "ks", "kz", "vs", "vz"):
            np.testing.assert_array_equal(qv[key].numpy(), o.q[key], err_msg=key)
        Kg, Vg = st.view_kv(0)
        np.testing.assert_array_equal(Kg.numpy(), Kr)
        np.testing.assert_array_equal(Vg.numpy(), Vr)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
