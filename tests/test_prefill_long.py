"""The prefill lane at the full-model workload's prompt length (32768 tokens).

The numpy oracle cannot run a 32k-token causal attention in test time, so the
checker here is a plain PyTorch fp32 restatement on the GPU (matmuls without
TF32), chunked over queries, with the reference's rounding points:

* output: the SDPA prefill of src/models/attention/module.py:258-304
  (oracle.prefill.sdpa_causal_attention): q.k rounded to the KV dtype, / sqrt(D)
  rounded, causal fp32 softmax, probabilities rounded to the KV dtype, P.V
  rounded once -- the rounding points the tensor-core lane reproduces;
* column sums: the chunked scorer of src/models/attention/ops_flash.py:56-141
  (oracle.prefill.chunked_prefill_scores): per 512-query chunk the same rounded
  logits, fp32 softmax, probabilities rounded, the GQA group mean rounded, the
  chunk's sum over queries rounded to the KV dtype, chunk sums accumulated in
  fp32.

Bounds, each from a rounding point:
* output, per element: both sides round the same quantities, but their fp32
  dot products are summed in different orders, so a logit can land one ulp
  apart at either rounding: d_k <= ulp(q.k_k) / sqrt(D) + ulp(logit_k).  A
  logit change d_k moves the output by at most sum_k p_k |v_k| d_k + |out|
  sum_k p_k d_k (the normaliser); a probability rounding the other way moves
  it by at most u * sum_k p_k |v_k| (u = unit roundoff of the KV dtype); plus
  one ulp of the output.  This is a worst case (every logit flipped);
* column sums, relative: one ulp of a chunk sum (2^-7 bf16, 2^-10 fp16) plus
  the probabilities' own one-ulp flips inside it (2^-8, 2^-11), preserved by
  the fp32 accumulation of positive chunk sums.
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
CS_RTOL = {"bf16": 2.0 ** -7 + 2.0 ** -8, "fp16": 2.0 ** -10 + 2.0 ** -11}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _ulp(x, dt):
    bits = {"bf16": 7, "fp16": 10}[dt]
    ax = x.abs().clamp_min(1e-30)
    return torch.exp2(torch.floor(torch.log2(ax)) - bits)


def reference(q, k, v, dt, chunk=512):
    """q [S, Hq, D], k/v [S, H, D] (KV dtype, on the GPU) -> (out [S, Hq, D]
    rounded to dt, bound [S, Hq, D] on |lane - out|, column sums [H, S] fp32)."""
    S, Hq, D = q.shape
    H = k.shape[1]
    G = Hq // H
    td = TD[dt]
    u = UNIT[dt]
    out = torch.empty(S, Hq, D, device=q.device)
    bound = torch.empty(S, Hq, D, device=q.device)
    cs = torch.zeros(H, S, device=q.device)
    sd = torch.tensor(math.sqrt(D), dtype=torch.float32)
    minv = torch.finfo(td).min
    for h in range(H):
        kh = k[:, h].float()                 # [S, D]
        vh = v[:, h].float()
        for i in range(0, S, chunk):
            c = min(chunk, S - i)
            n = i + c                         # keys a causal chunk can see
            qc = q[i:i + c, h * G:(h + 1) * G].float().permute(1, 0, 2)   # [G, c, D]
            raw = qc @ kh[:n].t()                                         # [G, c, n]
            causal = torch.arange(n, device=q.device)[None, :] <= torch.arange(i, i + c, device=q.device)[:, None]
            rr = raw.to(td).float()
            lg = (rr / sd).to(td).float()
            lg = torch.where(causal, lg, torch.tensor(minv, device=q.device)).to(td).float()
            p = torch.softmax(lg, dim=-1)                                  # fp32
            pr = p.to(td).float()
            o = (pr @ vh[:n]).to(td).float()                               # [G, c, D]
            out[i:i + c, h * G:(h + 1) * G] = o.permute(1, 0, 2)
            dlt = torch.where(causal, _ulp(rr, dt) / sd + _ulp(lg, dt), torch.zeros((), device=q.device))
            A = p @ vh[:n].abs()
            Ad = (p * dlt) @ vh[:n].abs()
            Bd = (p * dlt).sum(-1, keepdim=True)
            b = 1.01 * (u * A + Ad + o.abs() * Bd + 64 * 2.0 ** -24 * A) + _ulp(o, dt)
            bound[i:i + c, h * G:(h + 1) * G] = b.permute(1, 0, 2)
            # the chunked scorer (same rounded logits)
            gm = pr.mean(dim=0).to(td).float() if G > 1 else pr[0]
            cs[h, :n] += gm.sum(dim=0).to(td).float()
    return out, bound, cs


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
        ref_out, tol, ref_cs = reference(q[0], k[0], v[0], dt)
        got = out[0].float()
        err = (got - ref_out).abs()
        ratio = float((err / (tol + 1e-30)).max())
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
