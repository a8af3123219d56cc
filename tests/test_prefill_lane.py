"""Prefill lane (qv_prefill_attention) against the oracle.

The causal output is compared with the exact (float64, rounded once) causal
attention; the per-key column sums with the reference's chunked scorer
(ops_flash.py:56-141): rounded logits, fp32 softmax, probabilities rounded to
the KV dtype, group mean rounded, per-512-query-chunk sums rounded, chunks
accumulated in fp32.  Tolerances: outputs 1e-5 absolute (fp32, CUDA-core
lane) and 2e-2 + 1e-2 * |ref| (bf16: the tensor-core lane rounds P to bf16
before P.V, as the reference's flash-attention path does); column sums 1e-5 /
2e-2 relative (the fp32 softmax normaliser is summed in another order, which
can move a rounded probability by one ulp).
Sizes cross the 512-query chunk boundary; GQA group 4 and MHA.
"""

import numpy as np
import pytest
import torch

from oracle.prefill import causal_attention, chunked_prefill_scores

pytestmark = pytest.mark.gpu

TD = {"fp32": torch.float32, "bf16": torch.bfloat16}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


@pytest.mark.parametrize("dt", ["fp32", "bf16"])
@pytest.mark.parametrize("Hq,H,D,S", [(8, 2, 128, 600), (2, 2, 64, 1100)])
def test_prefill_lane_vs_oracle(dt, Hq, H, D, S):
    from qevict_b200.model import prefill_attention
    g = torch.Generator().manual_seed(S + Hq)
    q = torch.randn(1, S, Hq, D, generator=g).to(TD[dt])
    k = torch.randn(1, S, H, D, generator=g).to(TD[dt])
    v = torch.randn(1, S, H, D, generator=g).to(TD[dt])
    out, cs = prefill_attention(q.cuda().contiguous(), k.cuda().contiguous(), v.cuda().contiguous())
    qn = q[0].float().numpy().transpose(1, 0, 2)
    kn = k[0].float().numpy().transpose(1, 0, 2)
    vn = v[0].float().numpy().transpose(1, 0, 2)
    ref_out = causal_attention(qn, kn, vn, dt)
    got = out[0].float().cpu().numpy().transpose(1, 0, 2)
    atol, rtol = (1e-5, 0.0) if dt == "fp32" else (2e-2, 1e-2)
    np.testing.assert_allclose(got, ref_out, atol=atol, rtol=rtol)
    ref_cs = chunked_prefill_scores(qn, kn, dt)
    rtol = 1e-5 if dt == "fp32" else 2e-2
    np.testing.assert_allclose(cs[0].cpu().numpy(), ref_cs, rtol=rtol, atol=1e-6)
