"""Prefill lane (qv_prefill_attention) against the oracle, at sizes that cross the
512-query chunk boundary (GQA groups 1, 2, 4 and 8; head_dim 64 and 128;
lengths that end inside a query block).

* fp32 (CUDA-core lane): the output against the exact causal attention
  (oracle.prefill.causal_attention, float64 rounded once) within 1e-5, and the
  per-key column sums against the reference's chunked scorer
  (oracle.prefill.chunked_prefill_scores, ops_flash.py:56-141) within 1e-5
  relative;
* bf16 / fp16 (tensor-core lane at head_dim 128): the output within the per-element bound
  derived from the reference's rounding points (tests/test_prefill_long.py,
  which states it), and the column sums against the oracle's chunked scorer
  within one ulp of a chunk sum plus one of a probability (relative).
"""

import numpy as np
import pytest
import torch

from oracle.prefill import causal_attention, chunked_prefill_scores
from test_prefill_long import CS_RTOL, reference

pytestmark = pytest.mark.gpu

TD = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


@pytest.mark.parametrize("dt", ["fp32", "bf16", "fp16"])
@pytest.mark.parametrize("Hq,H,D,S", [(8, 2, 128, 600), (2, 2, 64, 1100), (16, 2, 128, 700), (4, 2, 128, 517),
                                      (8, 1, 64, 530)])
def test_prefill_lane_vs_oracle(dt, Hq, H, D, S):
    from qevict_b200.model import prefill_attention
    g = torch.Generator().manual_seed(S + Hq)
    q = torch.randn(1, S, Hq, D, generator=g).to(TD[dt]).cuda().contiguous()
    k = torch.randn(1, S, H, D, generator=g).to(TD[dt]).cuda().contiguous()
    v = torch.randn(1, S, H, D, generator=g).to(TD[dt]).cuda().contiguous()
    out, cs = prefill_attention(q, k, v)
    qn = q[0].float().cpu().numpy().transpose(1, 0, 2)
    kn = k[0].float().cpu().numpy().transpose(1, 0, 2)
    vn = v[0].float().cpu().numpy().transpose(1, 0, 2)
    got = out[0].float()
    ref_cs = chunked_prefill_scores(qn, kn, dt)
    if dt == "fp32":
        ref_out = causal_attention(qn, kn, vn, dt)
        np.testing.assert_allclose(got.cpu().numpy().transpose(1, 0, 2), ref_out, atol=1e-5, rtol=0.0)
        np.testing.assert_allclose(cs[0].cpu().numpy(), ref_cs, rtol=1e-5, atol=1e-6)
        return
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref_out, tol, _ = reference(q[0], k[0], v[0], dt)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    err = (got - ref_out).abs()
    assert bool((err <= tol).all()), f"output beyond the bound: worst err/bound {float((err / tol).max())}"
    rel = np.abs(cs[0].cpu().numpy() - ref_cs) / np.maximum(np.abs(ref_cs), 1e-30)
    assert float(rel.max()) <= CS_RTOL[dt], float(rel.max())
