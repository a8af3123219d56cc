"""The arithmetic identities the tensor-core prefill lane relies on
(qevict_b200/csrc/prefill_tc.cu), checked over every 16-bit input.

The reference scales the rounded logit by sqrt(D) with an fp32 division
(src/models/attention/ops.py:23-46: matmul(...) / math.sqrt(head_dim), the
result rounded to the KV dtype).  The lane multiplies by the fp32 reciprocal
instead:

* bf16 (D = 64 and 128) and fp16 at D = 64: round(x * fl(1/sqrt(D))) equals
  round(fl(x / sqrt(D))) for every value x of the dtype;
* fp16 at D = 128: the plain product differs for some inputs; one residual
  step q' = fma(fma(-q, sqrt(D), x), 1/sqrt(D), q) makes it equal in value for
  every x (-0 becomes +0).
The fused multiply-adds are evaluated exactly (rational arithmetic) and
rounded once to fp32, as the hardware does.
"""

from fractions import Fraction

import numpy as np
import pytest
import torch

TD = {"bf16": torch.bfloat16, "fp16": torch.float16}


def _all_values(dt):
    bits = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16)
    x = bits.view(TD[dt]).float().numpy()
    return x[np.isfinite(x)]


def _to_dt(a, dt):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(TD[dt]).view(torch.int16).numpy()


def _f32(fr):
    """Fraction -> the nearest fp32 (ties to even)."""
    c = np.float32(float(fr))
    best = None
    for cand in (np.nextafter(c, np.float32(-np.inf)), c, np.nextafter(c, np.float32(np.inf))):
        d = abs(Fraction(float(cand)) - fr)
        even = (int(np.float32(cand).view(np.uint32)) & 1) == 0
        key = (d, not even)
        if best is None or key < best[0]:
            best = (key, cand)
    return np.float32(best[1])


def _fma(a, b, c):
    return _f32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


@pytest.mark.parametrize("dt,D", [("bf16", 64), ("bf16", 128), ("fp16", 64)])
def test_reciprocal_multiply_is_exact(dt, D):
    x = _all_values(dt)
    sd = np.float32(np.sqrt(np.float32(D)))
    assert float(torch.tensor(float(D)).sqrt()) == float(sd)
    inv = np.float32(1.0) / sd
    with np.errstate(all="ignore"):
        ref = _to_dt(x / sd, dt)
        got = _to_dt(x * inv, dt)
    assert np.array_equal(ref, got)


def test_fp16_d128_needs_and_gets_one_correction():
    dt, D = "fp16", 128
    x = _all_values(dt)
    sd = np.float32(np.sqrt(np.float32(D)))
    inv = np.float32(1.0) / sd
    with np.errstate(all="ignore"):
        ref = _to_dt(x / sd, dt)
        plain = _to_dt(x * inv, dt)
    assert int((ref != plain).sum()) > 0    # the plain product is not enough here
    q = (x * inv).astype(np.float32)
    fixed = np.empty_like(q)
    for i in range(x.size):                  # every input
        e = _fma(-q[i], sd, x[i])
        fixed[i] = _fma(e, inv, q[i])
    # equal values (the correction turns the quotient of -0 into +0, the same logit)
    got = torch.from_numpy(_to_dt(fixed, dt)).view(torch.float16).float().numpy()
    want = torch.from_numpy(ref).view(torch.float16).float().numpy()
    assert np.array_equal(got, want)
