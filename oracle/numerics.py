"""Element-type emulation for the oracle (test infrastructure only).

PyTorch's CPU kernels evaluate a bf16/fp16 elementwise op by widening both
operands to fp32, computing in fp32 and rounding the result back to the tensor
dtype with round-to-nearest-even.  Reductions (``sum``/``mean``) accumulate in
fp32 and round once at the end.  The helpers below reproduce exactly that on
numpy float32 arrays whose values are representable in the emulated dtype.
"""

import numpy as np

DTYPES = ("fp32", "bf16", "fp16")


def f32(x):
    return np.asarray(x, dtype=np.float32)


def _bf16_rne(x32):
    """Round float32 values to the nearest bfloat16 (ties to even), as float32.

    In uint32 arithmetic: add 0x7FFF plus the lowest kept bit, then clear the
    low 16 bits.  No finite input overflows (the largest, 0xFF7FFFFF + 0x8000,
    stays below 2^32; infinities map to themselves); NaNs are restored after."""
    x32 = np.ascontiguousarray(x32, dtype=np.float32)
    u = x32.view(np.uint32)
    r = u >> 16
    r &= 1
    r += 0x7FFF
    r += u
    r &= 0xFFFF0000
    out = r.view(np.float32)
    nan = np.isnan(x32)
    if nan.any():
        out[nan] = np.float32(np.nan)
    return out


def rnd(x, dt):
    """Round float values to dtype ``dt`` ("fp32" | "bf16" | "fp16"), returned as float32."""
    x = np.asarray(x)
    x32 = x.astype(np.float32)
    if dt == "fp32":
        return x32
    if dt == "bf16":
        return _bf16_rne(x32)
    if dt == "fp16":
        with np.errstate(over="ignore"):
            return x32.astype(np.float16).astype(np.float32)
    raise ValueError(dt)


def op(fn, dt, *args):
    """Evaluate ``fn`` on fp32 operands and round the result to ``dt`` (one torch op)."""
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        return rnd(fn(*[f32(a) for a in args]), dt)


def sum_round(x, axis, dt):
    """torch ``x.sum(dim)`` on a dtype-``dt`` tensor: fp32 accumulation, one rounding."""
    return rnd(np.sum(f32(x).astype(np.float64), axis=axis), dt)


def mean_round(x, axis, dt):
    """torch ``x.mean(dim)`` on a dtype-``dt`` tensor: fp32 sum / n, one rounding."""
    x = f32(x)
    n = x.shape[axis]
    s = np.sum(x, axis=axis, dtype=np.float32)
    return rnd(s / np.float32(n), dt)


def tree_sum32(x):
    """Sum the last axis (one window's omega values, omega <= 128) in warp order.

    Lane l (0..31) accumulates x[l], x[l+32], x[l+64], ... sequentially in fp32;
    the 32 lanes then combine by xor-butterfly over offsets 16, 8, 4, 2, 1.
    The CUDA scoreboard kernel sums each window's votes in exactly this order,
    so the oracle uses it too when it must agree with the kernel bit-for-bit.
    """
    x = f32(x)
    n = x.shape[-1]
    a = np.zeros(x.shape[:-1] + (32,), np.float32)
    for lane in range(min(32, n)):
        acc = x[..., lane]
        for i in range(lane + 32, n, 32):
            acc = (acc + x[..., i]).astype(np.float32)
        a[..., lane] = acc
    off = 16
    idx = np.arange(32)
    while off >= 1:
        a = (a + a[..., idx ^ off]).astype(np.float32)
        off //= 2
    return a[..., 0]


def to_uint8_like_torch(x):
    """``.to(torch.uint8)`` of values already clamped to [0, 255]; NaN maps to 0 (x86 behaviour)."""
    x = f32(x)
    out = np.where(np.isnan(x), 0.0, x)
    return np.trunc(out).astype(np.uint8)
