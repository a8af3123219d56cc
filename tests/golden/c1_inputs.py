"""Seeded inputs of the single-layer fp32 workload (one Llama attention layer,
hidden 4096, 32 query / 8 KV heads, a 4096-token prompt, 256 decode steps).

Shared by make_golden.py, which runs the reference on them, and by the GPU
test that runs this library's module on the same arrays, so the two never
need to exchange the inputs themselves (only the reference's outputs are
stored, in module_c1_fp32.npz).
"""

import numpy as np

C1 = dict(hidden=4096, heads=32, kv_heads=8, omega=64, sink=64, local=256, k_windows=16, q_windows=16,
          prompt=4096, steps=256, seed=1001)


def c1_inputs(c=C1):
    """q/k/v/o weights ~ N(0, 0.02) ([out, in], nn.Linear layout), prompt hidden
    states [prompt, hidden] ~ N(0, 1), decode hidden states [steps, hidden]
    ~ N(0, 1), drawn in that order from one numpy generator (float32)."""
    rng = np.random.default_rng(c["seed"])
    hd = c["hidden"] // c["heads"]
    hid, kvd = c["hidden"], c["kv_heads"] * hd
    w = {}
    for name, shape in (("q", (hid, hid)), ("k", (kvd, hid)), ("v", (kvd, hid)), ("o", (hid, hid))):
        w[name] = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
    hs = rng.standard_normal((c["prompt"], hid), dtype=np.float32)
    dec = rng.standard_normal((c["steps"], hid), dtype=np.float32)
    return w, hs, dec
