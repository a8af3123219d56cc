"""Prefill lane restated in numpy (test infrastructure only, small sizes).

* ``causal_attention``: the causal prefill output that the reference obtains
  from ``flash_attn_func`` (src/models/attention/ops_flash.py:22-49) or the SDPA
  branch (src/models/attention/module.py:258-304 with ops.py:53-67 and
  ops.py:176-212).  Computed in float64 and rounded once to the KV dtype.
* ``chunked_prefill_scores``: per-key column sums of the GQA-group-mean causal
  softmax, in 512-query chunks (src/models/attention/ops_flash.py:56-141):
  per chunk the probabilities are rounded to the KV dtype, group-averaged
  (rounded), summed over the chunk's queries (rounded to the KV dtype) and
  accumulated across chunks in fp32.
"""

import math

import numpy as np

from .numerics import f32, mean_round, op, rnd, sum_round


def causal_attention(q, k, v, dt):
    """Causal GQA attention of the prompt: q [Hq, S, D], k/v [H, S, D] -> out [Hq, S, D]
    (values in dt) -- the SDPA prefill of src/models/attention/module.py:258-304 with
    the causal mask of ops.py:53-67 (FA2 path: ops_flash.py:22-49)."""
    Hq, S, D = q.shape
    H = k.shape[0]
    G = Hq // H
    qg = f32(q).reshape(H, G, S, D).astype(np.float64)
    s = np.einsum("hgqd,hkd->hgqk", qg, f32(k).astype(np.float64)) / math.sqrt(D)
    mask = np.triu(np.ones((S, S), bool), 1)
    s = np.where(mask, -np.inf, s)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    out = np.einsum("hgqk,hkd->hgqd", p, f32(v).astype(np.float64))
    return rnd(out.reshape(Hq, S, D), dt)


def sdpa_causal_attention(q, k, v, dt):
    """The reference's SDPA prefill branch with its rounding points.

    module.py:258-304: logits rounded to dt and divided by sqrt(D) (ops.py:35-41),
    the causal mask applied in place with finfo(dt).min (ops.py:53-67), fp32
    softmax, probabilities rounded to dt, P.V rounded (ops.py:196-207).
    Returns (out [Hq, S, D], group-mean probabilities [H, S, S]) in dt.
    """
    Hq, S, D = q.shape
    H = k.shape[0]
    G = Hq // H
    qg = f32(q).reshape(H, G, S, D).astype(np.float64)
    raw = rnd(np.einsum("hgqd,hkd->hgqk", qg, f32(k).astype(np.float64)), dt)
    lg = op(np.divide, dt, raw, np.float32(math.sqrt(D)))
    minv = {"fp32": np.finfo(np.float32).min, "bf16": -3.3895313892515355e38, "fp16": -65504.0}[dt]
    lg = np.where(np.triu(np.ones((S, S), bool), 1), np.float32(minv), lg)
    x = lg.astype(np.float64)
    x = x - x.max(axis=-1, keepdims=True)
    e = np.exp(x)
    p = rnd((e / e.sum(axis=-1, keepdims=True)).astype(np.float32), dt)
    out = rnd(np.einsum("hgqk,hkd->hgqd", p.astype(np.float64), f32(v).astype(np.float64)), dt)
    return out.reshape(Hq, S, D), mean_round(p, 1, dt)


def chunked_prefill_scores(q, k, dt, past_len=0, chunk=512):
    """q [Hq, Sq, D], k [H, Sk, D] -> column sums [H, Sk] fp32 (ops_flash.py:56-141)."""
    Hq, Sq, D = q.shape
    H, Sk, _ = k.shape
    G = Hq // H
    acc = np.zeros((H, Sk), np.float32)
    kk = f32(k).astype(np.float64)
    minv = {"fp32": np.finfo(np.float32).min, "bf16": -3.3895313892515355e38,
            "fp16": -65504.0}[dt]
    for i in range(0, Sq, chunk):
        c = min(chunk, Sq - i)
        qc = f32(q[:, i:i + c]).reshape(H, G, c, D).astype(np.float64)
        raw = rnd(np.einsum("hgqd,hkd->hgqk", qc, kk), dt)
        lg = op(np.divide, dt, raw, np.float32(math.sqrt(D)))
        qi = np.arange(i, i + c)[:, None]
        kj = np.arange(Sk)[None, :]
        maskv = np.where(kj <= qi + past_len, np.float32(0.0), np.float32(minv))
        lg = op(np.add, dt, lg, maskv)
        x = lg.astype(np.float64)
        x = x - x.max(axis=-1, keepdims=True)
        e = np.exp(x)
        p = rnd((e / e.sum(axis=-1, keepdims=True)).astype(np.float32), dt)
        if G > 1:
            p = mean_round(p, 1, dt)
        else:
            p = p[:, 0]
        acc = (acc + f32(sum_round(p, 1, dt))).astype(np.float32)
    return acc
