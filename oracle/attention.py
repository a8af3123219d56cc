"""Decode attention over the mixed cache, restated in numpy (test infrastructure only).

One sequence, one query token.  Follows the reference's SDPA decode path:
  * GQA logits ``q . K^T / sqrt(D)``                      (attention/ops.py:23-46)
  * Q-cache dequantisation + logits, joint fp32 softmax
    over [main | q], probabilities cast to the KV dtype,
    P.V for both zones, GQA-group-mean probabilities      (attention/ops.py:74-169)
  * the same without a Q-cache                           (attention/ops.py:176-212)

Rounding points are the reference's: each matmul output rounded to the KV
dtype, the ``/ sqrt(D)`` rounded, softmax in fp32, probabilities rounded, the
group mean rounded, ``out_main + out_q`` rounded.  Matmuls accumulate in
float64 here (torch accumulates in fp32), so logits can differ from the
reference by one unit in the last place of the KV dtype; comparisons of
attention outputs and ledger values therefore use a stated tolerance.
"""

import math

import numpy as np

from .codec import dequantize_from_quant
from .numerics import f32, op, rnd, mean_round


def _logits(q, k, dt):
    """q [H, G, D], k [H, S, D] -> logits [H, G, S] in dt (ops.py:35-41)."""
    raw = np.einsum("hgd,hsd->hgs", q.astype(np.float64), k.astype(np.float64))
    raw = rnd(raw, dt)
    return op(np.divide, dt, raw, np.float32(math.sqrt(q.shape[-1])))


def decode_attention(q, k_main, v_main, dt, qcache=None, bit_width=8):
    """Attention of one decode token.

    q        [Hq, D]  rotated query (values in dt)
    k_main   [H, S, D], v_main [H, S, D] physical main cache incl. the new token
    qcache   None or dict(kq [H,W,w,D] u8, ks [H,W,1,D], kz [H,W,1,D],
                          vq [H,W,w,D] u8, vs [H,W,w,1], vz [H,W,w,1])
    Returns (out [Hq, D] in dt, scores_main [H, S] in dt, scores_q [H, W*w] in dt or None)
    """
    q = f32(q)
    H, S, D = k_main.shape
    G = q.shape[0] // H
    qg = q.reshape(H, G, D)
    main = _logits(qg, f32(k_main), dt)  # [H, G, S]
    if qcache is not None:
        kdq = dequantize_from_quant(qcache["kq"], qcache["ks"], qcache["kz"], dt, bit_width)
        vdq = dequantize_from_quant(qcache["vq"], qcache["vs"], qcache["vz"], dt, bit_width)
        Hc, W, w, _ = kdq.shape
        kdq = kdq.reshape(H, W * w, D)
        vdq = vdq.reshape(H, W * w, D)
        ql = _logits(qg, kdq, dt)
        all_l = np.concatenate([main, ql], axis=-1)
    else:
        all_l = main
    x = all_l.astype(np.float64)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    p = (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
    p = rnd(p, dt)
    pm = p[..., :S]
    out = rnd(np.einsum("hgs,hsd->hgd", pm.astype(np.float64), f32(v_main).astype(np.float64)), dt)
    scores_q = None
    if qcache is not None:
        pq = p[..., S:]
        out_q = rnd(np.einsum("hgs,hsd->hgd", pq.astype(np.float64), vdq.astype(np.float64)), dt)
        out = op(np.add, dt, out, out_q)
        scores_q = mean_round(pq, 1, dt)
    scores_main = mean_round(pm, 1, dt)
    return out.reshape(H * G, D), scores_main, scores_q
