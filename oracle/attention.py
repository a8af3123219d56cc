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


def _exact_dequant(codes, scale, zp, bit_width):
    """code * scale + zp without intermediate rounding (float64): the tensor-core
    kernel's dequantisation, in place of dequantize_from_quant's per-op rounding
    to the KV dtype (quantize.py:62-71); INT4 codes unpacked high nibble first."""
    codes = np.asarray(codes)
    if bit_width == 4:
        hi = (codes >> 4) & 0x0F
        lo = codes & 0x0F
        codes = np.stack([hi, lo], axis=-1).reshape(*codes.shape[:-1], -1)
    return codes.astype(np.float64) * np.asarray(scale, np.float64) + np.asarray(zp, np.float64)


def _ulp(x, dt):
    """One unit in the last place of dtype dt at |x| (float64 array)."""
    bits = {"fp32": 23, "bf16": 7, "fp16": 10}[dt]
    ax = np.maximum(np.abs(np.asarray(x, np.float64)), 1e-30)
    return 2.0 ** (np.floor(np.log2(ax)) - bits)


def _logits(q, k, dt, raw=False):
    """q [H, G, D], k [H, S, D] -> logits [H, G, S] in dt (ops.py:35-41)."""
    r = np.einsum("hgd,hsd->hgs", q.astype(np.float64), k.astype(np.float64))
    lg = op(np.divide, dt, rnd(r, dt), np.float32(math.sqrt(q.shape[-1])))
    return (lg, r) if raw else lg


def exact_dequant_qcache(qcache, bit_width=8):
    """(kdq, vdq) float64 [H, W, w, D] of a Q-cache dict, dequantised exactly
    (code * scale + zp): pass them back in ``qcache`` as "kdq"/"vdq" to skip the
    work on every step while the Q-cache does not change."""
    return (_exact_dequant(qcache["kq"], qcache["ks"], qcache["kz"], bit_width),
            _exact_dequant(qcache["vq"], qcache["vs"], qcache["vz"], bit_width))


def decode_attention(q, k_main, v_main, dt, qcache=None, bit_width=8, dequant="reference",
                     logits_override=None, return_extras=False):
    """Attention of one decode token.

    dequant="reference" dequantises the Q-cache the way the reference does,
    rnd(rnd(code * scale) + zp) in the KV dtype (quantize.py:62-71);
    dequant="exact" applies scale and zero point without intermediate
    rounding (code * scale + zp in float64), which is what the tensor-core
    kernel computes.  The two differ by the reference's rounding of the
    intermediate code*scale (up to half an ulp of the KV dtype at |code*scale|,
    e.g. 2^-6 for values in [4, 8) in bf16).

    q        [Hq, D]  rotated query (values in dt)
    k_main   [H, S, D], v_main [H, S, D] physical main cache incl. the new token
    qcache   None or dict(kq [H,W,w,D] u8, ks [H,W,1,D], kz [H,W,1,D],
                          vq [H,W,w,D] u8, vs [H,W,w,1], vz [H,W,w,1]);
             with dequant="exact" it may also carry "kdq"/"vdq" from
             exact_dequant_qcache (reused instead of recomputed)
    logits_override: [H, G, S + W*w] rounded logits to use instead of the
        ones computed here (lets a test feed the kernel's own logits through the
        rest of the computation).
    Returns (out [Hq, D] in dt, scores_main [H, S] in dt, scores_q [H, W*w] in dt or None)
    and, with return_extras, a dict with the logits, the raw (pre-rounding) dot
    products, the bound on |kernel logit - oracle logit| per token, and the
    per-element magnitudes a tolerance on the output is derived from:
      out_ulps  ulp(out_main) + ulp(out_q) + ulp(out): the reference rounds the
                two zones' products and their sum separately (ops.py:132-150)
      abs_main  sum_t p_t |v_t| over the main zone   [Hq, D]
      abs_q     the same over the Q-cache            [Hq, D]
      abs_exp   sum_t p_t |v_t| (2 + 1.173 |x_t|), x_t = logit_t - max, both
                zones: the weight of the fast exponential's error, at most
                (2 + 1.173 |x|) fp32 ulps (CUDA's stated bound for __expf)
      vsum_main sum_t |v_t| over the main zone, vsum_q over the Q-cache
                [Hq, D]: the weight of an absolute error per probability
                (fp16 subnormals, below 2^-14, are spaced 2^-24 apart)
    """
    q = f32(q)
    H, S, D = k_main.shape
    G = q.shape[0] // H
    qg = q.reshape(H, G, D)
    kdq = vdq = None
    if qcache is not None:
        if dequant == "exact":
            if "kdq" in qcache:
                kdq, vdq = qcache["kdq"], qcache["vdq"]
            else:
                kdq, vdq = exact_dequant_qcache(qcache, bit_width)
        else:
            kdq = dequantize_from_quant(qcache["kq"], qcache["ks"], qcache["kz"], dt, bit_width)
            vdq = dequantize_from_quant(qcache["vq"], qcache["vs"], qcache["vz"], dt, bit_width)
        Hc, W, w, _ = kdq.shape
        kdq = kdq.reshape(H, W * w, D)
        vdq = vdq.reshape(H, W * w, D)
    need_logits = logits_override is None or return_extras
    if need_logits:
        main, raw_main = _logits(qg, f32(k_main), dt, raw=True)  # [H, G, S]
        fold = None
        if qcache is not None:
            ql, raw_q = _logits(qg, kdq, dt, raw=True)
            all_l = np.concatenate([main, ql], axis=-1)
            raw = np.concatenate([raw_main, raw_q], axis=-1)
        else:
            all_l = main
            raw = raw_main
    if logits_override is not None:
        all_l = f32(logits_override)
    x = all_l.astype(np.float64)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    p = (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
    p = rnd(p, dt)
    pm = p[..., :S]
    vm64 = f32(v_main).astype(np.float64)
    out = rnd(np.einsum("hgs,hsd->hgd", pm.astype(np.float64), vm64), dt)
    scores_q = None
    out_main, out_q = out, None
    if qcache is not None:
        pq = p[..., S:]
        vdq64 = np.asarray(vdq, np.float64)
        out_q = rnd(np.einsum("hgs,hsd->hgd", pq.astype(np.float64), vdq64), dt)
        out = op(np.add, dt, out, out_q)
        scores_q = mean_round(pq, 1, dt)
    scores_main = mean_round(pm, 1, dt)
    if not return_extras:
        return out.reshape(H * G, D), scores_main, scores_q
    # one ulp of the dtype at the rounded dot product, divided by sqrt(D), plus one
    # ulp at the logit, plus the fp16 scale-folding error of Q-cache tokens
    sd = math.sqrt(D)
    absdot = np.einsum("hgd,hsd->hgs", np.abs(qg.astype(np.float64)), np.abs(f32(k_main).astype(np.float64)))
    if qcache is not None:
        absdot = np.concatenate([absdot, np.einsum("hgd,hsd->hgs", np.abs(qg.astype(np.float64)),
                                                   np.abs(np.asarray(kdq, np.float64)))], axis=-1)
        if dequant == "exact":
            # the kernel folds the K scale into q and rounds q*scale to fp16
            codes = np.asarray(qcache["kq"])
            if bit_width == 4:
                codes = np.stack([(codes >> 4) & 15, codes & 15], -1).reshape(*codes.shape[:-1], -1)
            qs = np.abs(qg[:, :, None, None, :].astype(np.float64) * np.asarray(qcache["ks"], np.float64)[:, None])
            fold = np.einsum("hgwkd,hwtd->hgwt", qs, codes.astype(np.float64)) * 2.0 ** -11
            # fp32 accumulation of the 1024-offset products inside the MMA
            fold = fold + (np.sum(qs, axis=(3, 4))[..., None] * 1024.0 * 2.0 ** -20)
            fold = fold.reshape(H, G, -1)
    # fp32 accumulation of the D products (any order): at most ~64 u * sum|q_d k_d|
    acc = absdot * 64.0 * 2.0 ** -24
    bound = (_ulp(raw, dt) / sd + _ulp(all_l, dt) + acc / sd) * 1.01
    if fold is not None:
        bound[..., S:] += fold / sd
    # the reference rounds out_main and out_q separately and then their sum
    # (ops.py:150): an implementation whose pre-rounding values differ by a
    # hair can land one ulp away on any of the three
    out_ulps = _ulp(out_main, dt) + _ulp(out, dt)
    if out_q is not None:
        out_ulps = out_ulps + _ulp(out_q, dt)
    pf = p.astype(np.float64)
    ex = pf * (2.0 + 1.173 * np.abs(x - m))
    abs_main = np.einsum("hgs,hsd->hgd", pf[..., :S], np.abs(vm64))
    abs_exp = np.einsum("hgs,hsd->hgd", ex[..., :S], np.abs(vm64))
    abs_q = np.zeros_like(abs_main)
    vsum_main = np.broadcast_to(np.abs(vm64).sum(axis=1)[:, None, :], (H, G, D))
    vsum_q = np.zeros_like(vsum_main)
    if qcache is not None:
        abs_q = np.einsum("hgs,hsd->hgd", pf[..., S:], np.abs(vdq64))
        abs_exp = abs_exp + np.einsum("hgs,hsd->hgd", ex[..., S:], np.abs(vdq64))
        vsum_q = np.broadcast_to(np.abs(vdq64).sum(axis=1)[:, None, :], (H, G, D))
    return out.reshape(H * G, D), scores_main, scores_q, dict(
        logits=all_l, raw=raw, bound=bound, out_ulps=out_ulps.reshape(H * G, D),
        abs_main=abs_main.reshape(H * G, D), abs_q=abs_q.reshape(H * G, D),
        abs_exp=abs_exp.reshape(H * G, D), vsum_main=vsum_main.reshape(H * G, D),
        vsum_q=vsum_q.reshape(H * G, D))
