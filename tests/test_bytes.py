"""Algorithmic HBM bytes used by the rooflines (CPU only).

bench.py's roofline divides StickyLlamaDecoder.attention_bytes_per_layer by the
measured launch time, the microbenchmark divides microbench.algorithmic_bytes;
both restate B*H*[S_m*2*D*e + S_q*(2*qb + 2*e) + Wq*2*D*e] and must agree."""

from types import SimpleNamespace

import torch

from qevict_b200.microbench import algorithmic_bytes
from qevict_b200.model import LlamaShape, StickyLlamaDecoder, StickyShape


def _decoder_shape(**sticky):
    return SimpleNamespace(s=LlamaShape(), k=StickyShape(**sticky), B=1, dtype=torch.bfloat16)


def test_attention_bytes_formulas_agree():
    m = _decoder_shape()
    for t in (1, 17, 64):
        assert StickyLlamaDecoder.attention_bytes_per_layer(m, t) == algorithmic_bytes(1, 32, 32, 512, t)


def test_attention_bytes_by_hand():
    # full-model layer, t = 1: S_m = 64 + 32*64 + 512 + 1 = 2625 bf16 tokens, S_q = 2048 INT8 tokens
    per_head = 2625 * 2 * 128 * 2 + 2048 * (2 * 128 + 2 * 2) + 32 * 2 * 128 * 2
    assert StickyLlamaDecoder.attention_bytes_per_layer(_decoder_shape(), 1) == 8 * per_head
    # INT4 codes are half a byte per element
    m4 = _decoder_shape(bits=4)
    per_head4 = 2625 * 2 * 128 * 2 + 2048 * (2 * 64 + 2 * 2) + 32 * 2 * 128 * 2
    assert StickyLlamaDecoder.attention_bytes_per_layer(m4, 1) == 8 * per_head4


def test_batch64_microbenchmark_bytes():
    # 64 sequences x (64 + 512 + 2048 bf16 tokens + t, 4096 INT8 tokens): 1.258 GB per
    # launch on average over the window position t = 1..64
    mean = sum(algorithmic_bytes(64, 32, 64, 512, t) for t in range(1, 65)) / 64
    assert abs(mean - 1.2583e9) / 1.2583e9 < 1e-3
