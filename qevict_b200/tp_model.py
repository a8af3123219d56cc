"""A Llama-3-shaped decoder split over the GPUs of one node by KV head.

Rank r of N holds KV heads [r H/N, (r+1) H/N) of every layer with their query
heads, and the matching slices of every projection:

  * q/k/v (column-parallel): the rows of this rank's heads -- the attention,
    its Sticky-KV state (sticky windows, Q-cache, vote ledger) and its eviction
    cycle are per head, so they run on the rank with no exchange;
  * o_proj (row-parallel): the columns of this rank's heads, giving a partial
    [B, hidden] that one all-reduce (sum) completes -- the exchange of the
    attention outputs: each rank's heads enter every output element through
    W_o, so the all-gather of head outputs and the replicated projection are
    one all-reduce of the projected sum;
  * gate/up (column-parallel) and down (row-parallel): the FFN split in
    1/N, one all-reduce;
  * the LM head (vocabulary-parallel): each rank's share of the logits, its
    best (value, index) packed into one int64 and a MAX all-reduce picks the
    greedy token (smallest index among equal values, as torch.argmax).

Per eviction cycle each layer takes one MIN all-reduce of a [B] int32 count:
the reference's only coupling between heads (eviction_manager.py:335-345,
the number of Q-cache losers is the minimum over heads), through
qv_evict_cycle_count / qv_evict_cycle_ext.  The decode-size sums
([B, hidden] bf16) go through qv_peer_sum (one kernel: epoch-tagged stores
into every rank's buffer over NVLink, a rank-order sum), and so does the
greedy token's MAX (qv_peer_max_i64); the prefill's large sums and the
cycle's MIN are NCCL calls.  All run on the decode stream, captured with the
kernels in the step's CUDA graph.

Weights are random (uniform-free normal, std 0.02), each matrix drawn whole
from a generator seeded by (seed, layer, matrix) and then sliced, so the N-rank
model and the one-rank model hold the same global weights.
"""

import ctypes
import math

import torch
import torch.nn.functional as F

from . import _native as N
from .layer_state import StickyLayerState
from .model import LlamaShape, StickyShape, prefill_attention, rope_, rope_tables


def _draw(shape, seed, device, std, dtype):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std).to(dtype)


class TpStickyLlamaDecoder:
    """This rank's share of a KV-head-parallel Llama decoder (batch B, greedy decode)."""

    def __init__(self, shape: LlamaShape, sticky: StickyShape, rank, world, group=None, batch=1, max_pos=40960,
                 dtype=torch.bfloat16, device="cuda", seed=0, std=0.02, peer_sum=True):
        import torch.distributed as dist
        s = shape
        if s.kv_heads % world or s.ffn % world or s.vocab % world:
            raise N.QevictError(f"{world} ranks do not divide the KV heads / FFN / vocabulary")
        self.dist, self.group = dist, group
        self.s, self.k, self.B, self.rank, self.world = shape, sticky, batch, rank, world
        self.dtype, self.device = dtype, torch.device(device)
        H, Hq, D = s.kv_heads, s.heads, s.head_dim
        G = Hq // H
        self.hl, self.ql, self.G = H // world, Hq // world, G
        self.f = s.ffn // world
        self.vl = s.vocab // world
        hl, ql, f, vl = self.hl, self.ql, self.f, self.vl
        dev = self.device

        def mat(layer, idx, shape_):
            return _draw(shape_, (seed * 1000003 + layer * 16 + idx) & 0x7FFFFFFFFFFF, dev, std, dtype)

        self.embed = mat(99999, 0, (s.vocab, s.hidden))
        self.layers = []
        for li in range(s.layers):
            wq = mat(li, 0, (Hq * D, s.hidden))[rank * ql * D:(rank + 1) * ql * D]
            wk = mat(li, 1, (H * D, s.hidden))[rank * hl * D:(rank + 1) * hl * D]
            wv = mat(li, 2, (H * D, s.hidden))[rank * hl * D:(rank + 1) * hl * D]
            wo = mat(li, 3, (s.hidden, Hq * D))[:, rank * ql * D:(rank + 1) * ql * D].contiguous()
            wgu = mat(li, 4, (2 * s.ffn, s.hidden))
            wgu = torch.cat([wgu[rank * f:(rank + 1) * f], wgu[s.ffn + rank * f:s.ffn + (rank + 1) * f]]).contiguous()
            wd = mat(li, 5, (s.hidden, s.ffn))[:, rank * f:(rank + 1) * f].contiguous()
            self.layers.append(dict(ln1=torch.ones(s.hidden, dtype=dtype, device=dev),
                                    wqkv=torch.cat([wq, wk, wv]).contiguous(), wo=wo,
                                    ln2=torch.ones(s.hidden, dtype=dtype, device=dev), wgu=wgu, wd=wd))
            del wq, wk, wv
        self.norm = torch.ones(s.hidden, dtype=dtype, device=dev)
        self.lm_head = mat(99999, 1, (s.vocab, s.hidden))[rank * vl:(rank + 1) * vl].contiguous()
        self.cos, self.sin = rope_tables(max_pos, D, s.rope_theta, dtype, dev)
        self.max_pos = max_pos
        max_windows = max((max_pos - sticky.sink) // sticky.omega, 100)
        self.states = [StickyLayerState(batch, hl, G, D, sticky.omega, sticky.sink, sticky.local, sticky.k_windows,
                                        sticky.q_windows, max_windows, sticky.bits, dtype, dev)
                       for _ in range(s.layers)]
        self.counts = [torch.zeros(batch, dtype=torch.int32, device=dev) for _ in range(s.layers)]
        B = batch
        self.tok = torch.zeros(B, dtype=torch.long, device=dev)
        self.next_tok = torch.zeros(B, dtype=torch.long, device=dev)
        self.x = torch.empty(B, s.hidden, dtype=dtype, device=dev)
        self.h = torch.empty_like(self.x)
        self.proj = torch.empty_like(self.x)
        self.qkv = torch.empty(B, (ql + 2 * hl) * D, dtype=dtype, device=dev)
        self.attn_out = torch.empty(B, ql, D, dtype=dtype, device=dev)
        self.gu = torch.empty(B, 2 * f, dtype=dtype, device=dev)
        self.act = torch.empty(B, f, dtype=dtype, device=dev)
        self.logits = torch.empty(B, vl, dtype=dtype, device=dev)
        self.key = torch.empty(B, dtype=torch.int64, device=dev)
        self.graphs = {}
        # the decode-size all-reduces ([B, hidden] bf16) over NVLink peer memory
        self.ps = None
        if peer_sum and world > 1 and dev.type == "cuda" and dtype == torch.bfloat16:
            from .peer_sum import PeerSum
            self.ps = PeerSum(rank, world, group, max_bytes=max(64 * 1024, -(-B * s.hidden * 2 // 16) * 16))

    # ------------------------------------------------------------ collectives
    def _sum(self, t):
        if self.world > 1:
            if self.ps is not None and self.ps.fits(t):
                self.ps.sum_(t)
            else:
                self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM, group=self.group)

    def close(self):
        """Release the captured graphs and the peer-sum buffer (every rank, after
        its last step; the ranks synchronise here)."""
        self.graphs.clear()
        if self.ps is not None:
            torch.cuda.synchronize(self.device)
            if self.world > 1:
                self.dist.barrier(group=self.group)
            self.ps.close()
            self.ps = None

    def _greedy(self, logits):
        """Greedy token over the vocabulary shards: the local best value and index
        packed into an int64 (value bits ordered like the float, index inverted
        so that the smaller index wins a tie) and a MAX all-reduce."""
        val, idx = logits.float().max(dim=-1)
        bits = val.view(torch.int32).to(torch.int64)
        ordered = torch.where(bits >= 0, bits, bits ^ 0x7FFFFFFF)          # monotone in the float value
        gidx = idx.to(torch.int64) + self.rank * self.vl
        self.key.copy_((ordered << 32) | (0xFFFFFFFF - gidx))
        if self.world > 1:
            if self.ps is not None:
                self.ps.max_(self.key)
            else:
                self.dist.all_reduce(self.key, op=self.dist.ReduceOp.MAX, group=self.group)
        return 0xFFFFFFFF - (self.key & 0xFFFFFFFF)

    # ---------------------------------------------------------------- prefill
    @torch.no_grad()
    def prefill(self, ids, mlp_chunk=8192):
        """ids [B, S] (the same on every rank) -> first generated token [B]."""
        s = self.s
        B, S = ids.shape
        ql, hl, D = self.ql, self.hl, s.head_dim
        x = self.embed[ids]
        for li, L in enumerate(self.layers):
            h = F.rms_norm(x, (s.hidden,), L["ln1"], s.rms_eps)
            qkv = h @ L["wqkv"].t()
            del h
            q = qkv[..., :ql * D].reshape(B, S, ql, D).contiguous()
            k = qkv[..., ql * D:(ql + hl) * D].reshape(B, S, hl, D).contiguous()
            v = qkv[..., (ql + hl) * D:].reshape(B, S, hl, D).contiguous()
            del qkv
            rope_(q, self.cos, self.sin)
            rope_(k, self.cos, self.sin)
            o, cs = prefill_attention(q, k, v)
            del q
            self.states[li].prefill(k.transpose(1, 2).contiguous(), v.transpose(1, 2).contiguous(), cs)
            del k, v, cs
            part = o.reshape(B, S, ql * D) @ L["wo"].t()
            del o
            self._sum(part)
            x = x + part
            del part
            for i in range(0, S, mlp_chunk):
                xc = x[:, i:i + mlp_chunk]
                hc = F.rms_norm(xc, (s.hidden,), L["ln2"], s.rms_eps)
                gu = hc @ L["wgu"].t()
                part = (F.silu(gu[..., :self.f]) * gu[..., self.f:]) @ L["wd"].t()
                del gu, hc
                self._sum(part)
                x[:, i:i + mlp_chunk] = xc + part
        h = F.rms_norm(x[:, -1], (s.hidden,), self.norm, s.rms_eps)
        nxt = self._greedy(h @ self.lm_head.t())
        self.tok.copy_(nxt)
        return nxt

    # ----------------------------------------------------------------- decode
    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def _add_norm(self, delta, weight):
        rc = N.lib().qv_add_rmsnorm(self.B, self.s.hidden, N.ptr(self.x), N.ptr(delta), N.ptr(weight),
                                    self.s.rms_eps, N.ptr(self.h), self._stream())
        N.check(rc, "qv_add_rmsnorm")

    def _gemv(self, w, x, y):
        rc = N.lib().qv_gemv(self.B, w.shape[0], w.shape[1], N.ptr(w), N.ptr(x), N.ptr(y), self._stream())
        N.check(rc, "qv_gemv")

    def _layer_step(self, li, cycle):
        s, L, st = self.s, self.layers[li], self.states[li]
        B, ql, hl, D = self.B, self.ql, self.hl, s.head_dim
        self._gemv(L["wqkv"], self.h, self.qkv)
        q = self.qkv[:, :ql * D].view(B, ql, D)
        k = self.qkv[:, ql * D:(ql + hl) * D].view(B, hl, D)
        v = self.qkv[:, (ql + hl) * D:].view(B, hl, D)
        qr = st.append(q, k, v, self.cos, self.sin)
        st.attend(qr, self.attn_out)
        if cycle:
            # the cycle's one coupling between heads: the minimum loser count
            c = self.counts[li]
            rc = N.lib().qv_evict_cycle_count(ctypes.byref(st.dims), ctypes.byref(st.layer), N.ptr(st.ws.cycle),
                                              st.ws.cycle_bytes, N.ptr(c), self._stream())
            N.check(rc, "qv_evict_cycle_count")
            if self.world > 1:
                self.dist.all_reduce(c, op=self.dist.ReduceOp.MIN, group=self.group)
            rc = N.lib().qv_evict_cycle_ext(ctypes.byref(st.dims), ctypes.byref(st.layer), N.ptr(st.ws.cycle),
                                            st.ws.cycle_bytes, N.ptr(c), self._stream())
            N.check(rc, "qv_evict_cycle_ext")
        self._gemv(L["wo"], self.attn_out, self.proj)
        self._sum(self.proj)
        self._add_norm(self.proj, L["ln2"])
        self._gemv(L["wgu"], self.h, self.gu)
        rc = N.lib().qv_silu_mul(B, self.f, N.ptr(self.gu), N.ptr(self.act), self._stream())
        N.check(rc, "qv_silu_mul")
        self._gemv(L["wd"], self.act, self.proj)
        self._sum(self.proj)
        nxt = self.layers[li + 1]["ln1"] if li + 1 < s.layers else self.norm
        self._add_norm(self.proj, nxt)

    def _step_body(self, cycle):
        torch.index_select(self.embed, 0, self.tok, out=self.x)
        self._add_norm(None, self.layers[0]["ln1"])
        for li in range(self.s.layers):
            self._layer_step(li, cycle)
        self._gemv(self.lm_head, self.h, self.logits)
        self.next_tok.copy_(self._greedy(self.logits))
        self.tok.copy_(self.next_tok)

    def cycle_next(self):
        st = self.states[0]
        return (st.n_tokens + 1 - st.prompt_len) % st.omega == 0

    def _advance(self, cycle):
        for st in self.states:
            st.n_tokens += 1
            if cycle:
                st.last_compaction = st.n_tokens

    @torch.no_grad()
    def step_eager(self):
        cycle = self.cycle_next()
        saved = [st.n_tokens for st in self.states]
        self._step_body(cycle)
        # attend() advanced the host counters; the cycle's bookkeeping follows
        for st, n in zip(self.states, saved):
            st.n_tokens = n
        self._advance(cycle)
        return self.next_tok

    @torch.no_grad()
    def capture(self):
        """Capture the plain and the cycle step (collectives included) into CUDA graphs."""
        saved = [(st.n_tokens, st.last_compaction) for st in self.states]
        for cycle in (False, True):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                self._step_body(cycle)
            self.graphs[cycle] = gr
            for st, (n, lc) in zip(self.states, saved):
                st.n_tokens, st.last_compaction = n, lc

    def step_graph(self):
        cycle = self.cycle_next()
        self.graphs[cycle].replay()
        self._advance(cycle)
        return cycle

    def attention_bytes_per_layer(self, t_mean):
        """Algorithmic HBM bytes of this rank's fused decode-attention launch per layer."""
        k, s = self.k, self.s
        e = torch.finfo(self.dtype).bits // 8
        qb = s.head_dim if k.bits == 8 else s.head_dim // 2
        s_m = k.sink + k.k_windows * k.omega + k.local + t_mean
        s_q = k.q_windows * k.omega
        return self.B * self.hl * (s_m * 2 * s.head_dim * e + s_q * (2 * qb + 2 * e) + k.q_windows * 2 * s.head_dim * e)

    def weight_bytes(self):
        n = sum(L[k].numel() for L in self.layers for k in ("wqkv", "wo", "wgu", "wd")) + self.lm_head.numel()
        return n * torch.finfo(self.dtype).bits // 8
