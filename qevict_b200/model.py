"""A lean Llama-3-shaped decoder whose attention is the Sticky-KV hot path.

Used for the full-model decode workload (Llama-3-8B shape: 32 layers, hidden
4096, 32 query / 8 KV heads, head_dim 128, FFN 14336, vocab 128256).  A decode
step per layer: the projections are weight-streaming GEMVs (qv_gemv, each
launched as a programmatic dependent so its weight stream starts while the
kernel before it drains) into preallocated buffers, with the elementwise work
between them fused (qv_add_rmsnorm: residual add + the next RMSNorm;
qv_silu_mul: the MLP activation); attention runs the sm_100a
kernels: RoPE + append, fused decode attention with the ledger fold, and the
eviction cycle every omega tokens; the LM head's greedy token comes from one
argmax kernel (qv_argmax).  The prefill (prompt) path is torch/cuBLAS
around the prefill lane (causal attention + column sums -> state build).

Decode steps are captured in two CUDA graphs (a plain step and a step that
ends an omega-window and runs the eviction cycle of every layer); all
per-step indices live on the device, so the graphs replay unchanged.  With
side_fold, a plain step runs each layer's vote-ledger fold on a side stream
beside the layer's projections (the ledger only feeds the next eviction cycle)
and joins it at the step's end; each layer then has its own decode workspace.
A cycle step folds inline, since the cycle reads the ledger.  The default
folds inline: on a B200 the full-model step measured 3.74 ms inline against
3.81 ms with the side stream (batch 1, 32k context).
"""

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _native as N
from .layer_state import StickyLayerState, Workspace, kv_dtype_code


@dataclass
class LlamaShape:
    vocab: int = 128256
    hidden: int = 4096
    layers: int = 32
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5


@dataclass
class StickyShape:
    omega: int = 64
    sink: int = 64
    local: int = 512
    k_windows: int = 32
    q_windows: int = 32
    bits: int = 8


def rope_tables(max_pos, head_dim, theta, dtype, device):
    """HF default RoPE (transformers LlamaRotaryEmbedding): fp32 cos/sin cast to the model dtype."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64, device=device).float() / head_dim))
    t = torch.arange(max_pos, device=device, dtype=torch.float32)
    fr = torch.outer(t, inv)
    emb = torch.cat([fr, fr], dim=-1)
    return emb.cos().to(dtype).contiguous(), emb.sin().to(dtype).contiguous()


def rope_(x, cos, sin, pos0=0):
    """In-place RoPE of a contiguous [B, S, heads, D] tensor (qv_rope)."""
    B, S, nh, D = x.shape
    rc = N.lib().qv_rope(B, S, nh, D, kv_dtype_code(x.dtype), N.ptr(x), N.ptr(cos), N.ptr(sin), pos0,
                         torch.cuda.current_stream(x.device).cuda_stream)
    N.check(rc, "qv_rope")
    return x


def prefill_attention(q, k, v, colsum=True, check=True):
    """Causal prefill attention + per-key column sums (qv_prefill_attention).

    q [B, S, Hq, D], k/v [B, S, H, D] contiguous -> (out [B, S, Hq, D], colsum [B, H, S] fp32).
    With check, the device error word is read back (a stream synchronisation)
    and a pipelined kernel that gave up waiting raises QevictError."""
    B, S, Hq, D = q.shape
    H = k.shape[2]
    dims = N.QvDims(B, H, Hq // H, D, 64, 0, 64, 0, 0, 1, 8, kv_dtype_code(q.dtype), 0)
    import ctypes
    wsb = int(N.lib().qv_prefill_workspace_bytes(ctypes.byref(dims), S))
    ws = torch.empty(wsb, dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q)
    cs = torch.empty(B, H, S, dtype=torch.float32, device=q.device) if colsum else None
    rc = N.lib().qv_prefill_attention(ctypes.byref(dims), N.ptr(q), N.ptr(k), N.ptr(v), S, N.ptr(out),
                                      N.ptr(cs), N.ptr(ws), wsb, torch.cuda.current_stream(q.device).cuda_stream)
    N.check(rc, "qv_prefill_attention")
    if check:
        err = ctypes.c_int32(0)
        N.check(N.lib().qv_prefill_read_error(N.ptr(ws), wsb, ctypes.byref(err),
                                              torch.cuda.current_stream(q.device).cuda_stream),
                "qv_prefill_read_error")
        if err.value:
            raise N.QevictError(f"qv_prefill_attention: device error word {err.value:#x} (a bounded wait gave up)")
    return out, cs


class StickyLlamaDecoder:
    """Random-init Llama decoder, batch B, with Sticky-KV attention in every layer."""

    def __init__(self, shape: LlamaShape, sticky: StickyShape, batch=1, max_pos=40960,
                 dtype=torch.bfloat16, device="cuda", seed=0, std=0.02, side_fold=False):
        self.s, self.k, self.B = shape, sticky, batch
        self.dtype, self.device = dtype, torch.device(device)
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        s = shape
        Hq, H, D = s.heads, s.kv_heads, s.head_dim

        def w(*shp):
            return (torch.randn(*shp, generator=g, device=self.device, dtype=torch.float32) * std).to(dtype)

        self.embed = w(s.vocab, s.hidden)
        self.layers = []
        for _ in range(s.layers):
            self.layers.append(dict(
                ln1=torch.ones(s.hidden, dtype=dtype, device=self.device),
                wqkv=w((Hq + 2 * H) * D, s.hidden),
                wo=w(s.hidden, Hq * D),
                ln2=torch.ones(s.hidden, dtype=dtype, device=self.device),
                wgu=w(2 * s.ffn, s.hidden),
                wd=w(s.hidden, s.ffn)))
        self.norm = torch.ones(s.hidden, dtype=dtype, device=self.device)
        self.lm_head = w(s.vocab, s.hidden)
        self.cos, self.sin = rope_tables(max_pos, D, s.rope_theta, dtype, self.device)
        self.max_pos = max_pos
        max_windows = max((max_pos - sticky.sink) // sticky.omega, 100)
        self.states = []
        self.side_fold = side_fold
        ws = None
        for _ in range(s.layers):
            st = StickyLayerState(batch, H, Hq // H, D, sticky.omega, sticky.sink, sticky.local,
                                  sticky.k_windows, sticky.q_windows, max_windows, sticky.bits, dtype,
                                  self.device, workspace=None if side_fold else ws)
            ws = st.ws
            self.states.append(st)
        self.fold_stream = torch.cuda.Stream(device=self.device) if side_fold else None
        # static decode buffers (graph inputs/outputs)
        self.tok = torch.zeros(batch, dtype=torch.long, device=self.device)
        self.next_tok = torch.zeros(batch, dtype=torch.long, device=self.device)
        self.attn_out = torch.empty(batch, Hq, D, dtype=dtype, device=self.device)
        # decode-step buffers (graph inputs/outputs)
        self.x = torch.empty(batch, s.hidden, dtype=dtype, device=self.device)
        self.h = torch.empty_like(self.x)
        self.proj = torch.empty_like(self.x)
        self.qkv = torch.empty(batch, (Hq + 2 * H) * D, dtype=dtype, device=self.device)
        self.gu = torch.empty(batch, 2 * s.ffn, dtype=dtype, device=self.device)
        self.act = torch.empty(batch, s.ffn, dtype=dtype, device=self.device)
        self.logits = torch.empty(batch, s.vocab, dtype=dtype, device=self.device)
        self.argmax_ws = torch.zeros(int(N.lib().qv_argmax_workspace_bytes(batch)), dtype=torch.uint8,
                                     device=self.device)
        self.graphs = {}

    # ---------------------------------------------------------------- prefill
    @torch.no_grad()
    def prefill(self, ids):
        """ids [B, S] -> first generated token [B]; builds every layer's Sticky-KV state."""
        s = self.s
        B, S = ids.shape
        Hq, H, D = s.heads, s.kv_heads, s.head_dim
        x = self.embed[ids]
        for li, L in enumerate(self.layers):
            h = F.rms_norm(x, (s.hidden,), L["ln1"], s.rms_eps)
            qkv = h @ L["wqkv"].t()
            q = qkv[..., :Hq * D].reshape(B, S, Hq, D).contiguous()
            k = qkv[..., Hq * D:(Hq + H) * D].reshape(B, S, H, D).contiguous()
            v = qkv[..., (Hq + H) * D:].reshape(B, S, H, D).contiguous()
            del qkv, h
            rope_(q, self.cos, self.sin)
            rope_(k, self.cos, self.sin)
            o, cs = prefill_attention(q, k, v)
            del q
            self.states[li].prefill(k.transpose(1, 2).contiguous(), v.transpose(1, 2).contiguous(), cs)
            del k, v, cs
            x = x + o.reshape(B, S, Hq * D) @ L["wo"].t()
            del o
            x = self._mlp(x, L)
        h = F.rms_norm(x[:, -1], (s.hidden,), self.norm, s.rms_eps)
        nxt = torch.argmax(h @ self.lm_head.t(), dim=-1)
        self.tok.copy_(nxt)
        return nxt

    def _mlp(self, x, L, chunk=8192):
        s = self.s
        if x.dim() == 3 and x.shape[1] > chunk:
            return torch.cat([self._mlp(x[:, i:i + chunk], L) for i in range(0, x.shape[1], chunk)], dim=1)
        h = F.rms_norm(x, (s.hidden,), L["ln2"], s.rms_eps)
        gu = h @ L["wgu"].t()
        g, u = gu.chunk(2, dim=-1)
        return x + (F.silu(g) * u) @ L["wd"].t()

    # ----------------------------------------------------------------- decode
    def _add_norm(self, delta, weight):
        """x += delta (if given); h = RMSNorm(x) * weight (qv_add_rmsnorm)."""
        rc = N.lib().qv_add_rmsnorm(self.B, self.s.hidden, N.ptr(self.x), N.ptr(delta), N.ptr(weight),
                                    self.s.rms_eps, N.ptr(self.h), torch.cuda.current_stream(self.device).cuda_stream)
        N.check(rc, "qv_add_rmsnorm")

    def _gemv(self, w, x, y):
        """y = x @ w.T for the decode rows (qv_gemv: weight-streaming GEMV)."""
        rc = N.lib().qv_gemv(self.B, w.shape[0], w.shape[1], N.ptr(w), N.ptr(x), N.ptr(y),
                             torch.cuda.current_stream(self.device).cuda_stream)
        N.check(rc, "qv_gemv")

    def _layer_step(self, li, cycle=False):
        """One decoder layer on self.x; expects self.h = RMSNorm(x) * ln1 and leaves
        self.h = RMSNorm(x_out) * (the next layer's ln1, or the final norm)."""
        s, L, st = self.s, self.layers[li], self.states[li]
        B = self.B
        Hq, H, D = s.heads, s.kv_heads, s.head_dim
        self._gemv(L["wqkv"], self.h, self.qkv)
        q = self.qkv[:, :Hq * D].view(B, Hq, D)
        k = self.qkv[:, Hq * D:(Hq + H) * D].view(B, H, D)
        v = self.qkv[:, (Hq + H) * D:].view(B, H, D)
        qr = st.append(q, k, v, self.cos, self.sin)
        if cycle or not self.side_fold:
            st.attend(qr, self.attn_out)
        else:
            # the ledger fold goes to the side stream, beside the projections below
            st.attend(qr, self.attn_out, fold=False)
            self.fold_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.fold_stream):
                st.fold()
        self._gemv(L["wo"], self.attn_out, self.proj)
        self._add_norm(self.proj, L["ln2"])
        self._gemv(L["wgu"], self.h, self.gu)
        rc = N.lib().qv_silu_mul(B, s.ffn, N.ptr(self.gu), N.ptr(self.act),
                                 torch.cuda.current_stream(self.device).cuda_stream)
        N.check(rc, "qv_silu_mul")
        self._gemv(L["wd"], self.act, self.proj)
        nxt = self.layers[li + 1]["ln1"] if li + 1 < s.layers else self.norm
        self._add_norm(self.proj, nxt)

    def _step_body(self, cycle):
        torch.index_select(self.embed, 0, self.tok, out=self.x)
        self._add_norm(None, self.layers[0]["ln1"])
        for li in range(self.s.layers):
            self._layer_step(li, cycle)
            if cycle:
                self.states[li].evict_cycle()
        self._gemv(self.lm_head, self.h, self.logits)
        rc = N.lib().qv_argmax(self.B, self.s.vocab, N.ptr(self.logits), N.ptr(self.next_tok), N.ptr(self.argmax_ws),
                               self.argmax_ws.numel(), torch.cuda.current_stream(self.device).cuda_stream)
        N.check(rc, "qv_argmax")
        self.tok.copy_(self.next_tok)
        if self.side_fold and not cycle:
            # join the side stream's ledger folds
            torch.cuda.current_stream(self.device).wait_stream(self.fold_stream)

    def cycle_next(self):
        """Whether the next decode token completes an omega-window."""
        st = self.states[0]
        return (st.n_tokens + 1 - st.prompt_len) % st.omega == 0

    @torch.no_grad()
    def step_eager(self):
        self._step_body(self.cycle_next())
        return self.next_tok

    def close(self):
        """Release the captured graphs."""
        self.graphs.clear()

    @torch.no_grad()
    def capture(self):
        """Capture the plain and the cycle step into CUDA graphs (host counters restored)."""
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
        for st in self.states:
            st.n_tokens += 1
            if cycle:
                st.last_compaction = st.n_tokens
        return cycle

    def attention_bytes_per_layer(self, t_mean):
        """Algorithmic HBM bytes of one fused decode-attention launch (per layer).

        B*H*[S_m*2*D*e + S_q*(2*D*qb/D + 2*e) + Wq*2*D*e] with S_m = sink + k*omega + local + t."""
        k, s = self.k, self.s
        e = torch.finfo(self.dtype).bits // 8
        qb = s.head_dim if k.bits == 8 else s.head_dim // 2
        s_m = k.sink + k.k_windows * k.omega + k.local + t_mean
        s_q = k.q_windows * k.omega
        per = s_m * 2 * s.head_dim * e + s_q * (2 * qb + 2 * e) + k.q_windows * 2 * s.head_dim * e
        return self.B * s.kv_heads * per
