"""Device-resident Sticky-KV state of one attention layer, for B sequences.

Owns the HBM buffers of the slot layout described in include/qevict_b200.h and
drives the C ABI.  Everything on the decode path is stream-ordered and free of
host synchronisation: the host only mirrors the token counter (all sequences of
a batch advance in lockstep), which tells it when an eviction cycle is due.

The ``view_*`` helpers (which do synchronise) present the state in the
reference's logical order -- sticky windows by ascending id, Q-cache windows in
top-k order, the physical cache as [sinks | sticky | local | new tokens] -- so
that it can be compared with the reference (``STICKYKVCache_LayerWise`` in
src/models/kv_cache/cache.py) field by field.
"""

import ctypes

import torch

from . import _native as N

_DT = {torch.float32: N.QV_F32, torch.bfloat16: N.QV_BF16, torch.float16: N.QV_F16}


def kv_dtype_code(dtype):
    try:
        return _DT[dtype]
    except KeyError:
        raise N.QevictError(f"unsupported KV dtype {dtype}") from None


class Workspace:
    """Scratch for the split-K decode kernel and the eviction cycle.

    One workspace can serve every layer of a model that runs on one stream.
    It must start zero-filled (the decode kernel's tickets self-reset after
    each launch) and must not be used by two launches at the same time.
    """

    def __init__(self, dims, device):
        lib = N.lib()
        d = ctypes.byref(dims)
        self.decode_bytes = int(lib.qv_decode_workspace_bytes(d))
        self.cycle_bytes = int(lib.qv_cycle_workspace_bytes(d))
        if self.decode_bytes == 0 or self.cycle_bytes == 0:
            raise N.QevictError("invalid layer dimensions for the native library")
        self.decode = torch.zeros(self.decode_bytes, dtype=torch.uint8, device=device)
        self.cycle = torch.zeros(self.cycle_bytes, dtype=torch.uint8, device=device)

    def fits(self, dims):
        lib = N.lib()
        d = ctypes.byref(dims)
        return (int(lib.qv_decode_workspace_bytes(d)) <= self.decode_bytes
                and int(lib.qv_cycle_workspace_bytes(d)) <= self.cycle_bytes)


class StickyLayerState:
    def __init__(self, batch, kv_heads, group, head_dim, omega, sink, local, k_windows, q_windows,
                 max_windows, bits=8, dtype=torch.bfloat16, device="cuda", workspace=None,
                 reference_rounding=False):
        if local % omega or local < omega:
            raise N.QevictError("the local zone must be a positive whole number of windows")
        self.B, self.H, self.G, self.D = batch, kv_heads, group, head_dim
        self.omega, self.sink, self.local = omega, sink, local
        self.kw, self.qw, self.maxW, self.bits = k_windows, q_windows, max_windows, bits
        self.dtype = dtype
        self.device = torch.device(device)
        self.dims = N.QvDims(batch, kv_heads, group, head_dim, omega, sink, local, k_windows,
                             q_windows, max_windows, bits, kv_dtype_code(dtype),
                             N.QV_FLAG_REFERENCE_ROUNDING if reference_rounding else 0)
        lib = N.lib()
        self.R = int(lib.qv_ring_windows(ctypes.byref(self.dims)))
        self.S_cap = int(lib.qv_main_capacity(ctypes.byref(self.dims)))
        # 1: tensor-core decode (exact fp32 dequantisation of the Q-cache);
        # 0: CUDA-core decode with the reference's dequantisation rounding
        self.decode_path = int(lib.qv_decode_path(ctypes.byref(self.dims)))
        if self.R < 0 or self.S_cap < 0:
            raise N.QevictError("invalid layer dimensions for the native library")
        B, H, D, om, dev = batch, kv_heads, head_dim, omega, self.device
        qb = head_dim if bits == 8 else head_dim // 2
        z = lambda *s, dt=dtype: torch.zeros(*s, dtype=dt, device=dev)  # noqa: E731
        self.k = z(B, H, self.S_cap, D)
        self.v = z(B, H, self.S_cap, D)
        self.kq = z(B, H, q_windows, om, qb, dt=torch.uint8)
        self.vq = z(B, H, q_windows, om, qb, dt=torch.uint8)
        self.ks = z(B, H, q_windows, D)
        self.kz = z(B, H, q_windows, D)
        self.vs = z(B, H, q_windows, om)
        self.vz = z(B, H, q_windows, om)
        self.sticky_wid = torch.full((B, H, k_windows), -1, dtype=torch.int32, device=dev)
        self.sticky_score = z(B, H, k_windows, dt=torch.float32)
        self.sticky_order = z(B, H, k_windows, dt=torch.int32)
        self.q_wid = torch.full((B, H, q_windows), -1, dtype=torch.int32, device=dev)
        self.q_score = z(B, H, q_windows, dt=torch.float32)
        self.q_order = z(B, H, q_windows, dt=torch.int32)
        self.votes = z(B, H, self.S_cap, dt=torch.float32)
        self.local_hist = z(B, H, max_windows, dt=torch.float32)
        self.arch_valid = z(B, H, max_windows, dt=torch.uint8)
        self.arch_ks = z(B, H, max_windows, D)
        self.arch_kz = z(B, H, max_windows, D)
        self.arch_vs = z(B, H, max_windows, om)
        self.arch_vz = z(B, H, max_windows, om)
        self.seq = z(B, 4, dt=torch.int32)
        self.step_ctr = z(4, dt=torch.int32)
        self.err = z(1, dt=torch.int32)
        self.layer = N.QvLayer(*[N.ptr(t).value for t in (
            self.k, self.v, self.kq, self.vq, self.ks, self.kz, self.vs, self.vz, self.sticky_wid,
            self.sticky_score, self.sticky_order, self.q_wid, self.q_score, self.q_order,
            self.votes, self.local_hist, self.arch_valid, self.arch_ks, self.arch_kz, self.arch_vs,
            self.arch_vz, self.seq, self.step_ctr, self.err)])
        if workspace is None:
            workspace = Workspace(self.dims, dev)
        elif not workspace.fits(self.dims):
            raise N.QevictError("workspace too small for this layer")
        self.ws = workspace
        self.n_tokens = 0      # host mirror of step_ctr[0]
        self.prompt_len = 0
        self.last_compaction = 0  # token count at the last prefill / eviction cycle
        self.q_rot = z(B, H * group, D)

    # -- helpers ---------------------------------------------------------------
    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _call(self, name, *args):
        rc = getattr(N.lib(), name)(*args)
        N.check(rc, name)

    def cycle_due(self):
        """True when the token just processed completed a window (eviction_manager.py:375)."""
        return self.n_tokens > self.prompt_len and (self.n_tokens - self.prompt_len) % self.omega == 0

    # -- prefill -----------------------------------------------------------------
    def prefill(self, k_prompt, v_prompt, colsum):
        """k/v_prompt [B, H, S, D] (rotated, KV dtype); colsum [B, H, S] fp32 or KV dtype."""
        S = k_prompt.shape[2]
        if S < self.sink + self.local or (S - self.sink) % self.omega:
            raise N.QevictError(
                f"prompt length {S} unsupported: needs sink + local <= S and (S - sink) % omega == 0")
        k_prompt = k_prompt.contiguous()
        v_prompt = v_prompt.contiguous()
        colsum = colsum.contiguous()
        sd = N.QV_F32 if colsum.dtype == torch.float32 else kv_dtype_code(colsum.dtype)
        self._call("qv_prefill_build", ctypes.byref(self.dims), ctypes.byref(self.layer),
                   N.ptr(k_prompt), N.ptr(v_prompt), S, N.ptr(colsum), sd, self._stream())
        self.n_tokens = S
        self.prompt_len = S
        self.last_compaction = S

    # -- decode ------------------------------------------------------------------
    def append(self, q, k_new, v_new, cos=None, sin=None):
        """RoPE (when cos/sin tables are given) + in-place append; returns the rotated q."""
        self._call("qv_rope_append", ctypes.byref(self.dims), ctypes.byref(self.layer),
                   N.ptr(q.contiguous()), N.ptr(k_new.contiguous()), N.ptr(v_new.contiguous()),
                   N.ptr(cos), N.ptr(sin), N.ptr(self.q_rot), self._stream())
        return self.q_rot

    def attend(self, q_rot, out, fold=True):
        """Fused attention of the token appended last; fold=False leaves the
        vote-ledger fold pending for fold() (qv_decode_attention_nofold)."""
        name = "qv_decode_attention" if fold else "qv_decode_attention_nofold"
        self._call(name, ctypes.byref(self.dims), ctypes.byref(self.layer),
                   N.ptr(q_rot), N.ptr(out), N.ptr(self.ws.decode), self.ws.decode_bytes, self._stream())
        self.n_tokens += 1

    def fold(self):
        """The ledger fold left pending by attend(..., fold=False) (qv_decode_fold), on
        the current stream; it must run before the next append / attend / cycle."""
        self._call("qv_decode_fold", ctypes.byref(self.dims), ctypes.byref(self.layer),
                   N.ptr(self.ws.decode), self.ws.decode_bytes, self._stream())

    def evict_cycle(self):
        self._call("qv_evict_cycle", ctypes.byref(self.dims), ctypes.byref(self.layer),
                   N.ptr(self.ws.cycle), self.ws.cycle_bytes, self._stream())
        self.last_compaction = self.n_tokens

    def step(self, q, k_new, v_new, cos=None, sin=None, out=None):
        """One decode token for all B sequences: append, attend + ledger fold, cycle when due."""
        if self.n_tokens == 0:
            raise N.QevictError("decode before prefill")
        if out is None:
            out = torch.empty(self.B, self.H * self.G, self.D, dtype=self.dtype, device=self.device)
        qr = self.append(q, k_new, v_new, cos, sin)
        self.attend(qr, out)
        if self.cycle_due():
            self.evict_cycle()
        return out

    # -- diagnostics ---------------------------------------------------------------
    def read_error(self):
        v = ctypes.c_int32(0)
        self._call("qv_read_error", ctypes.byref(self.layer), ctypes.byref(v), self._stream())
        return v.value

    # -- logical views (synchronising; for tests and inspection) -------------------
    def counts(self):
        s = self.seq.cpu()
        return s[:, 0].tolist(), s[:, 1].tolist()

    def view_sticky(self, b):
        """(ids [H, k], scores [H, k]) in ascending-id order, like window_scores[:, :k, 1/0]."""
        ck = self.counts()[0][b]
        order = self.sticky_order[b, :, :ck].long()
        ids = torch.gather(self.sticky_wid[b], 1, order)
        sc = torch.gather(self.sticky_score[b], 1, order)
        return ids.cpu(), sc.cpu()

    def view_q(self, b):
        """Q-cache in top-k order: dict of ids, scores, kq, ks, kz, vq, vs, vz (reference shapes)."""
        qc = self.counts()[1][b]
        if qc == 0:
            return None
        o = self.q_order[b, :, :qc].long()
        hh = torch.arange(self.H, device=self.device)[:, None]
        return dict(ids=self.q_wid[b][hh, o].float().cpu(), scores=self.q_score[b][hh, o].cpu(),
                    kq=self.kq[b][hh, o].cpu(), vq=self.vq[b][hh, o].cpu(),
                    ks=self.ks[b][hh, o].unsqueeze(2).float().cpu(),
                    kz=self.kz[b][hh, o].unsqueeze(2).float().cpu(),
                    vs=self.vs[b][hh, o].unsqueeze(-1).float().cpu(),
                    vz=self.vz[b][hh, o].unsqueeze(-1).float().cpu())

    def reference_positions(self, b):
        """Slot-layout positions [H, S_ref] of the reference's physical order:
        sinks, sticky windows by ascending id, then every token appended since
        the last compaction's local zone, oldest first (cache.py:505-573)."""
        ck = self.counts()[0][b]
        om, sink, dev = self.omega, self.sink, self.device
        ar = torch.arange(om, device=dev)
        order = self.sticky_order[b, :, :ck].long()
        sticky = (sink + order[:, :, None] * om + ar).reshape(self.H, -1)
        p = torch.arange(self.last_compaction - self.local, self.n_tokens, device=dev) - sink
        ring = sink + self.kw * om + ((p // om) % self.R) * om + p % om
        sinks = torch.arange(sink, device=dev)
        return torch.cat([sinks[None].expand(self.H, -1), sticky, ring[None].expand(self.H, -1)], dim=1)

    def reference_token_ids(self, b):
        """Token index [H, S_ref] (int64, on the device) held at each position of
        the reference's physical order, the positions of reference_positions(b):
        sinks, the tokens of the sticky windows by ascending id, the local zone."""
        ck = self.counts()[0][b]
        om, sink, dev = self.omega, self.sink, self.device
        order = self.sticky_order[b, :, :ck].long()
        wid = torch.gather(self.sticky_wid[b], 1, order).long()
        sticky = (sink + wid[:, :, None] * om + torch.arange(om, device=dev)).reshape(self.H, -1)
        ring = torch.arange(self.last_compaction - self.local, self.n_tokens, device=dev)
        sinks = torch.arange(sink, device=dev)
        return torch.cat([sinks[None].expand(self.H, -1), sticky, ring[None].expand(self.H, -1)], dim=1)

    def view_kv(self, b):
        """Physical cache in the reference's order: (K [H, S_ref, D], V) as float32 on CPU."""
        pos = self.reference_positions(b)
        idx = pos[:, :, None].expand(-1, -1, self.D)
        return (torch.gather(self.k[b], 1, idx).float().cpu(), torch.gather(self.v[b], 1, idx).float().cpu())

    def view_logits(self, b):
        """Rounded logits of the last decode step, [H, G, S_ref + Q tokens] in the
        reference's order (main zone as reference_positions, then Q windows in
        top-k order), as float32 on CPU."""
        off = int(N.lib().qv_decode_logits_offset(ctypes.byref(self.dims)))
        S_tot = self.S_cap + self.qw * self.omega
        n = self.B * self.H * S_tot * self.G
        lg = self.ws.decode[off:off + n * self.k.element_size()].view(self.dtype)
        lg = lg.view(self.B, self.H, S_tot, self.G)[b]
        pos = self.reference_positions(b)                          # [H, S_ref]
        main = torch.gather(lg, 1, pos[:, :, None].expand(-1, -1, self.G))
        parts = [main]
        qc = self.counts()[1][b]
        if qc:
            o = self.q_order[b, :, :qc].long()
            qpos = self.S_cap + (o[:, :, None] * self.omega + torch.arange(self.omega, device=self.device)).reshape(self.H, -1)
            parts.append(torch.gather(lg, 1, qpos[:, :, None].expand(-1, -1, self.G)))
        return torch.cat(parts, dim=1).permute(0, 2, 1).float().cpu()

    def view_votes(self, b):
        pos = self.reference_positions(b)
        return torch.gather(self.votes[b], 1, pos).cpu()
