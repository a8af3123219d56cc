"""Sticky-KV attention with the KV heads split over devices (tensor parallel).

Each rank of a process group holds ``kv_heads / world`` KV heads of a layer
(their query-head groups, their sticky windows, Q-cache and vote ledger) in
its own ``StickyLayerState``.  Per decode token a rank appends its heads' new
K/V, runs the fused attention for its query heads, and the ranks exchange the
attention outputs with one all-gather (NCCL over NVLink) so that every rank
holds ``[B, Hq, D]`` for the output projection.  Every omega tokens the
eviction cycle runs per rank; its single coupling between heads -- the number
of Q-cache losers is the minimum over all heads (eviction_manager.py:335-345)
-- is one MIN all-reduce of a ``[B]`` int32 count between a counting pass and
the cycle proper (``qv_evict_cycle_count`` / ``qv_evict_cycle_ext``).  The
prefill split is per head with no exchange (every head sees the same number
of prompt windows).

All exchanges are stream-ordered device collectives, so a decode step stays
free of host synchronisation and can be captured in a CUDA graph.

``TorchDistExchange`` carries the two collectives over a torch.distributed
process group (NCCL on GPUs, gloo on CPU).  ``step_local`` runs all shards of a
layer one after another in one process on one device, with the same
collectives done as device ops (used to check the split against a single
unsharded state).
"""

import ctypes

import torch

from . import _native as N
from .layer_state import StickyLayerState


class TorchDistExchange:
    """Collectives over a torch.distributed process group."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._staging = {}

    def gather_heads(self, local, out):
        """local [B, hl, D] of this rank -> out [B, world*hl, D], heads in rank order.

        One all_gather_into_tensor into a staging buffer kept across calls
        ([world * B, hl, D]: no allocation per token, so the call can be
        captured in a CUDA graph), then one copy into out's head order (the
        copy is a no-op reshape when B == 1)."""
        B, hl, D = local.shape
        key = (B, hl, D, local.dtype, local.device)
        buf = self._staging.get(key)
        if buf is None:
            # the concatenated form [world * B, hl, D] (every backend takes it)
            buf = torch.empty(self.world * B, hl, D, dtype=local.dtype, device=local.device)
            self._staging[key] = buf
        self.dist.all_gather_into_tensor(buf, local.contiguous(), group=self.group)
        if B == 1:
            out.view(self.world, hl, D).copy_(buf)
        else:
            out.view(B, self.world, hl, D).copy_(buf.view(self.world, B, hl, D).permute(1, 0, 2, 3))

    def min_(self, t):
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MIN, group=self.group)


def gather_heads_local(locals_, out):
    """The all-gather of step_local: per-shard [B, hl, D] tensors -> out [B, world*hl, D]."""
    B, hl, D = locals_[0].shape
    out.view(B, len(locals_), hl, D).copy_(torch.stack(locals_, dim=1))


class KVHeadShardedLayer:
    """This rank's share of one Sticky-KV attention layer whose KV heads are split over ``world`` ranks.

    kv_heads/group/... describe the whole layer; the rank holds heads
    [rank * kv_heads/world, (rank + 1) * kv_heads/world) and their query heads.
    """

    def __init__(self, rank, world, batch, kv_heads, group, head_dim, omega, sink, local, k_windows, q_windows,
                 max_windows, bits=8, dtype=torch.bfloat16, device="cuda", workspace=None):
        if kv_heads % world:
            raise N.QevictError(f"{kv_heads} KV heads do not split over {world} ranks")
        self.rank, self.world = rank, world
        self.kv_heads, self.group, self.D = kv_heads, group, head_dim
        self.hl = kv_heads // world
        self.state = StickyLayerState(batch, self.hl, group, head_dim, omega, sink, local, k_windows, q_windows,
                                      max_windows, bits, dtype, device, workspace=workspace)
        self.counts = torch.zeros(batch, dtype=torch.int32, device=self.state.device)

    # head ranges of this rank
    def kv_slice(self):
        return slice(self.rank * self.hl, (self.rank + 1) * self.hl)

    def q_slice(self):
        return slice(self.rank * self.hl * self.group, (self.rank + 1) * self.hl * self.group)

    def prefill(self, k_prompt, v_prompt, colsum):
        """The rank's heads of the rotated prompt: k/v [B, hl, S, D], colsum [B, hl, S]."""
        self.state.prefill(k_prompt, v_prompt, colsum)

    def attend_local(self, q, k_new, v_new, cos=None, sin=None):
        """Append + fused attention for this rank's heads: q [B, hl*G, D], k/v [B, hl, D] -> [B, hl*G, D]."""
        st = self.state
        out = torch.empty(st.B, self.hl * self.group, self.D, dtype=st.dtype, device=st.device)
        qr = st.append(q, k_new, v_new, cos, sin)
        st.attend(qr, out)
        return out

    def count_losers(self):
        st = self.state
        rc = N.lib().qv_evict_cycle_count(ctypes.byref(st.dims), ctypes.byref(st.layer), N.ptr(st.ws.cycle),
                                          st.ws.cycle_bytes, N.ptr(self.counts), st._stream())
        N.check(rc, "qv_evict_cycle_count")
        return self.counts

    def cycle_with(self, counts):
        st = self.state
        rc = N.lib().qv_evict_cycle_ext(ctypes.byref(st.dims), ctypes.byref(st.layer), N.ptr(st.ws.cycle),
                                        st.ws.cycle_bytes, N.ptr(counts), st._stream())
        N.check(rc, "qv_evict_cycle_ext")
        st.last_compaction = st.n_tokens

    def step(self, q, k_new, v_new, out, exchange, cos=None, sin=None):
        """One decode token on this rank with a TorchDistExchange: q [B, Hq, D] and
        k/v [B, H, D] for the whole layer (this rank slices its heads); out [B, Hq, D]
        receives every rank's attention output."""
        local = self.attend_local(q[:, self.q_slice()].contiguous(), k_new[:, self.kv_slice()].contiguous(),
                                  v_new[:, self.kv_slice()].contiguous(), cos, sin)
        exchange.gather_heads(local, out)
        if self.state.cycle_due():
            c = self.count_losers()
            exchange.min_(c)
            self.cycle_with(c)
        return out


def step_local(shards, q, k_new, v_new, out, cos=None, sin=None):
    """One decode token for all shards of a layer in this process: the same
    collectives as the distributed path, done with device ops."""
    locals_ = [s.attend_local(q[:, s.q_slice()].contiguous(), k_new[:, s.kv_slice()].contiguous(),
                              v_new[:, s.kv_slice()].contiguous(), cos, sin) for s in shards]
    gather_heads_local(locals_, out)
    if shards[0].state.cycle_due():
        counts = [s.count_losers().clone() for s in shards]
        m = torch.stack(counts).min(dim=0).values.to(torch.int32).contiguous()
        for s in shards:
            s.cycle_with(m)
    return out
