"""Host side of the one-shot NVLink sum (qv_peer_sum_*): the all-reduce of the
KV-head-parallel decode's row-parallel partials.

Every rank of the group creates its buffer, the CUDA IPC handles are
exchanged with one all_gather_object over the group, and every rank maps
every other rank's buffer.  sum_(t) then adds t over the ranks in place
(rank order, fp32, one bf16 rounding: the same bits on every rank) with one
kernel on the current stream, capturable in a CUDA graph.  Tensors that do
not fit (not bf16, larger than max_bytes, size not a multiple of 8) are left
to the caller's collective.
"""

import ctypes

import torch

from . import _native as N


class PeerSum:
    def __init__(self, rank, world, group=None, max_bytes=64 * 1024):
        import torch.distributed as dist
        self.world, self.max_bytes = world, max_bytes
        self.handle = ctypes.c_void_p()
        h = ctypes.create_string_buffer(N.QV_PEER_HANDLE_BYTES)
        N.check(N.lib().qv_peer_sum_create(rank, world, max_bytes, ctypes.byref(self.handle), h),
                "qv_peer_sum_create")
        mine = bytes(h.raw)
        handles = [None] * world
        dist.all_gather_object(handles, mine, group=group)
        if len(set(handles)) != world:
            raise N.QevictError("qv_peer_sum: the ranks' IPC handles are not distinct")
        N.check(N.lib().qv_peer_sum_open(self.handle, b"".join(handles)), "qv_peer_sum_open")

    def fits(self, t):
        return (self.handle is not None and t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous()
                and t.numel() % 8 == 0 and t.numel() * 2 <= self.max_bytes and t.data_ptr() % 16 == 0)

    def sum_(self, t):
        """t (bf16, on this rank's GPU) <- the sum of every rank's t."""
        N.check(N.lib().qv_peer_sum_bf16(self.handle, N.ptr(t), N.ptr(t), t.numel(),
                                         torch.cuda.current_stream(t.device).cuda_stream), "qv_peer_sum_bf16")
        return t

    def max_(self, t):
        """t (int64, on this rank's GPU, at most max_bytes / 8 values) <- the
        elementwise maximum of every rank's t."""
        N.check(N.lib().qv_peer_max_i64(self.handle, N.ptr(t), N.ptr(t), t.numel(),
                                        torch.cuda.current_stream(t.device).cuda_stream), "qv_peer_max_i64")
        return t

    def read_error(self):
        err = ctypes.c_int32(0)
        N.check(N.lib().qv_peer_sum_read_error(self.handle, ctypes.byref(err),
                                               torch.cuda.current_stream().cuda_stream), "qv_peer_sum_read_error")
        return err.value

    def close(self):
        """Release the buffer and the mappings; every rank's last call must have
        completed first (synchronise and barrier before)."""
        if self.handle is not None and self.handle.value:
            N.check(N.lib().qv_peer_sum_destroy(self.handle), "qv_peer_sum_destroy")
        self.handle = None
