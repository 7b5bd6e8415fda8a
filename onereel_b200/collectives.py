"""The C ABI's NCCL collectives (orl_comm_*, csrc/comm.cpp) from Python: one communicator per rank over the ranks of
the torch.distributed group, operations enqueued on a dedicated high-priority CUDA stream that is ordered after the
caller's stream, completion either as a device-side dependency of the caller's stream or as the timeout-aware host
wait (orl_comm_wait: an NCCL error or the time limit aborts the communicator instead of waiting forever).

`comm.HaloExchange(..., collectives=NcclComm(...))` runs the K/V exchange through it instead of torch.distributed —
the same operation lists in the same order (the reference's src/onereel/parallel/comm.py:126-201 exchange).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from onereel_b200 import _lib as L
from onereel_b200 import dist as D


class NcclComm:
    def __init__(self, device=None):
        if not L.lib().orl_comm_available():
            raise RuntimeError('NCCL (libnccl.so.2) could not be loaded')
        self.device = torch.device('cuda', torch.cuda.current_device()) if device is None else torch.device(device)
        self.rank, self.world = D.rank(), D.world()
        uid = (ctypes.c_uint8 * 128)()
        if self.rank == 0:
            L.check(L.lib().orl_comm_unique_id(uid), 'orl_comm_unique_id')
        box = [bytes(uid)]
        if self.world > 1:
            dist.broadcast_object_list(box, src=0, group=D.group())
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(box[0])
        self.handle = ctypes.c_void_p()
        L.check(L.lib().orl_comm_init(ctypes.byref(self.handle), uid, self.world, self.rank, self.device.index),
                'orl_comm_init')
        self.stream = torch.cuda.Stream(self.device, priority=-1)
        self.keep = []

    def _begin(self):
        """order the comm stream after the caller's current stream (the inputs are written there)"""
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        return self.stream.cuda_stream

    def exchange(self, sends, recvs):
        """sends / recvs: [(peer, contiguous tensor)] in per-peer order (both sides list a peer's operations alike)"""
        s = self._begin()
        mk = lambda ops: (L.P2P * max(len(ops), 1))(*[L.P2P(p, 0, t.data_ptr(), t.numel() * t.element_size())
                                                      for p, t in ops])
        self.keep += [t for _, t in sends] + [t for _, t in recvs]
        L.check(L.lib().orl_comm_exchange(self.handle, mk(sends), len(sends), mk(recvs), len(recvs), s),
                'orl_comm_exchange')

    def broadcast(self, t: torch.Tensor, root: int):
        s = self._begin()
        self.keep.append(t)
        L.check(L.lib().orl_comm_broadcast(self.handle, t.data_ptr(), t.numel() * t.element_size(), root, s),
                'orl_comm_broadcast')

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor):
        """equal split over the ranks along dim 0 (all_to_all_single)"""
        s = self._begin()
        self.keep += [out, inp]
        L.check(L.lib().orl_comm_all_to_all(self.handle, inp.data_ptr(), out.data_ptr(),
                                            inp.numel() * inp.element_size() // self.world, s), 'orl_comm_all_to_all')

    def all_reduce(self, t: torch.Tensor):
        assert t.dtype == torch.float32 and t.is_contiguous()
        s = self._begin()
        self.keep.append(t)
        L.check(L.lib().orl_comm_all_reduce_f32(self.handle, t.data_ptr(), t.numel(), s), 'orl_comm_all_reduce_f32')

    def wait(self, timeout_s: float | None = None):
        """without a limit: the caller's stream waits for the comm stream on the device (no host block); with one:
        the host waits at most timeout_s (orl_comm_wait), then the caller's stream is ordered after the comm stream"""
        if timeout_s is not None:
            L.check(L.lib().orl_comm_wait(self.handle, self.stream.cuda_stream, int(timeout_s * 1e9)), 'orl_comm_wait')
        torch.cuda.current_stream(self.device).wait_stream(self.stream)
        for t in self.keep:
            t.record_stream(self.stream)
        self.keep = []

    def close(self):
        if self.handle:
            L.lib().orl_comm_destroy(self.handle)
            self.handle = ctypes.c_void_p()
