"""Host side of the gather/pack kernel (orl_pack): run tables of row-range copies.

A run table is built once per layout (video/text row ranges relative to slot base pointers, e.g. "rows 3180..4770 of
slot 0 (this layer's K) to row 0 of slot 2 (the packed K)"), prepared (16-byte vector prefix sums) and uploaded once;
every call then passes only the slots' current base pointers, so per-layer packing costs one kernel launch and no
host-to-device traffic. For one-off packs (the generic `attention.packed` drop-in) the sources are absolute device
addresses against a null slot base.
"""
from __future__ import annotations

import numpy as np
import torch

from onereel_b200 import _lib as L


def _err_word(device):
    # the error word the attention launches on this device report through (attention.check reads it)
    from onereel_b200.attention import _err_word as word
    return word(device)


class RunTable:
    """a prepared run table on one device: runs_dev (uint8 view of orl_copy_run [n]), total 16-byte vectors"""
    launches = 0          # pack launches issued by this process (benchmark launch accounting)

    def __init__(self, src_slot, dst_slot, src_off, dst_off, nbytes, device):
        n = len(nbytes)
        arr = np.zeros(n, dtype=L.RUN_DTYPE)
        arr['src_slot'], arr['dst_slot'] = src_slot, dst_slot
        arr['src_off'], arr['dst_off'] = src_off, dst_off
        nb = np.ascontiguousarray(nbytes, dtype=np.int64)
        total = L.check(L.lib().orl_pack_prepare(arr.ctypes.data, L.i64p(nb), n), 'orl_pack_prepare')
        self.n_runs, self.total_vecs, self.nbytes = n, int(total), int(nb.sum())
        # the table as built (host lists), for accounting
        self.src_slot = [int(x) for x in src_slot]
        self.src_off, self.dst_off = [int(x) for x in src_off], [int(x) for x in dst_off]
        self.nbytes_list = nb.tolist()
        self.dev = torch.from_numpy(arr.view(np.uint8)).to(device) if n else None
        self.device = torch.device(device)

    def run(self, src_bases, dst_bases, n_planes=1, seg_len_dev=None, cu_out=None, stream=None):
        """execute on `stream` (default: torch's current stream). src_bases / dst_bases: per plane, per slot device
        addresses (ints), flattened plane-major; cu_out (int32 [n_seg + 1] tensor) receives cu_seqlens of
        seg_len_dev (int32 [n_seg] tensor)."""
        n_slots = len(src_bases) // n_planes
        assert len(src_bases) == len(dst_bases) == n_slots * n_planes
        SrcArr = L.c_vp * len(src_bases)
        s = stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream
        n_seg = 0 if seg_len_dev is None else seg_len_dev.numel()
        RunTable.launches += 1
        L.check(L.lib().orl_pack(self.dev.data_ptr() if self.dev is not None else None, self.n_runs, self.total_vecs,
                                 n_planes, n_slots, SrcArr(*src_bases), SrcArr(*dst_bases),
                                 None if seg_len_dev is None else seg_len_dev.data_ptr(), n_seg,
                                 None if cu_out is None else cu_out.data_ptr(), _err_word(self.device).data_ptr(),
                                 s), 'orl_pack')


def row_bytes(x: torch.Tensor) -> int:
    return x.stride(0) * x.element_size()


def pack_rows(parts, dst: torch.Tensor):
    """one-off pack: parts = list of 2-D-or-more row tensors (rows contiguous), copied back to back into dst rows.
    Every part is viewed as raw bytes at its absolute address (slot 0 = null base)."""
    rb = row_bytes(dst)
    src_off, dst_off, nbytes = [], [], []
    row = 0
    for p in parts:
        n = p.shape[0]
        if n:
            assert p.is_contiguous() and row_bytes(p) == rb, 'pack_rows: parts must be contiguous with dst row size'
            src_off.append(p.data_ptr())
            dst_off.append(row * rb)
            nbytes.append(n * rb)
        row += n
    assert row == dst.shape[0]
    if not nbytes:
        return dst
    t = RunTable(np.zeros(len(nbytes), np.int32), np.zeros(len(nbytes), np.int32), src_off, dst_off, nbytes,
                 dst.device)
    t.run([0], [dst.data_ptr()])
    return dst
