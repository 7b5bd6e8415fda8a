"""K/V exchange over peer memory on NVLink / NVSwitch — the B200 replacement for the NCCL send/recv of the reference's
HaloExchange (src/onereel/parallel/comm.py:126-201).

Every rank keeps its own K and V rows of a layer in a symmetric buffer (torch's symmetric memory: one allocation per
rank, mapped into every peer's address space). A layer's exchange is then, on the compute stream:
  1. copy the rank's K / V rows into its symmetric buffer (skipped when the producer already wrote them there);
  2. orl_peer_barrier: a device-side barrier through signal pads in symmetric memory (bounded wait, error bit on
     timeout) — after it, every rank's rows of this layer have landed;
  3. one orl_pack launch pulls every interval this rank reads from its owner's buffer (TMA bulk loads from the peer's
     memory, no multicast) into the receive buffers, K and V as two planes of one run table.
The receive layout (`remote_index`, `remote_k`, `remote_v`) is HaloExchange's, so the compiled scene plans use either.
Buffers come in two generations used alternately: a rank rewrites generation g only after the next layer's barrier,
which every peer reaches after its pull from g in stream order, so one barrier per layer suffices. Symmetric memory
is allocated without NVLink multicast objects (plain peer mappings only).

Bit-exact with the NCCL path (the rows move unchanged). world == 1 needs no exchange.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

from onereel_b200 import _lib as L
from onereel_b200 import dist as D
from onereel_b200.pack import RunTable

# a peer that does not reach the barrier within this time ends the step with an error bit instead of a hang
BARRIER_TIMEOUT_NS = 2_000_000_000


class PeerSpace:
    """symmetric K/V buffers of `rows` rows x `row_elems` elements (two generations) and the signal pad, on every rank
    of the process group; the same shape must be requested on every rank (collective)"""

    def __init__(self, rows: int, row_elems: int, dtype: torch.dtype, device: torch.device, planes: int = 2):
        os.environ.setdefault('TORCH_SYMM_MEM_DISABLE_MULTICAST', '1')
        from torch.distributed import _symmetric_memory as symm
        g = D.group()
        if hasattr(symm, 'enable_symm_mem_for_group') and hasattr(g, 'group_name'):
            try:
                symm.enable_symm_mem_for_group(g.group_name)
            except Exception:        # already enabled, or enabled implicitly by this torch version
                pass
        self.n, self.r = D.world(), D.rank()
        self.rows, self.row_elems, self.dtype, self.device = rows, row_elems, dtype, torch.device(device)
        self.planes = planes
        self.row_bytes = row_elems * torch.tensor([], dtype=dtype).element_size()
        self.gens = []
        for _ in range(2):
            buf = symm.empty((planes, rows, row_elems), dtype=dtype, device=self.device)
            h = symm.rendezvous(buf, g)
            self.gens.append((buf, [int(p) for p in h.buffer_ptrs], h))
        pad = symm.empty(self.n, dtype=torch.int32, device=self.device)
        pad.zero_()
        ph = symm.rendezvous(pad, g)
        self.pad, self.pad_handle = pad, ph
        self.pad_ptrs = (ctypes.c_void_p * self.n)(*[int(p) for p in ph.buffer_ptrs])
        self.epoch, self.gen = 0, 0
        torch.cuda.synchronize(self.device)
        D.barrier()                  # every pad zeroed before any rank signals

    def next_gen(self):
        """the generation this layer writes (alternating)"""
        g = self.gen
        self.gen ^= 1
        return g

    def barrier(self, stream, err_dev):
        self.epoch += 1
        L.check(L.lib().orl_peer_barrier(self.pad_ptrs, self.n, self.r, self.epoch, BARRIER_TIMEOUT_NS,
                                         err_dev.data_ptr(), stream.cuda_stream), 'orl_peer_barrier')


_SPACES = {}


def initialised() -> bool:
    """whether a symmetric space exists (a failure after that is an error, not an unavailable feature)"""
    return bool(_SPACES)


def space_for(rows: int, row_elems: int, dtype, device, planes: int = 2, tag: str = 'kv') -> PeerSpace:
    """one PeerSpace per (use, planes, shape, dtype, device), created collectively on first use and kept (layers
    reuse it)"""
    key = (tag, planes, rows, row_elems, dtype, str(device))
    sp = _SPACES.get(key)
    if sp is None:
        sp = _SPACES[key] = PeerSpace(rows, row_elems, dtype, device, planes)
    return sp


def kv_inputs(own, H, Dh, dtype, device):
    """where a producer writes this rank's K / V rows of the next layer so the exchange need not copy them:
    (k [b - a, H, D], v [b - a, H, D]) views of the symmetric buffer of the generation the next PeerExchange of this
    shape uses (collective on first use, like the exchange). Rows written there must not change until that exchange
    has run; a PeerExchange given other tensors copies them in as usual."""
    r = D.rank()
    rows = own[r][1] - own[r][0]
    sp = space_for(max(b - a for a, b in own), H * Dh, dtype, device)
    buf = sp.gens[sp.gen][0]
    return buf[0, :rows].view(rows, H, Dh), buf[1, :rows].view(rows, H, Dh)


def _recv_layout(need_r, own, r):
    """rank r's receive layout: [(token lo, token hi, buffer row, owner)] sorted by lo (HaloExchange's order)"""
    from onereel_b200 import comm
    recv = [(lo, hi, p) for p in range(len(own)) if p != r for lo, hi in comm.clip(need_r, *own[p])]
    out, off = [], 0
    for lo, hi, p in sorted(recv):
        out.append((lo, hi, off, p))
        off += hi - lo
    return out, off


def _row_of(layout_r, lo):
    """buffer row of token lo in a receive layout"""
    for a, b, off, _ in layout_r:
        if a <= lo < b:
            return off + lo - a
    raise KeyError(lo)


def _stripes(lo, hi, readers):
    """[lo, hi) cut into len(readers) nearly equal consecutive stripes, one per reader"""
    k = len(readers)
    cuts = [lo + (hi - lo) * i // k for i in range(k + 1)]
    return [(q, cuts[i], cuts[i + 1]) for i, q in enumerate(readers) if cuts[i] < cuts[i + 1]]


class PeerExchange:
    """one layer's K/V exchange over peer memory, with HaloExchange's result interface (remote_index, remote_k,
    remote_v, wait). own: every rank's token range; k / v: this rank's rows [b - a, H, D] (contiguous).

    Rows that every other rank reads (frame-memory frames; `common` of comm.exchange_plan, from 3 ranks up) would
    make their owner's NVLink egress the bottleneck if every reader pulled them from it. They move in two stages
    instead: each reader pulls one stripe from the owner into its (symmetric) receive buffer, a second barrier, then
    each reader pulls the other stripes from the readers that fetched them — the owner sends every row once."""

    def __init__(self, layout, own, T, k, v, extra=()):
        from onereel_b200 import attention as A, comm
        n, r = D.world(), D.rank()
        self.a, self.b = own[r]
        self.remote_index, self.remote_k, self.remote_v = [], None, None
        self.bytes_in = 0
        if n == 1:
            return
        H, Dh = k.shape[1:]
        rows_max = max(b - a for a, b in own)
        sp = space_for(rows_max, H * Dh, k.dtype, k.device)
        rb = sp.row_bytes
        key = (tuple(map(tuple, own)), T, tuple(layout.lengths), layout.halo, layout.sides,
               tuple(sorted((j, tuple(f)) for j, f in (layout.extra or {}).items())), tuple(extra), rb)
        plan = _PLANS.get(key)
        if plan is None:
            plan = _PLANS[key] = _Plan(layout, own, T, extra, r, k.device, rb)
        self.remote_index = plan.remote_index
        rsp = space_for(max(plan.remote_rows, 1), H * Dh, k.dtype, k.device, tag='kv_remote') if plan.two_stage \
            else None
        stream = torch.cuda.current_stream(k.device)
        g = sp.next_gen()
        buf, ptrs, _ = sp.gens[g]
        if rsp is not None:
            rg = rsp.next_gen()
            rbuf, rptrs, _ = rsp.gens[rg]
            self.remote_k = rbuf[0, :plan.rows].view(plan.rows, H, Dh)
            self.remote_v = rbuf[1, :plan.rows].view(plan.rows, H, Dh)
        else:
            self.remote_k = k.new_empty((plan.rows, H, Dh))
            self.remote_v = v.new_empty((plan.rows, H, Dh))
        nr = self.b - self.a
        # a producer that wrote this layer's rows straight into the generation's buffer (kv_inputs) saves the copy
        if k.data_ptr() != buf[0].data_ptr():
            buf[0, :nr].copy_(k.reshape(nr, H * Dh))
        if v.data_ptr() != buf[1].data_ptr():
            buf[1, :nr].copy_(v.reshape(nr, H * Dh))
        err = A._err_word(k.device)
        sp.barrier(stream, err)
        kplane, dst = sp.rows * rb, [0] * n + [self.remote_k.data_ptr()] + [0] * n + [self.remote_v.data_ptr()]
        if plan.stage1 is not None:            # from the owners: every private interval and this rank's stripes
            plan.stage1.run([ptrs[p] for p in range(n)] + [0] + [ptrs[p] + kplane for p in range(n)] + [0], dst,
                            n_planes=2, stream=stream.cuda_stream)
        if rsp is not None:
            rsp.barrier(stream, err)           # every reader holds its stripes
            if plan.stage2 is not None:        # the other stripes, from the readers that fetched them
                rplane = rsp.rows * rb
                plan.stage2.run([rptrs[p] for p in range(n)] + [0] + [rptrs[p] + rplane for p in range(n)] + [0], dst,
                                n_planes=2, stream=stream.cuda_stream)
        self.bytes_in = 2 * plan.rows * rb

    def wait(self, timeout_s=None):
        """the pull ran on the compute stream: nothing to wait for"""


class _Plan:
    """the run tables of one exchange on rank r (cached per layout): stage 1 pulls from the owners, stage 2 the
    stripes of common rows from the other readers' receive buffers"""

    def __init__(self, layout, own, T, extra, r, device, rb):
        from onereel_b200 import comm
        n = len(own)
        need, common, _ = comm.exchange_plan(layout, own, T, extra)
        lay = [_recv_layout(need[q], own, q)[0] for q in range(n)]
        self.remote_index = [(lo, hi, off) for lo, hi, off, _ in lay[r]]
        self.rows = sum(hi - lo for lo, hi, _, _ in lay[r])
        self.remote_rows = max(sum(hi - lo for lo, hi, _, _ in lay[q]) for q in range(n))
        # common intervals by owner, cut into stripes over the readers
        stripes = {}                           # (owner, lo, hi) -> [(reader, s_lo, s_hi)]
        for p in range(n):
            readers = [q for q in range(n) if q != p]
            for lo, hi in common[p]:
                stripes[(p, lo, hi)] = _stripes(lo, hi, readers)
        self.two_stage = bool(stripes)
        s1, s2 = [], []                        # (src slot, src row, dst row, rows)

        def from_reader(q, a, b, dst_row):
            # token rows [a, b) out of reader q's receive buffer, split where q's layout is not contiguous
            for u, w, off_q, _ in lay[q]:
                x, y = max(a, u), min(b, w)
                if x < y:
                    s2.append((q, off_q + x - u, dst_row + x - a, y - x))

        for lo, hi, off, p in lay[r]:
            cur = lo
            mine = sorted((clo, chi, parts) for (cp, clo, chi), parts in stripes.items()
                          if cp == p and clo < hi and chi > lo)
            for clo, chi, parts in mine:
                clo, chi = max(clo, lo), min(chi, hi)
                if clo > cur:
                    s1.append((p, cur - own[p][0], off + cur - lo, clo - cur))
                for q, a, b in parts:
                    a, b = max(a, clo), min(b, chi)
                    if a >= b:
                        continue
                    if q == r:
                        s1.append((p, a - own[p][0], off + a - lo, b - a))
                    else:
                        from_reader(q, a, b, off + a - lo)
                cur = max(cur, chi)
            if cur < hi:
                s1.append((p, cur - own[p][0], off + cur - lo, hi - cur))
        self.stage1 = self._table(s1, n, device, rb)
        self.stage2 = self._table(s2, n, device, rb)

    @staticmethod
    def _table(runs, n, device, rb):
        runs = [x for x in runs if x[3] > 0]
        if not runs:
            return None
        return RunTable(np.array([x[0] for x in runs], np.int32), np.full(len(runs), n, np.int32),
                        [x[1] * rb for x in runs], [x[2] * rb for x in runs], [x[3] * rb for x in runs], device)


_PLANS = {}



# ------------------------------------------------------------------------------------------------ Ulysses
# The all-to-alls of the Ulysses path (the reference's a2a_heads / a2a_tokens, parallel/comm.py:276-295) as pulls
# over peer memory: q / k / v of every rank go into a three-plane symmetric buffer; after a barrier each rank pulls
# its heads of every peer's tokens straight into [all tokens, local heads, D]; the attention writes its output into
# a symmetric buffer, and after a second barrier each rank pulls its tokens of every peer's heads straight into
# [local tokens, all heads, D]. Generations alternate per call as for the K/V exchange.

def _elem(dtype) -> int:
    return torch.tensor([], dtype=dtype).element_size()


def _gather(src, dst, planes, n, rows, seg, src_row0, src_stride, dst_pstride, dst_stride, stream):
    S = ctypes.c_void_p * len(src)
    Dd = ctypes.c_void_p * len(dst)
    L.check(L.lib().orl_peer_gather(S(*src), Dd(*dst), planes, n, rows, seg, src_row0, src_stride, dst_pstride,
                                    dst_stride, stream.cuda_stream), 'orl_peer_gather')


def a2a_heads_qkv(q, k, v):
    """[S / N, H, D] x 3 (this rank's tokens, all heads) -> [S, H / N, D] x 3 (all tokens, this rank's heads)"""
    from onereel_b200 import attention as A
    n, r = D.world(), D.rank()
    rows, H, Dh = q.shape
    Hl, es = H // n, _elem(q.dtype)
    sp = space_for(rows, H * Dh, q.dtype, q.device, planes=3, tag='ulysses_in')
    stream = torch.cuda.current_stream(q.device)
    buf, ptrs, _ = sp.gens[sp.next_gen()]
    for pl, x in enumerate((q, k, v)):
        buf[pl].copy_(x.reshape(rows, H * Dh))
    sp.barrier(stream, A._err_word(q.device))
    outs = [q.new_empty(n * rows, Hl, Dh) for _ in range(3)]
    plane = rows * H * Dh * es
    seg = Hl * Dh * es
    _gather([ptrs[p] + pl * plane for pl in range(3) for p in range(n)], [o.data_ptr() for o in outs], 3, n, rows,
            seg, r * seg, H * Dh * es, rows * seg, seg, stream)
    return outs


def out_buffer(total_rows, Hl, Dh, dtype, device, text_rows: int = 0):
    """the attention outputs of this rank's heads in symmetric memory (this call's generation): video [S, H / N, D]
    and, when text_rows > 0, text [text_rows, H / N, D] right after it"""
    sp = space_for(total_rows + text_rows, Hl * Dh, dtype, device, planes=1, tag='ulysses_out')
    g = sp.next_gen()
    flat = sp.gens[g][0][0]
    ov = flat[:total_rows].view(total_rows, Hl, Dh)
    ot = flat[total_rows:total_rows + text_rows].view(text_rows, Hl, Dh) if text_rows else None
    return ov, ot, (sp, g, total_rows)


def a2a_tokens_from(ov, handle, ot=None):
    """[S, H / N, D] in symmetric memory (out_buffer) -> [S / N, H, D]: this rank's tokens of every rank's heads; with
    ot (the text outputs of this rank's heads, same buffer) also [text rows, H, D]: every rank's heads of the text
    rows (what the reference assembles with an all-reduce of head-sliced zeros, hunyuan15.py:279-303). One barrier."""
    from onereel_b200 import attention as A
    sp, g, vrows = handle
    n, r = D.world(), D.rank()
    total, Hl, Dh = ov.shape
    rows, H, es = total // n, Hl * n, _elem(ov.dtype)
    stream = torch.cuda.current_stream(ov.device)
    sp.barrier(stream, A._err_word(ov.device))
    seg = Hl * Dh * es
    ptrs = sp.gens[g][1]
    out = ov.new_empty(rows, H, Dh)
    _gather(ptrs, [out.data_ptr()], 1, n, rows, seg, r * rows * seg, seg, seg, H * Dh * es, stream)
    if ot is None:
        return out
    tr = ot.shape[0]
    text = ot.new_empty(tr, H, Dh)
    if tr:
        _gather(ptrs, [text.data_ptr()], 1, n, tr, seg, vrows * seg, seg, seg, H * Dh * es, stream)
    return out, text
