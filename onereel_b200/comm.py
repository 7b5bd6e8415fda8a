"""Partitioning, path choice (Eq. 2) and the collectives of the two parallel paths (K/V gathering, Ulysses) — the
reference's `onereel.parallel.comm` (src/onereel/parallel/comm.py:1-308), same names and return values.

The planner (query_cost, balanced, partition, needed, gather_rows, choose_path) runs in the native library
(csrc/planner.cpp) with the reference's float64 arithmetic, so partitions are bit-identical. The exchange posts
grouped NCCL point-to-point transfers on the process group's (high-priority) NCCL stream; received intervals land in
one contiguous buffer per tensor, addressed by `remote_index` so the pack kernel reads them like local rows.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from onereel_b200 import _lib as L
from onereel_b200 import dist as D

_MODE = {'scene': 0, 'ulysses': 1}
_GRAN = {'balanced': 0, 'tokens': 1, 'scenes': 2}
_SIDES = {'adj': 0, 'prev': 1, 'next': 2}


class _CLayout:
    """an orl_layout over numpy buffers kept alive with it"""

    def __init__(self, layout):
        self.lengths = np.ascontiguousarray(layout.lengths, dtype=np.int32)
        ex = [list(layout.extra.get(j, ())) for j in range(layout.n_scenes)]
        self.offs = np.ascontiguousarray(np.concatenate([[0], np.cumsum([len(e) for e in ex])]), dtype=np.int32)
        self.frames = np.ascontiguousarray([f for e in ex for f in e] or [0], dtype=np.int32)
        self.s = L.Layout(L.i32p(self.lengths), layout.n_scenes, layout.halo, _SIDES[layout.sides], L.i32p(self.offs),
                          L.i32p(self.frames))

    @property
    def ref(self):
        return ctypes.byref(self.s)


def _i32(x):
    return None if x is None else np.ascontiguousarray(x, dtype=np.int32)


def query_cost(layout, T: int, text=None, extra_keys: int = 0) -> list[float]:
    """comm.py:18-22"""
    cl = _CLayout(layout)
    out = np.zeros(layout.n_scenes)
    t = _i32(text) if text else None
    L.check(L.lib().orl_query_cost(cl.ref, T, None if t is None else L.i32p(t), extra_keys,
                                   out.ctypes.data_as(ctypes.POINTER(ctypes.c_double))), 'orl_query_cost')
    return out.tolist()


def balanced(sizes, cost, n: int) -> list[tuple[int, int]]:
    """comm.py:25-40 (paper Algorithm 1)"""
    s = np.ascontiguousarray(sizes, dtype=np.int64)
    c = np.ascontiguousarray(cost, dtype=np.float64)
    b = np.zeros(n + 1, dtype=np.int64)
    rc = L.lib().orl_balanced(L.i64p(s), c.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), len(s), n, L.i64p(b))
    if rc < 0:
        raise AssertionError(f'{int(s.sum())} queries for {n} ranks')
    return [(int(b[p]), int(b[p + 1])) for p in range(n)]


def partition(layout, n: int, T: int, mode: str, text=None, extra_keys: int = 0,
              granularity: str = 'balanced') -> list[tuple[int, int]]:
    """comm.py:43-66: per rank (video token lo, hi)"""
    Ltok = layout.n_frames * T
    if (mode == 'ulysses' or n == 1) and Ltok % n:
        raise AssertionError(f'{Ltok} video tokens do not split evenly over {n} ranks')
    if granularity == 'scenes' and mode != 'ulysses' and n > 1 and layout.n_scenes < n:
        raise AssertionError(f'{layout.n_scenes} scenes for {n} ranks')
    cl = _CLayout(layout)
    t = _i32(text) if text else None
    b = np.zeros(n + 1, dtype=np.int64)
    L.check(L.lib().orl_partition(cl.ref, T, n, _MODE[mode], None if t is None else L.i32p(t), extra_keys,
                                  _GRAN[granularity], L.i64p(b)), 'orl_partition')
    return [(int(b[p]), int(b[p + 1])) for p in range(n)]


def merge(iv) -> list[tuple[int, int]]:
    """comm.py:69-77: union of half-open intervals, sorted and merged"""
    out = []
    for lo, hi in sorted(x for x in iv if x[0] < x[1]):
        if out and lo <= out[-1][1]:
            out[-1] = (out[-1][0], max(out[-1][1], hi))
        else:
            out.append((lo, hi))
    return out


def clip(iv, a: int, b: int) -> list[tuple[int, int]]:
    """comm.py:80-81"""
    return [(max(lo, a), min(hi, b)) for lo, hi in iv if lo < b and hi > a]


def runs(frames) -> list[tuple[int, int]]:
    """comm.py:115-123: frame list (in order) -> contiguous runs"""
    out = []
    for f in frames:
        if out and out[-1][1] == f:
            out[-1] = (out[-1][0], f + 1)
        else:
            out.append((f, f + 1))
    return out


def frame_tokens(frames, T: int) -> list[tuple[int, int]]:
    """comm.py:84-85"""
    return [(lo * T, hi * T) for lo, hi in runs(frames)]


def needed(layout, T: int, own, extra=()) -> list[tuple[int, int]]:
    """comm.py:88-96: video token intervals outside `own` that the scenes intersecting it read"""
    cl = _CLayout(layout)
    ex = _i32(list(extra) or [0])
    n_ex = len(list(extra))
    rc = L.lib().orl_needed(cl.ref, T, own[0], own[1], L.i32p(ex), n_ex, None, 0)
    cap = -rc - 1000 if rc < 0 else 0
    buf = np.zeros(2 * max(cap, 1), dtype=np.int64)
    n = L.check(L.lib().orl_needed(cl.ref, T, own[0], own[1], L.i32p(ex), n_ex, L.i64p(buf), cap), 'orl_needed')
    return [(int(buf[2 * i]), int(buf[2 * i + 1])) for i in range(n)]


def gather_rows(layout, own, T: int, extra=()) -> int:
    """comm.py:99-101"""
    return max(sum(hi - lo for lo, hi in needed(layout, T, o, extra)) for o in own)


def eq2(remote_rows: int, L_: int, n: int, theta: float) -> dict:
    """comm.py:104-108: gather when V_G < theta * V_U"""
    vg, vu = 2 * remote_rows, 4 * L_ * (n - 1) / n ** 2
    return dict(path='scene' if vg < theta * vu else 'ulysses', V_G=vg, V_U=vu, theta=theta)


def choose_path(layout, own, T: int, theta: float, extra=()) -> dict:
    """comm.py:111-112, computed natively (orl_choose_path)"""
    cl = _CLayout(layout)
    b = np.ascontiguousarray([o[0] for o in own] + [own[-1][1]], dtype=np.int64)
    ex = _i32(list(extra) or [0])
    p = L.Path()
    L.check(L.lib().orl_choose_path(cl.ref, T, L.i64p(b), len(own), float(theta), L.i32p(ex), len(list(extra)),
                                    ctypes.byref(p)), 'orl_choose_path')
    return dict(path='scene' if p.gather else 'ulysses', V_G=int(p.remote_rows) * 2, V_U=p.V_U, theta=theta)


# ------------------------------------------------------------------------------------------------ K/V gathering

def _intersect(x, y) -> list[tuple[int, int]]:
    """intersection of two sorted lists of disjoint intervals"""
    out, i, j = [], 0, 0
    while i < len(x) and j < len(y):
        lo, hi = max(x[i][0], y[j][0]), min(x[i][1], y[j][1])
        if lo < hi:
            out.append((lo, hi))
        if x[i][1] < y[j][1]:
            i += 1
        else:
            j += 1
    return out


def _subtract(x, y) -> list[tuple[int, int]]:
    """x minus y, both sorted lists of disjoint intervals"""
    out = []
    for lo, hi in x:
        cur = lo
        for u, w in y:
            if w <= cur or u >= hi:
                continue
            if u > cur:
                out.append((cur, u))
            cur = max(cur, w)
        if cur < hi:
            out.append((cur, hi))
    return out


def exchange_plan(layout, own, T: int, extra=()):
    """the operation lists of one K/V exchange, for every rank at once (every rank computes the same lists):
    need[r] = the token intervals rank r reads outside its range; common[p] = the intervals of owner p's range that
    every other rank reads (broadcast from p, when there are more than 2 ranks); p2p[(p, q)] = the remaining
    intervals owner p sends to reader q, in token order"""
    n = len(own)
    need = [sorted(needed(layout, T, o, extra)) for o in own]
    common = []
    for p in range(n):
        c = [tuple(own[p])] if n > 2 else []
        for q in range(n):
            if q != p and c:
                c = _intersect(c, need[q])
        common.append(c)
    p2p = {(p, q): _subtract(clip(need[q], *own[p]), common[p]) for p in range(n) for q in range(n) if p != q}
    return need, common, p2p


PEER_UNAVAILABLE = None       # why the peer-memory exchange could not be set up in this process (then NCCL is used)


def kv_exchange(kind, layout, own, T, k, v, extra=()):
    """the layer's K/V exchange: over peer memory (kind 'peer': symmetric buffers, a device barrier and one pull
    launch, onereel_b200.peer) or NCCL send/recv (kind 'nccl': HaloExchange, the reference's scheme). Both deliver
    the same receive buffers bit for bit. If symmetric memory cannot be set up, the NCCL path is used and the reason
    kept in PEER_UNAVAILABLE."""
    global PEER_UNAVAILABLE
    if kind == 'peer' and PEER_UNAVAILABLE is None:
        from onereel_b200 import peer
        try:
            return peer.PeerExchange(layout, own, T, k, v, extra)
        except (RuntimeError, AttributeError, NotImplementedError) as e:
            if peer.initialised():
                raise
            PEER_UNAVAILABLE = f'{type(e).__name__}: {e}'
            import warnings
            warnings.warn(f'peer-memory K/V exchange unavailable, using NCCL: {PEER_UNAVAILABLE}')
    elif kind not in ('peer', 'nccl'):
        raise ValueError(f'exchange must be peer or nccl, got {kind!r}')
    return HaloExchange(layout, own, T, k, v, extra)


class HaloExchange:
    """comm.py:126-201. Posts the K/V exchange of one layer: rank r receives the tokens it reads from their owners and
    sends every peer the tokens of its range that the peer reads. Received intervals land back to back in one buffer
    per tensor: `remote_index` = [(token lo, token hi, buffer row of lo)], `remote_k` / `remote_v` = the buffers.
    heads: exchange only these heads (contiguous copies are made, as the reference does).

    Rows that every other rank reads (frame-memory frames, shared by every scene, are the common case) travel as one
    NCCL broadcast from their owner instead of one send per peer: on NVSwitch the broadcast leaves the owner once and
    is replicated by the switch (NVLS) or along a ring, where the reference's per-peer sends leave the owner n - 1
    times. Everything else moves point to point, per peer K then V of each interval in token order on both sides, as
    the reference. Every rank derives the same operation list from the global plan, so the collectives match.
    collectives: None (torch.distributed) or an onereel_b200.collectives.NcclComm (the C ABI's orl_comm_*)."""

    def __init__(self, layout, own, T, k, v, extra=(), heads=None, collectives=None):
        if heads is not None:
            k, v = k[:, heads].contiguous(), v[:, heads].contiguous()
        self.T, self.k, self.v, self.L = T, k, v, layout.n_frames * T
        r, n = D.rank(), D.world()
        self.a, self.b = own[r]
        self.works, self.keep, self.remote_index = [], [k, v], []
        self.remote_k = self.remote_v = None
        self.broadcast_rows = 0                  # rows this rank takes part in broadcasting (sent or received)
        if n == 1:
            return
        need, common, p2p = exchange_plan(layout, own, T, extra)
        recv = [(p, lo, hi) for p in range(n) if p != r for lo, hi in clip(need[r], *own[p])]
        rows = sum(hi - lo for _, lo, hi in recv)
        self.remote_k = k.new_empty((rows,) + tuple(k.shape[1:]))
        self.remote_v = v.new_empty((rows,) + tuple(v.shape[1:]))
        off = 0
        for p, lo, hi in sorted(recv, key=lambda x: x[1]):
            self.remote_index.append((lo, hi, off))
            off += hi - lo

        def recv_rows(lo, hi):
            x, y, o = next(t for t in self.remote_index if t[0] <= lo and hi <= t[1])
            return self.remote_k[o + lo - x:o + hi - x], self.remote_v[o + lo - x:o + hi - x]
        g = D.group()
        self.collectives = collectives
        bcasts, sends, recvs = [], [], []
        for p in range(n):
            for lo, hi in common[p]:
                bk, bv = ((k[lo - self.a:hi - self.a], v[lo - self.a:hi - self.a]) if p == r else recv_rows(lo, hi))
                bcasts += [(bk, p), (bv, p)]
                self.broadcast_rows += hi - lo
        for p in range(n):
            if p == r:
                continue
            for lo, hi in p2p[(r, p)]:
                sends += [(p, k[lo - self.a:hi - self.a]), (p, v[lo - self.a:hi - self.a])]
            for lo, hi in p2p[(p, r)]:
                bk, bv = recv_rows(lo, hi)
                recvs += [(p, bk), (p, bv)]
        if collectives is not None:
            for x, p in bcasts:
                collectives.broadcast(x, D.peer_rank(p))
            if sends or recvs:
                collectives.exchange([(D.peer_rank(p), x) for p, x in sends], [(D.peer_rank(p), x) for p, x in recvs])
            return
        for x, p in bcasts:
            self.works.append(dist.broadcast(x, D.peer_rank(p), group=g, async_op=True))
        # per peer: sends (K then V of each interval in token order), then receives, as batch_isend_irecv expects
        ops = []
        for p in range(n):
            if p == r:
                continue
            ops += [dist.P2POp(dist.isend, x, D.peer_rank(p), group=g) for q, x in sends if q == p]
            ops += [dist.P2POp(dist.irecv, x, D.peer_rank(p), group=g) for q, x in recvs if q == p]
        if ops:
            self.works += dist.batch_isend_irecv(ops)

    def wait(self, timeout_s: float | None = None):
        """the exchange's results are usable on the current stream after this (torch.distributed: Work.wait;
        NcclComm: a device-side dependency, or the timeout-aware host wait when timeout_s is given)"""
        if getattr(self, 'collectives', None) is not None:
            self.collectives.wait(timeout_s)
            self.collectives = None
        for w in self.works:
            w.wait()
        self.works = []

    def buffer(self):
        """comm.py:162-173: (k, v, token_row) — local rows, then the received intervals; token_row [L] (CPU) buffer row
        of each held video token, -1 for tokens not held"""
        token_row = torch.full((self.L,), -1, dtype=torch.long)
        token_row[self.a:self.b] = torch.arange(self.b - self.a)
        base = self.b - self.a
        for lo, hi, off in self.remote_index:
            token_row[lo:hi] = base + off + torch.arange(hi - lo)
        if self.remote_k is None:
            return self.k, self.v, token_row
        return torch.cat([self.k, self.remote_k]), torch.cat([self.v, self.remote_v]), token_row

    def rows(self, i: int, side: str | None = None):
        """comm.py:180-201: i = 0 for K, 1 for V: callable frame list -> rows (in the list's order); side 'local' /
        'remote': only the rows held locally / received"""
        local = (self.k, self.v)[i]
        remote = (self.remote_k, self.remote_v)[i]
        a, b = self.a, self.b

        def get(frames):
            parts = []
            for lo, hi in frame_tokens(frames, self.T):
                while lo < hi:
                    if a <= lo < b:
                        e = min(hi, b)
                        if side != 'remote':
                            parts.append(local[lo - a:e - a])
                    else:
                        x, y, off = next(t for t in self.remote_index if t[0] <= lo < t[1])
                        e = min(hi, y)
                        if side != 'local':
                            parts.append(remote[off + lo - x:off + e - x])
                    lo = e
            return torch.cat(parts) if parts else local[:0]
        return get


def send_text_rows(x: torch.Tensor, layout, own, T: int, text_ranges) -> None:
    """comm.py:204-223: the text query outputs of scene j, computed on the rank holding its first frame, go to every
    other rank whose video range intersects scene j (in place into x)"""
    r, n = D.rank(), D.world()
    if n == 1:
        return
    touches = lambda p, lo, hi: lo * T < own[p][1] and hi * T > own[p][0]
    ops, g = [], D.group()
    for (lo, hi), (t0, t1) in zip(layout.ranges, text_ranges):
        if t0 == t1:
            continue
        src = next(p for p in range(n) if own[p][0] <= lo * T < own[p][1])
        if src == r:
            ops += [dist.P2POp(dist.isend, x[t0:t1], D.peer_rank(p), group=g) for p in range(n)
                    if p != r and touches(p, lo, hi)]
        elif touches(r, lo, hi):
            ops.append(dist.P2POp(dist.irecv, x[t0:t1], D.peer_rank(src), group=g))
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()


# ------------------------------------------------------------------------------------------------ Ulysses

def a2a_heads(x: torch.Tensor) -> torch.Tensor:
    """comm.py:276-284: [S/N, H, D] (local tokens) -> [S, H/N, D] (all tokens, local heads)"""
    n = D.world()
    if n == 1:
        return x
    x = x.unflatten(1, (n, x.shape[1] // n)).transpose(0, 1).contiguous()
    y = torch.empty_like(x)
    dist.all_to_all_single(y, x, group=D.group())
    return y.flatten(0, 1)


def a2a_tokens(x: torch.Tensor) -> torch.Tensor:
    """comm.py:287-295: [S, H/N, D] -> [S/N, H, D]"""
    n = D.world()
    if n == 1:
        return x
    x = x.unflatten(0, (n, -1)).contiguous()
    y = torch.empty_like(x)
    dist.all_to_all_single(y, x, group=D.group())
    return y.transpose(0, 1).flatten(1, 2)


def gather_tokens(x: torch.Tensor, own) -> torch.Tensor:
    """comm.py:298-308: [B, local tokens, C] -> [B, all tokens, C] for per-rank ranges of unequal length"""
    n = D.world()
    if n == 1:
        return x
    m = max(b - a for a, b in own)
    buf = x.new_zeros(x.shape[0], m, x.shape[2])
    buf[:, :x.shape[1]] = x
    allb = [torch.empty_like(buf) for _ in range(n)]
    dist.all_gather(allb, buf, group=D.group())
    return torch.cat([y[:, :b - a] for y, (a, b) in zip(allb, own)], 1)
