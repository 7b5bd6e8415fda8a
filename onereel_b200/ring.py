"""Scene Ring attention on B200 — the reference's `onereel.parallel.ring` (src/onereel/parallel/ring.py:1-120), the
USP-Ring baseline of the communication study, on the B200 kernels.

Every scene's video tokens are split into n near-equal contiguous chunks and rank r holds chunk r of every scene; the
rows are permuted so that each rank's rows are one contiguous range (perm / inv). Per layer the K/V of the local rows
travel around the ring in n - 1 point-to-point steps (grouped NCCL send/recv, the next transfer posted before the
visiting block is used); at each step every local query row attends to the rows of the visiting block that lie in its
scene's key set and the partial results are merged by log-sum-exp into an fp32 accumulator. Text queries read their
scene's own frames and their sentence and are computed on every rank in full.

Device work per step: one gather/pack launch (K and V planes) assembling the step's segments from the visiting block
and the text rows (run tables cached per (source rank, layout extra)), one attention launch per query source with LSE
output, and one fp32 merge launch per segment.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from onereel_b200 import attention as A
from onereel_b200 import dist as D
from onereel_b200.pack import RunTable

_VIDEO, _TEXT = 0, 1


class RingPlan:
    """ring.py:23-60: per-scene split, permutation, per-rank rows; keys(src, tag) = per scene, the rows of rank src's
    block in that scene's key set"""

    def __init__(self, layout, n: int, T: int, device='cuda'):
        self.layout, self.n, self.T = layout, n, T
        bounds = [np.linspace(lo * T, hi * T, n + 1).round().astype(int) for lo, hi in layout.ranges]
        self.chunks = [[(j, int(b[r]), int(b[r + 1])) for j, b in enumerate(bounds)] for r in range(n)]
        self.perm = torch.cat([torch.arange(lo, hi) for r in range(n) for _, lo, hi in self.chunks[r]]).to(device)
        self.inv = torch.empty_like(self.perm)
        self.inv[self.perm] = torch.arange(len(self.perm), device=self.perm.device)
        sizes = [sum(hi - lo for _, lo, hi in self.chunks[r]) for r in range(n)]
        c = np.cumsum([0] + sizes)
        self.own = [(int(c[r]), int(c[r + 1])) for r in range(n)]
        self.local = []
        for r in range(n):
            off, rows = 0, []
            for j, lo, hi in self.chunks[r]:
                rows.append((j, off, off + hi - lo))
                off += hi - lo
            self.local.append(rows)
        self._keys, self._steps = {}, {}

    def volume(self) -> float:
        """ring.py:43-45: K/V rows each rank sends per layer (Eq. 2 units)"""
        return 2 * max(b - a for a, b in self.own) * (self.n - 1)

    def keys(self, src: int, tag) -> dict:
        """ring.py:47-60: scene -> LongTensor rows of rank src's block in the scene's key set (None when empty)"""
        key = (src, tag)
        if key not in self._keys:
            self._keys = {k: v for k, v in self._keys.items() if k[1] == tag}
            lay, T = self.layout, self.T
            frame = torch.cat([torch.arange(lo, hi) for _, lo, hi in self.chunks[src]]) // T
            out = {}
            for j in range(lay.n_scenes):
                sel = torch.isin(frame, torch.tensor(lay.key_frames(j))).nonzero().flatten()
                out[j] = sel.to(self.perm.device) if len(sel) else None
            self._keys[key] = out
        return self._keys[key]

    def step_plan(self, r: int, src: int, first: bool, tag, text_ranges, row_bytes: int, device):
        """the segments of ring step (r receiving src's block): video segments of r's scene pieces with keys in the
        block (+ the sentence at the first step), text segments of src's pieces; compiled into a K/V run table over
        (slot 0 = the visiting block's K or V, slot 1 = the text K or V) and the per-segment query ranges"""
        key = (r, src, first, tag, tuple(text_ranges or ()), row_bytes, str(device))
        hit = self._steps.get(key)
        if hit is not None:
            return hit
        keys = self.keys(src, tag)
        segs = []                                   # (kind, q lo, q hi, [(src slot, row lo, row hi)])

        def rle(idx):
            out = []
            for x in idx.tolist():
                if out and out[-1][1] == x:
                    out[-1][1] = x + 1
                else:
                    out.append([x, x + 1])
            return [(_VIDEO, a, b) for a, b in out]
        for j, lo, hi in self.local[r]:
            runs = rle(keys[j]) if keys[j] is not None else []
            if text_ranges is not None and first:
                t0, t1 = text_ranges[j]
                runs = runs + [(_TEXT, t0, t1)]
            if runs and hi > lo:
                segs.append(('v', lo, hi, runs))
        if text_ranges is not None:
            for j, lo, hi in self.local[src]:
                t0, t1 = text_ranges[j]
                runs = ([(_VIDEO, lo, hi)] if hi > lo else []) + ([(_TEXT, t0, t1)] if first else [])
                segs.append(('t', t0, t1, runs))
        src_slot, dst_slot, src_off, dst_off, nbytes, k_start, k_len = [], [], [], [], [], [], []
        row = 0
        for _, _, _, runs in segs:
            k_start.append(row)
            for sl, a, b in runs:
                src_slot.append(sl)
                dst_slot.append(2)
                src_off.append(a * row_bytes)
                dst_off.append(row * row_bytes)
                nbytes.append((b - a) * row_bytes)
                row += b - a
            k_len.append(row - k_start[-1])
        table = RunTable(src_slot, dst_slot, src_off, dst_off, nbytes, device)
        plan = (segs, table, row, k_start, k_len)
        self._steps[key] = plan
        return plan


def attention(plan: RingPlan, q, k, v, eq=None, ek=None, ev=None, text_ranges=None, tag=None):
    """ring.py:73-120: q / k / v [local rows, H, D] in the permuted order; eq / ek / ev [text, H, D] replicated (or
    None). Returns (video out, text out or None), bf16."""
    n, r = D.world(), D.rank()
    Nq, H, Dh = q.shape
    rb = H * Dh * q.element_size()
    o = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    lse = torch.full((H, Nq), float('-inf'), device=q.device)
    has_text = eq is not None
    if has_text:
        ot = torch.zeros(eq.shape, dtype=torch.float32, device=q.device)
        lse_t = torch.full((H, eq.shape[0]), float('-inf'), device=q.device)
    cur, src = torch.stack([k, v]).contiguous(), r
    part_v, lse_pv = torch.empty_like(q), torch.empty(H, Nq, dtype=torch.float32, device=q.device)
    if has_text:
        part_t, lse_pt = torch.empty_like(eq), torch.empty(H, eq.shape[0], dtype=torch.float32, device=q.device)
    for s in range(n):
        works = None
        if s < n - 1:
            nxt = (src - 1) % n
            buf = cur.new_empty((2, plan.own[nxt][1] - plan.own[nxt][0]) + tuple(cur.shape[2:]))
            works = dist.batch_isend_irecv([dist.P2POp(dist.isend, cur, D.peer_rank((r + 1) % n), group=D.group()),
                                            dist.P2POp(dist.irecv, buf, D.peer_rank((r - 1) % n), group=D.group())])
        segs, table, n_keys, k_start, k_len = plan.step_plan(r, src, s == 0, tag, text_ranges if has_text else None,
                                                             rb, q.device)
        if segs:
            kp = q.new_empty(max(n_keys, 1), H, Dh)
            vp = q.new_empty(max(n_keys, 1), H, Dh)
            ptr = lambda x: 0 if x is None else x.data_ptr()
            table.run([cur[0].data_ptr(), ptr(ek), 0, cur[1].data_ptr(), ptr(ev), 0],
                      [0, 0, kp.data_ptr(), 0, 0, vp.data_ptr()], n_planes=2)
            for kind, qsrc, part, lp in (('v', q, part_v, lse_pv), ('t', eq, part_t if has_text else None,
                                                                    lse_pt if has_text else None)):
                idx = [i for i, sg in enumerate(segs) if sg[0] == kind]
                if not idx:
                    continue
                A.attend(qsrc, kp, vp, [segs[i][1] for i in idx], [segs[i][2] - segs[i][1] for i in idx],
                         [k_start[i] for i in idx], [k_len[i] for i in idx], out=part, lse=lp)
                acc, lacc = (o, lse) if kind == 'v' else (ot, lse_t)
                for i in idx:
                    lo, hi = segs[i][1], segs[i][2]
                    A.lse_merge_acc(acc[lo:hi], lacc[:, lo:hi], part[lo:hi], lp[:, lo:hi])
        if works is not None:
            for w in works:
                w.wait()
            cur, src = buf, nxt
    return o.to(q.dtype), (ot.to(eq.dtype) if has_text else None)
