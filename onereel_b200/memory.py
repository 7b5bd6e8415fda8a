"""Bounded cross-scene memory on the B200 kernels — the reference's `onereel.memory` (src/onereel/memory.py:1-174).

Candidates are the first and last latent frame of every scene (a one-frame scene's frame once). Per (layer, CFG
branch) and head, the L2-normalised candidate keys are clustered by k-means into at most M groups (up to ITERS_INIT
iterations from evenly spaced seeds the first time, ITERS_UPDATE iterations warm-started from the previous centroids
later); each non-empty cluster keeps the candidate nearest its centroid (lowest index on ties). A scene's video
queries read their own frames, their sentence and the representatives that belong to other scenes, in one softmax;
its sentence queries read the scene's frames and the sentence.

B200 layout. The reference repacks the layer head-major (every (head, piece) pair a one-head sequence, q / k / v
gathered row * H + head) because the representatives differ per head. Here the pieces stay multi-head: a video
piece's packed K / V rows are its local keys — identical for every head, gathered by the pack kernel's run table —
followed by M representative slots whose head columns differ (slot r of head h holds that head's r-th foreign
representative). The attention work items are per (piece, head) anyway, so each item's key count is set per head —
local keys plus that head's foreign representatives — in the device work list from the selection, with no host round
trip. Queries are read in place and outputs written in place, as on the scene path.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from onereel_b200 import _lib as L
from onereel_b200 import attention as A
from onereel_b200.layout import SceneLayout
from onereel_b200.pack import RunTable
from onereel_b200.scene import TEXT, VIDEO, Segment, scene_segments

ITERS_INIT, ITERS_UPDATE = 50, 2


def candidate_frames(layout: SceneLayout) -> tuple[list[int], list[int]]:
    """memory.py:31-38: boundary frames (first, last of every scene; a frame once) and the scene of each"""
    frames, owner = [], []
    for j, (lo, hi) in enumerate(layout.ranges):
        for f in ((lo,) if hi - 1 == lo else (lo, hi - 1)):
            frames.append(f)
            owner.append(j)
    return frames, owner


def candidates(layout: SceneLayout, T: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """memory.py:41-46: video token rows of the boundary frames (all tokens of each) and their scene"""
    frames, owner = candidate_frames(layout)
    rows = (torch.as_tensor(frames)[:, None] * T + torch.arange(T)[None]).flatten().to(device)
    scene = torch.as_tensor(owner).repeat_interleave(T).to(device)
    return rows, scene


class BoundaryMemory:
    """memory.py:49-105: per-(layer, branch) centroids and the deterministic representative selection"""

    def __init__(self, M: int = 128):
        self.M = M
        self.centroids = {}                  # key -> [H, M, D] float32

    def reset(self):
        self.centroids = {}

    @torch.no_grad()
    def select(self, key, kc: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """kc [B, H, D] candidate keys -> (rep [H, M'] candidate index, valid [H, M']), M' = min(M, B): one
        representative per non-empty cluster, in ascending cluster order, the rest padded with valid = False.

        The k-means steps are the reference's (memory.py:64-88) so that every rank and the reference pick the same
        set: squared distances |x|^2 - 2 x.c + |c|^2, nearest centroid (lowest index on ties), centroids from one-hot
        matrix products (deterministic sums), an empty cluster keeps its centroid, stop when no centroid moves."""
        x = F.normalize(kc.float().transpose(0, 1), dim=-1)                       # [H, B, D]
        H, B, Dh = x.shape
        M = min(self.M, B)
        c = self.centroids.get(key)
        if c is None or c.shape != (H, M, Dh):
            seeds = torch.linspace(0, B - 1, M, device=x.device).round().long()
            c, iters = x[:, seeds].clone(), ITERS_INIT
        else:
            iters = ITERS_UPDATE
        xx = (x * x).sum(-1, keepdim=True)
        it = 0
        while True:
            d = xx - 2 * x @ c.transpose(1, 2) + (c * c).sum(-1)[:, None]         # [H, B, M]
            z = d.argmin(-1)                                                        # [H, B]
            if it == iters:
                break
            onehot = F.one_hot(z, M).float()
            sums, n = onehot.transpose(1, 2) @ x, onehot.sum(1)
            moved = torch.where((n > 0)[..., None], sums / n.clamp_min(1)[..., None], c)
            it += 1
            if torch.equal(moved, c):
                break
            c = moved
        self.centroids[key] = c
        # the medoid of each cluster: smallest distance to its centroid, then the lowest candidate index
        dist = d.gather(-1, z[..., None])[..., 0]                                   # [H, B]
        dmin = torch.full((H, M), float('inf'), device=x.device).scatter_reduce(1, z, dist, 'amin')
        idx = torch.arange(B, device=x.device).expand(H, B)
        at_min = torch.where(dist == dmin.gather(1, z), idx, torch.full_like(idx, B))
        medoid = torch.full((H, M), B, dtype=torch.long, device=x.device).scatter_reduce(1, z, at_min, 'amin')
        filled = medoid < B
        order = (~filled).to(torch.int8).argsort(dim=1, stable=True)               # non-empty clusters first
        valid = filled.gather(1, order)
        rep = torch.where(valid, medoid.gather(1, order), torch.zeros_like(medoid))
        return rep, valid


class MemoryPlan:
    """one compiled memory call (memory.py:108-140 `Plan` / `make_plan` / `frame_plan`, B200 layout): the segments
    (video segments read the memory, text segments do not), the candidates' sources and scenes; per (heads, head
    dim), compiled on first use: the packed K / V rows (each video segment's local keys, then M' representative
    slots; one spare row at the end), the pack run table and the two launches' work lists (video queries in place
    from one source, text queries from the other)."""

    def __init__(self, segs, cand_local, cand_remote, cand_owner, device):
        """segs: scene.Segment list; cand_local / cand_remote: (candidate positions, source rows) in the local video
        rows / the received buffer; cand_owner: the scene of every candidate (numpy)"""
        self.segs, self.device = segs, torch.device(device)
        self.B = len(cand_owner)
        lt = lambda x: torch.as_tensor(np.asarray(x, dtype=np.int64), device=self.device)
        self.cand_local_pos, self.cand_local_rows = lt(cand_local[0]), lt(cand_local[1])
        self.cand_remote_pos, self.cand_remote_rows = lt(cand_remote[0]), lt(cand_remote[1])
        self.cand_owner = lt(cand_owner)
        self.vid = [i for i, sg in enumerate(segs) if sg.kind == 'v']
        self.txt = [i for i, sg in enumerate(segs) if sg.kind == 't']
        self.n_video = len(self.vid)
        self.H = self.Dh = self.M = None
        self.buffers = None

    @classmethod
    def for_rank(cls, layout: SceneLayout, T: int, counts, own, remote_index, scenes, text_for, device):
        """the pieces of a rank owning video tokens own = (a, b) (hunyuan15.py:305-333 / wan.py:154-173): its scene
        pieces with their scenes' own frames (halo-free) and sentence as local keys, the text segments of text_for;
        candidates from the local rows or the received buffer (remote_index, which must cover them)"""
        plain = SceneLayout(layout.lengths, halo=0)             # local keys: the scene's own frames (memory.py:134)
        segs = scene_segments(plain, T, counts, scenes, text_for, own, remote_index)
        frames, owner = candidate_frames(layout)
        a, b = own
        tokens = (np.asarray(frames)[:, None] * T + np.arange(T)[None]).reshape(-1)
        loc = (tokens >= a) & (tokens < b)
        rem_rows = np.zeros(len(tokens), dtype=np.int64)
        for i in np.flatnonzero(~loc):
            t = int(tokens[i])
            hit = next(((x, y, r) for x, y, r in remote_index if x <= t < y), None)
            if hit is None:
                raise ValueError(f'candidate token {t} is neither local {own} nor received')
            rem_rows[i] = hit[2] + t - hit[0]
        return cls(segs, (np.flatnonzero(loc), tokens[loc] - a), (np.flatnonzero(~loc), rem_rows[~loc]),
                   np.repeat(owner, T), device)

    def compile(self, H: int, Dh: int, M: int):
        """packed row layout, run table and work lists for H heads of Dh and at most M representatives (once)"""
        if self.H is not None:
            assert (self.H, self.Dh, self.M) == (H, Dh, min(M, self.B)), 'a memory plan serves one head layout'
            return
        self.H, self.Dh, self.M = H, Dh, min(M, self.B)
        self.base, self.n_local, row = [], [], 0
        for sg in self.segs:
            self.base.append(row)
            self.n_local.append(sg.lk)
            row += sg.lk + (self.M if sg.kind == 'v' else 0)
        self.spare, self.n_rows = row, row + 1
        lt = lambda x: torch.as_tensor(np.asarray(x, dtype=np.int64), device=self.device)
        vid, txt = self.vid, self.txt
        self.v_scene = lt([self.segs[i].scene for i in vid])
        self.v_base = lt([self.base[i] for i in vid])
        self.v_local = lt([self.n_local[i] for i in vid])
        rb = H * Dh * 2
        src_slot, dst_slot, src_off, dst_off, nbytes = [], [], [], [], []
        for i, sg in enumerate(self.segs):
            row = self.base[i]
            for src, lo, hi in sg.kv:
                src_slot.append(src)
                dst_slot.append(3)
                src_off.append(lo * rb)
                dst_off.append(row * rb)
                nbytes.append((hi - lo) * rb)
                row += hi - lo
        self.table = RunTable(src_slot, dst_slot, src_off, dst_off, nbytes, self.device)
        self.v_work, self.v_items, self.v_key = self._work([self.segs[i].q[1] for i in vid],
                                                           [self.segs[i].lq for i in vid],
                                                           [self.base[i] for i in vid],
                                                           [self.n_local[i] + self.M for i in vid])
        self.t_q = ([self.segs[i].q[1] for i in txt], [self.segs[i].lq for i in txt],
                    [self.base[i] for i in txt], [self.n_local[i] for i in txt])

    def _work(self, qs, ql, ks, kl):
        """attention work list of the video segments with their largest key counts (the LPT order); per item, the
        index (head * n_video + segment) of its key count in the per-call [H, n_video] table"""
        H = self.H
        arrs = [np.ascontiguousarray(x, dtype=np.int32) for x in (qs, ql, ks, kl)]
        n_seg = len(qs)
        need = L.lib().orl_attn_plan_ranges(*(L.i32p(x) for x in arrs), n_seg, H, None, 0)
        n_need = 0 if need >= 0 else -need - 1000
        work = np.zeros(max(n_need, 1), dtype=L.WORK_DTYPE)
        n = L.check(L.lib().orl_attn_plan_ranges(*(L.i32p(x) for x in arrs), n_seg, H, work.ctypes.data, len(work)),
                    'orl_attn_plan_ranges')
        key = work['head'][:n].astype(np.int64) * max(n_seg, 1) + work['seg'][:n].astype(np.int64)
        return (torch.from_numpy(work.view(np.uint8)).to(self.device), n,
                torch.as_tensor(key, device=self.device))

    def kv_buffers(self, like: torch.Tensor):
        """persistent packed K / V (zero-initialised once: representative slots beyond a head's count and the spare
        row are read by the last key tile of a segment and must hold finite values)"""
        if self.buffers is None:
            self.buffers = (like.new_zeros(self.n_rows, self.H, self.Dh), like.new_zeros(self.n_rows, self.H, self.Dh))
        return self.buffers


def frame_plan(layout: SceneLayout, T: int, token_row, Lv: int, q_pieces, text_ranges=None, text_for=(), Sq: int = 0,
               device='cuda') -> MemoryPlan:
    """memory.py:118-140 with the reference's arguments: key buffer = Lv video rows (video token t at token_row[t])
    then the text rows; query buffer = Sq video rows then the text rows; q_pieces [(scene, video query row lo, hi)].
    Video queries read their scene's frames, their sentence and the memory; sentence queries (scenes in text_for)
    their scene's frames and sentence. For MemoryAttention's reference-style call."""
    token_row = np.asarray(torch.as_tensor(token_row).cpu(), dtype=np.int64)

    def frame_runs(frames):
        toks = np.concatenate([np.arange(f * T, (f + 1) * T) for f in frames]) if len(frames) else np.zeros(0, int)
        rows = token_row[toks]
        runs = []
        for r in rows.tolist():
            if runs and runs[-1][2] == r:
                runs[-1] = (VIDEO, runs[-1][1], r + 1)
            else:
                runs.append((VIDEO, r, r + 1))
        return runs
    text = lambda j: ([(VIDEO, Lv + text_ranges[j][0], Lv + text_ranges[j][1])]
                      if text_ranges and text_ranges[j][1] > text_ranges[j][0] else [])
    segs = [Segment('v', j, (VIDEO, lo, hi), frame_runs(layout.frames[j]) + text(j), ('v', lo, hi))
            for j, lo, hi in q_pieces if hi > lo]
    segs += [Segment('t', j, (TEXT, Sq + text_ranges[j][0], Sq + text_ranges[j][1]),
                     frame_runs(layout.frames[j]) + text(j), ('t', text_ranges[j][0], text_ranges[j][1]))
             for j in sorted(text_for) if text_ranges and text_ranges[j][1] > text_ranges[j][0]]
    frames, owner = candidate_frames(layout)
    tokens = (np.asarray(frames)[:, None] * T + np.arange(T)[None]).reshape(-1)
    return MemoryPlan(segs, (np.arange(len(tokens)), token_row[tokens]), (np.zeros(0, int), np.zeros(0, int)),
                      np.repeat(owner, T), device)


class MemoryAttention:
    """memory.py:143-174: scene attention with the bounded memory on the B200 kernels; plans are cached by the
    caller's key"""

    def __init__(self, memory: BoundaryMemory):
        self.memory = memory
        self.plans = {}

    def __call__(self, key, q, k, v, plan: MemoryPlan) -> torch.Tensor:
        """the reference's call (memory.py:150-174): q [Sq, H, D] query buffer, k / v [L, H, D] key buffers laid out
        as `frame_plan` describes -> [Sq, H, D] (rows outside the plan's queries are zero)"""
        out = q.new_zeros(q.shape)
        self.run(key, plan, q, k, v, q, k, v, out, out)
        return out

    @torch.no_grad()
    def run(self, key, plan: MemoryPlan, q, k, v, eq, ek, ev, ov, ot, remote_k=None, remote_v=None):
        """q / k / v: the video rows [rows, H, D] (bf16); eq / ek / ev: the text rows (or None); remote_k / remote_v:
        the received exchange buffers (gather path). Writes the video segments' outputs into ov and the text
        segments' into ot."""
        H, Dh = q.shape[1:]
        plan.compile(H, Dh, self.memory.M)
        dev = q.device
        kc = k.new_empty(plan.B, H, Dh)
        vc = v.new_empty(plan.B, H, Dh)
        for dst, src, r_src in ((kc, k, remote_k), (vc, v, remote_v)):
            if plan.cand_local_pos.numel():
                dst.index_copy_(0, plan.cand_local_pos, src.index_select(0, plan.cand_local_rows))
            if plan.cand_remote_pos.numel():
                dst.index_copy_(0, plan.cand_remote_pos, r_src.index_select(0, plan.cand_remote_rows))
        rep, valid = self.memory.select(key, kc)                                 # [H, M']
        kp, vp = plan.kv_buffers(q)
        ptr = lambda x: 0 if x is None else x.data_ptr()
        plan.table.run([ptr(k), ptr(ek), ptr(remote_k), 0, ptr(v), ptr(ev), ptr(remote_v), 0],
                       [0, 0, 0, kp.data_ptr(), 0, 0, 0, vp.data_ptr()], n_planes=2)
        if plan.n_video:
            foreign = valid[:, None, :] & (plan.cand_owner[rep][:, None, :] != plan.v_scene[None, :, None])
            slot = foreign.cumsum(-1) - 1                                         # [H, n_video, M']
            dst = torch.where(foreign, (plan.v_base + plan.v_local)[None, :, None] + slot,
                              torch.full_like(slot, plan.spare))
            src = rep[:, None, :].expand_as(dst)
            hh = torch.arange(H, device=dev)[:, None, None].expand_as(dst)
            kp[dst.flatten(), hh.flatten()] = kc[src.flatten(), hh.flatten()]
            vp[dst.flatten(), hh.flatten()] = vc[src.flatten(), hh.flatten()]
            k_len = (plan.v_local[None, :] + foreign.sum(-1)).flatten()           # [H * n_video]
            items = plan.v_work.view(torch.int32).view(-1, 8)
            items[:plan.v_items, 3] = k_len[plan.v_key].to(torch.int32)
            A.attend_work(q, kp, vp, plan.v_work, plan.v_items, ov)
        if plan.t_q[0]:
            A.attend(eq, kp, vp, *plan.t_q, out=ot)
        return ov, ot
