"""Scene-scope layout builder: a scene layout -> packed segments -> gather/pack run tables + attention work list.

This is the B200 replacement of the reference's per-layer Python segment assembly
(src/onereel/models/hunyuan15.py:153-170 `_segments`, 212-251 `Processor.scene`, 279-303 `Processor.ulysses`;
src/onereel/models/wan.py:110-152 `ranges` / `scene`; src/onereel/attention.py:56-71 `packed`). The reference builds
the segment list with Python loops and torch.cat copies in every layer; here the list is compiled once per layout
(cached: layouts change at most once per denoising step) into

  - a K/V run table: per segment, its key rows as row runs from the sources (this rank's video rows, the received
    exchange buffers, the text rows), executed by the pack kernel for K and V in one launch (two planes);
  - the query rows read in place (video queries straight from the rank's q, text queries from eq) and the outputs
    written in place (video rows of ov, text rows of ot): no q pack and no output scatter;
  - the attention work list and cu_seqlens (bit-exact with attention.cu_seqlens of the reference's call).

Packed segment order (must match the reference, pinned by tests/golden/segments.json): per scene piece j ascending,
the video segment (queries = its token rows; keys = key_frames(j) tokens, then sentence j's text rows), then, if the
rank runs scene j's text queries, the text segment (queries = sentence j; keys = scene j's own frames, then sentence j).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from onereel_b200 import attention as A
from onereel_b200.pack import RunTable

# source ids of row runs
VIDEO, TEXT, REMOTE = 0, 1, 2


def frame_runs(frames) -> list[tuple[int, int]]:
    """frame list in order -> contiguous frame runs (comm.py:115-123 `runs`)"""
    out = []
    for f in frames:
        if out and out[-1][1] == f:
            out[-1][1] = f + 1
        else:
            out.append([f, f + 1])
    return [(a, b) for a, b in out]


def frame_tokens(frames, T: int) -> list[tuple[int, int]]:
    """frame list -> token intervals in the list's order (comm.py:84-85)"""
    return [(a * T, b * T) for a, b in frame_runs(frames)]


@dataclass
class Segment:
    kind: str                      # 'v' video queries, 't' text queries
    scene: int
    q: tuple                       # (source, row lo, row hi) in source rows (VIDEO rows are rank-local)
    kv: list                       # [(source, row lo, row hi)] in key order
    out: tuple                     # where the output rows go: ('v', local lo, hi) or ('t', text lo, hi)

    @property
    def lq(self) -> int:
        return self.q[2] - self.q[1]

    @property
    def lk(self) -> int:
        return sum(hi - lo for _, lo, hi in self.kv)


def text_ranges(counts) -> list[tuple[int, int]]:
    """hunyuan15.py:87-89"""
    c = np.cumsum([0] + list(counts))
    return [(int(c[j]), int(c[j + 1])) for j in range(len(counts))]


def video_key_runs(frames, T, own, remote_index, side=None):
    """token intervals of a frame list -> source runs: rows inside own = (a, b) come from the local rows, the others
    from the received buffer intervals (remote_index: sorted [(token lo, token hi, buffer row of lo)]).
    side 'local' / 'remote' keeps only the local / received runs (comm.py:180-201 `rows(i, side)`)."""
    a, b = own
    runs = []
    for lo, hi in frame_tokens(frames, T):
        while lo < hi:
            if a <= lo < b:
                e = min(hi, b)
                if side != 'remote':
                    runs.append((VIDEO, lo - a, e - a))
            else:
                hit = next(((x, y, r) for x, y, r in remote_index if x <= lo < y), None)
                if hit is None:
                    raise ValueError(f'token {lo} is neither local ({a}, {b}) nor received')
                x, y, r = hit
                e = min(hi, y)
                if side != 'local':
                    runs.append((REMOTE, r + lo - x, r + e - x))
            lo = e
    return _merge_runs(runs)


def _merge_runs(runs):
    out = []
    for s, lo, hi in runs:
        if hi <= lo:
            continue
        if out and out[-1][0] == s and out[-1][2] == lo:
            out[-1] = (s, out[-1][1], hi)
        else:
            out.append((s, lo, hi))
    return out


def scene_segments(layout, T, counts, scenes, text_for, own, remote_index=(), side=None):
    """the packed segments of `scenes` [(j, (token lo, token hi))] on a rank owning video tokens own = (a, b);
    text_for: scenes whose text queries this call runs (hunyuan15.py:153-170). counts None: no joint text (Wan).
    side None: every key; 'local': local video keys and the text (the first pass of the LSE overlap,
    hunyuan15.py:258-260); 'remote': received video keys only (its second pass, 262-268; segments without any are
    dropped)."""
    tr = text_ranges(counts) if counts is not None else None
    a = own[0]
    segs = []
    for j, (qlo, qhi) in scenes:
        kv = video_key_runs(layout.key_frames(j), T, own, remote_index, side)
        if tr is not None and tr[j][1] > tr[j][0] and side != 'remote':
            kv = kv + [(TEXT, tr[j][0], tr[j][1])]
        if kv or side is None:
            segs.append(Segment('v', j, (VIDEO, qlo - a, qhi - a), kv, ('v', qlo - a, qhi - a)))
        if tr is not None and j in text_for:
            t0, t1 = tr[j]
            kv_t = video_key_runs(layout.frames[j], T, own, remote_index, side)
            if side != 'remote':
                kv_t = kv_t + [(TEXT, t0, t1)]
            if kv_t or side is None:
                segs.append(Segment('t', j, (TEXT, t0, t1), kv_t, ('t', t0, t1)))
    return segs


def is_local(layout, T, own, j) -> bool:
    """hunyuan15.py:224: every key frame of scene j lies in the rank's own token range"""
    a, b = own
    return all(a <= lo and hi <= b for lo, hi in frame_tokens(layout.key_frames(j), T))


def pieces(layout, T, own):
    """hunyuan15.py:222-223: scene pieces of a rank's token range and the scenes whose text queries it runs"""
    a, b = own
    mine = [(j, (max(lo * T, a), min(hi * T, b))) for j, (lo, hi) in enumerate(layout.ranges)
            if lo * T < b and hi * T > a]
    text_for = {j for j, (lo, _) in enumerate(layout.ranges) if a <= lo * T < b}
    return mine, text_for


def remote_index_of(layout, T, own_all, r, needed_fn):
    """the receive-buffer layout of comm.HaloExchange for rank r: [(token lo, token hi, buffer row)] sorted by lo"""
    need = needed_fn(layout, T, own_all[r])
    recv = []
    for p, (a, b) in enumerate(own_all):
        if p == r:
            continue
        recv += [(max(lo, a), min(hi, b)) for lo, hi in need if lo < b and hi > a]
    out, off = [], 0
    for lo, hi in sorted(recv):
        out.append((lo, hi, off))
        off += hi - lo
    return out


@dataclass
class ScenePlan:
    """compiled segments of one packed call on one device: K/V run table (slots VIDEO, TEXT, REMOTE -> slot 3 =
    packed buffer), query rows in place per segment, the attention work list, cu_seqlens (host lists cu_q / cu_k;
    cu_k_dev: the packed K/V's cu_seqlens_k as the reference's int32 device tensor, attention.py:28-29, written by
    every pack_kv launch)"""
    segs: list
    row_bytes: int
    heads: int
    device: torch.device
    kv_table: RunTable = None
    n_keys: int = 0
    lq: list = field(default_factory=list)
    lk: list = field(default_factory=list)
    cu_q: list = field(default_factory=list)
    cu_k: list = field(default_factory=list)
    cu_k_dev: torch.Tensor = None
    lk_dev: torch.Tensor = None

    def __post_init__(self):
        rb = self.row_bytes
        src_slot, dst_slot, src_off, dst_off, nbytes = [], [], [], [], []
        row = 0
        for s in self.segs:
            for src, lo, hi in s.kv:
                src_slot.append(src)
                dst_slot.append(3)
                src_off.append(lo * rb)
                dst_off.append(row * rb)
                nbytes.append((hi - lo) * rb)
                row += hi - lo
        self.n_keys = row
        self.kv_table = RunTable(src_slot, dst_slot, src_off, dst_off, nbytes, self.device)
        self.lq = [s.lq for s in self.segs]
        self.lk = [s.lk for s in self.segs]
        self.cu_q = np.concatenate([[0], np.cumsum(self.lq)]).astype(np.int32).tolist()
        self.cu_k = np.concatenate([[0], np.cumsum(self.lk)]).astype(np.int32).tolist()
        self.lk_dev = torch.tensor(self.lk, dtype=torch.int32, device=self.device)
        self.cu_k_dev = torch.empty(len(self.lk) + 1, dtype=torch.int32, device=self.device)

    def pack_kv(self, k_video, v_video, k_text, v_text, k_remote=None, v_remote=None, out=None):
        """one pack launch for K and V (two planes): returns packed (k, v) [n_keys, H, D]; the same launch writes
        cu_k_dev"""
        H, Dh = k_video.shape[1:]
        if out is None:
            kp = k_video.new_empty(self.n_keys, H, Dh)
            vp = k_video.new_empty(self.n_keys, H, Dh)
        else:
            kp, vp = out
        ptr = lambda x: 0 if x is None else x.data_ptr()
        src = [ptr(k_video), ptr(k_text), ptr(k_remote), 0, ptr(v_video), ptr(v_text), ptr(v_remote), 0]
        dst = [0, 0, 0, kp.data_ptr(), 0, 0, 0, vp.data_ptr()]
        self.kv_table.run(src, dst, n_planes=2, seg_len_dev=self.lk_dev, cu_out=self.cu_k_dev)
        return kp, vp


# Optional launch timing for benchmarks: when TIMING is a list, every attend_segments call appends (start, end) CUDA
# events recorded on its stream, with the useful FLOPs it computes.
TIMING = None


_TEXT_STREAM = {}


def attend_segments(plan: ScenePlan, q, eq, kp, vp, ov, ot, lse_v=None, lse_t=None, split_keys=False):
    """attention of every segment of the plan: queries read in place from q (video) and eq (text). Video outputs go
    straight to their rows of ov; text outputs straight to their rows of ot. One kernel launch per query source; the
    text launch (a few long items: every sentence attends to its whole scene) runs on a second stream beside the
    video launch, so its items fill the video launch's last wave instead of running after it (scheduling only: the
    results are the same bits). split_keys: allow the key split of coarse launches (attention.attend)."""
    launches = []
    for kind, qsrc, dst, lse in (('v', q, ov, lse_v), ('t', eq, ot, lse_t)):
        idx = [i for i, s in enumerate(plan.segs) if s.kind == kind]
        if idx:
            launches.append((qsrc, dst, lse, [plan.segs[i].q[1] for i in idx], [plan.segs[i].lq for i in idx],
                             [plan.cu_k[i] for i in idx], [plan.lk[i] for i in idx]))
    if not launches:
        return
    dev = launches[0][0].device
    cur = torch.cuda.current_stream(dev)
    if TIMING is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
    if len(launches) == 2:
        key = dev.index if dev.index is not None else torch.cuda.current_device()
        side = _TEXT_STREAM.get(key)
        if side is None:
            side = _TEXT_STREAM[key] = torch.cuda.Stream(dev)
        side.wait_stream(cur)
        qsrc, dst, lse, qs, ql, ks, kl = launches[1]
        with torch.cuda.stream(side):
            A.attend(qsrc, kp, vp, qs, ql, ks, kl, out=dst, lse=lse, stream=side.cuda_stream)
    qsrc, dst, lse, qs, ql, ks, kl = launches[0]
    A.attend(qsrc, kp, vp, qs, ql, ks, kl, out=dst, lse=lse, split_keys=split_keys)
    if len(launches) == 2:
        cur.wait_stream(side)
    if TIMING is not None:
        e1.record(cur)
        H, Dh = launches[0][0].shape[1:]
        TIMING.append((e0, e1, sum(4.0 * a * b * H * Dh for x in launches for a, b in zip(x[4], x[6]))))
