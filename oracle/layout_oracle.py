"""CPU restatement of the reference's scene layout, partitioner, exchange sets, Eq. 2 and packed segment order.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). Every function names the reference lines it restates. Integer work is
plain Python; Algorithm 1 runs in float64 numpy exactly as the reference does (np.cumsum, np.searchsorted with the
1e-12 relative tolerance, Python's round-half-even), so its cuts are bit-identical.
"""
from __future__ import annotations

import numpy as np

# src/onereel/parallel/comm.py:15 — fitted cost-model weights (ms per token / per query-key pair and forward)
C_LIN, C_ATT, EFF_SCENE = 0.02581842, 6.753627e-07, 1.0


class Layout:
    """src/onereel/layout.py:10-78 (SceneLayout). lengths: latent frames per scene; halo frames of the neighbours on
    `sides`; extra[j]: frame-memory frames scene j also reads."""

    def __init__(self, lengths, halo=2, sides='adj', extra=None):
        assert sides in ('adj', 'prev', 'next') and all(n > 0 for n in lengths)
        self.lengths, self.halo, self.sides = list(lengths), halo, sides
        self.extra = dict(extra or {})

    @property
    def n_scenes(self):
        return len(self.lengths)

    @property
    def n_frames(self):
        return sum(self.lengths)

    def ranges(self):                                   # layout.py:42-45
        out, start = [], 0
        for n in self.lengths:
            out.append((start, start + n))
            start += n
        return out

    def frames(self, j):                                # layout.py:47-49
        lo, hi = self.ranges()[j]
        return list(range(lo, hi))

    def halo_frames(self, j):                           # layout.py:54-63: previous scene's tail, then next's head
        k = self.halo
        if k == 0:
            return []
        res = []
        if j > 0 and self.sides != 'next':
            res += self.frames(j - 1)[-k:]
        if j + 1 < self.n_scenes and self.sides != 'prev':
            res += self.frames(j + 1)[:k]
        return res

    def shared_frames(self, j):                         # layout.py:65-69: halo, then sorted extras not own / not listed
        lo, hi = self.ranges()[j]
        res = self.halo_frames(j)
        for f in sorted(self.extra.get(j, ())):
            if (f < lo or f >= hi) and f not in res:
                res.append(f)
        return res

    def key_frames(self, j):                            # layout.py:71-73
        return self.frames(j) + self.shared_frames(j)

    def key_range(self, j):                             # layout.py:75-78
        kf = self.key_frames(j)
        return min(kf), max(kf) + 1


def even_lengths(n_frames, n_scenes):                   # layout.py:24-28: scene of frame f = f * S // F
    counts = [0] * n_scenes
    for f in range(n_frames):
        counts[f * n_scenes // n_frames] += 1
    return counts


# ---------------------------------------------------------------- intervals (comm.py:69-85, 115-123)

def merge(iv):
    res = []
    for lo, hi in sorted(x for x in iv if x[0] < x[1]):
        if res and lo <= res[-1][1]:
            res[-1] = (res[-1][0], max(res[-1][1], hi))
        else:
            res.append((lo, hi))
    return res


def clip(iv, a, b):
    return [(max(lo, a), min(hi, b)) for lo, hi in iv if lo < b and hi > a]


def runs(frames):
    res = []
    for f in frames:
        if res and res[-1][1] == f:
            res[-1] = (res[-1][0], f + 1)
        else:
            res.append((f, f + 1))
    return res


def frame_tokens(frames, T):
    return [(lo * T, hi * T) for lo, hi in runs(frames)]


# ---------------------------------------------------------------- Algorithm 1 and Eq. 2 (comm.py:18-112)

def query_cost(lay, T, text=None, extra_keys=0):   # comm.py:18-22
    res = []
    for j in range(lay.n_scenes):
        keys = len(lay.key_frames(j)) * T + (text[j] if text else 0) + extra_keys
        res.append(C_LIN + C_ATT * EFF_SCENE * keys)
    return res


def balanced(sizes, cost, n):                       # comm.py:25-40 (paper Algorithm 1), float64 throughout
    L = sum(sizes)
    assert L >= n
    starts = np.cumsum([0] + list(sizes))
    work = np.cumsum([0.0] + [m * c for m, c in zip(sizes, cost)])
    per_rank = work[-1] / n
    cuts = [0]
    for p in range(1, n):
        i = int(np.searchsorted(work, p * per_rank - 1e-12 * work[-1], side='left'))
        off = int(round((p * per_rank - work[i - 1]) / cost[i - 1]))
        cuts.append(min(max(int(starts[i - 1]) + off, cuts[-1] + 1), L - (n - p)))
    cuts.append(L)
    return [(cuts[p], cuts[p + 1]) for p in range(n)]


def partition(lay, n, T, mode, text=None, extra_keys=0, granularity='balanced'):   # comm.py:43-66
    L = lay.n_frames * T
    if mode == 'ulysses' or n == 1:
        assert L % n == 0
        return [(r * L // n, (r + 1) * L // n) for r in range(n)]
    if granularity == 'tokens':
        return [(r * L // n, (r + 1) * L // n) for r in range(n)]
    own = balanced([m * T for m in lay.lengths], query_cost(lay, T, text, extra_keys), n)
    if granularity == 'scenes':
        starts = [0]
        for m in lay.lengths:
            starts.append(starts[-1] + m * T)
        assert lay.n_scenes >= n
        cuts = [0]
        for p in range(1, n):
            ok = [s for s in starts[1:-1] if s > cuts[-1] and starts.index(s) <= lay.n_scenes - (n - p)]
            cuts.append(min(ok, key=lambda s: abs(s - own[p][0])))
        cuts.append(L)
        return [(cuts[p], cuts[p + 1]) for p in range(n)]
    assert granularity == 'balanced'
    return own


def needed(lay, T, own, extra=()):                  # comm.py:88-96
    a, b = own
    iv = frame_tokens(sorted(extra), T)
    for j, (lo, hi) in enumerate(lay.ranges()):
        if lo * T < b and hi * T > a:
            iv += [(lo * T, hi * T)] + frame_tokens(lay.shared_frames(j), T)
    res = []
    for lo, hi in merge(iv):
        for x in ((lo, min(hi, a)), (max(lo, b), hi)):
            if x[0] < x[1]:
                res.append(x)
    return res


def gather_rows(lay, own, T, extra=()):             # comm.py:99-101
    return max(sum(hi - lo for lo, hi in needed(lay, T, o, extra)) for o in own)


def eq2(remote_rows, L, n, theta):                  # comm.py:104-108
    vg, vu = 2 * remote_rows, 4 * L * (n - 1) / n ** 2
    return dict(path='scene' if vg < theta * vu else 'ulysses', V_G=vg, V_U=vu, theta=theta)


def choose_path(lay, own, T, theta, extra=()):      # comm.py:111-112
    return eq2(gather_rows(lay, own, T, extra), lay.n_frames * T, len(own), theta)


def plan_parallel(lay, n, T, mode, heads, text=None, theta=1.0, granularity='balanced'):
    """src/onereel/models/hunyuan15.py:553-573 (wan.py:248-271 is the same with text=None): (run_mode, own, path)"""
    if n == 1:
        return 'scene', [(0, lay.n_frames * T)], {}
    gather = partition(lay, n, T, 'scene', text, 0, granularity)
    path = choose_path(lay, gather, T, theta)
    path['ulysses_ok'] = lay.n_frames * T % n == 0 and heads % n == 0
    run_mode = mode if mode != 'auto' else (path['path'] if path['ulysses_ok'] else 'scene')
    assert run_mode != 'ulysses' or path['ulysses_ok']
    own = gather if run_mode == 'scene' else partition(lay, n, T, 'ulysses')
    return run_mode, own, path


# ---------------------------------------------------------------- packed segment order (hunyuan15.py:153-170)

def text_ranges(counts):
    """hunyuan15.py:87-89: per sentence (t0, t1) in the concatenated text rows"""
    res, c = [], 0
    for n in counts:
        res.append((c, c + n))
        c += n
    return res


def token_rows(frames, T):
    """video token rows of a frame list, in the list's order (the reference's kf/vf row functions)"""
    return [t for lo, hi in frame_tokens(frames, T) for t in range(lo, hi)]


def hunyuan_segments(lay, T, counts, scenes, text_for):
    """the packed segments of hunyuan15._segments (153-170) as source rows. scenes: [(j, (q token lo, hi))].
    Returns [(kind, j, q_rows, k_rows)] where a video row is its token index t >= 0 and text row i is ('t', i): q_rows of
    a video segment are tokens lo..hi, of a text segment sentence j's rows; k_rows = key frames' tokens then sentence
    j's rows (video segment) or own frames' tokens then sentence j's rows (text segment)."""
    tr = text_ranges(counts)
    res = []
    for j, (qlo, qhi) in scenes:
        t0, t1 = tr[j]
        txt = [('t', i) for i in range(t0, t1)]
        res.append(('v', j, list(range(qlo, qhi)), token_rows(lay.key_frames(j), T) + txt))
        if j in text_for:
            res.append(('t', j, txt, token_rows(lay.frames(j), T) + txt))
    return res


def scene_pieces(lay, T, own):
    """hunyuan15.py:222-223: the scene pieces of a rank's range and the scenes whose text queries it runs"""
    a, b = own
    mine = [(j, (max(lo * T, a), min(hi * T, b))) for j, (lo, hi) in enumerate(lay.ranges()) if lo * T < b and hi * T > a]
    text_for = {j for j, (lo, _) in enumerate(lay.ranges()) if a <= lo * T < b}
    return mine, text_for


def is_local(lay, T, own, j):
    """hunyuan15.py:224: every key frame of scene j lies in the rank's own token range"""
    a, b = own
    return all(a <= lo and hi <= b for lo, hi in frame_tokens(lay.key_frames(j), T))


def cu_seqlens(lengths):
    """src/onereel/attention.py:28-29: int32 [0, cumsum]"""
    return np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)


def flops(segs_lq_lk, H, D):
    """experiments/kernel_breakdown.py:101: useful FLOPs = sum over segments of 4 * lq * lk * H * D"""
    return sum(4.0 * lq * lk * H * D for lq, lk in segs_lq_lk)
