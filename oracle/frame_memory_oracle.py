"""CPU restatement of the reference's frame-memory selection — TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

src/onereel/frame_memory.py: per-frame mean pooling of hidden states (76-85 `collect`, 87-101 `finish`), the candidate
frames (103-108) and the representative choice (110-132 `select`): cosine k-means over L2-normalised features with
farthest-point initialisation from the first candidate, Lloyd steps (assignment = first maximum of x.c; centroid =
normalised mean of its members, unchanged when empty) until no centroid changes or `iters` steps, then per non-empty
cluster the member with the largest x.c (the first on ties), sorted. Restated in float64 numpy; checked against the
golden selections that tests/golden/make_golden.py records by running the reference itself.
"""
from __future__ import annotations

import numpy as np


def pool(frame: np.ndarray, hs: np.ndarray, n_frames: int):
    """frame_memory.py:76-85: per-frame sums and row counts (rows with frame < 0 skipped)"""
    keep = frame >= 0
    sums = np.zeros((n_frames, hs.shape[1]))
    np.add.at(sums, frame[keep], hs[keep].astype(np.float64))
    counts = np.bincount(frame[keep], minlength=n_frames).astype(np.float64)
    return sums, counts


def features(sums: np.ndarray, counts: np.ndarray) -> np.ndarray:
    """frame_memory.py:97: L2-normalised per-frame means (norm clamped at 1e-12)"""
    mean = sums / np.maximum(counts, 1.0)[:, None]
    return mean / np.maximum(np.linalg.norm(mean, axis=1, keepdims=True), 1e-12)


def candidate_frames(lengths, candidates: str, sink) -> list[int]:
    """frame_memory.py:103-108"""
    bounds = np.cumsum([0] + list(lengths))
    if candidates == 'all':
        frames = list(range(int(bounds[-1])))
    else:
        frames = sorted({int(f) for lo, hi in zip(bounds[:-1], bounds[1:]) for f in (lo, hi - 1)})
    return [f for f in frames if f not in set(sink)]


# Two members of one cluster can be equally near its centroid in exact arithmetic (always so in a two-member cluster:
# both have the same cosine to their normalised mean), and then floating-point rounding alone picks the medoid. The
# reference states the rule "lowest index on ties"; scores within TIE_TOL count as ties here and in the kernel.
TIE_TOL = 1e-6


def select(feats: np.ndarray, cand: list[int], k: int, iters: int = 20, detail: bool = False):
    """frame_memory.py:110-132; detail: also return per cluster (member candidates, their x.c scores)"""
    x = feats[np.asarray(cand, dtype=np.int64)]
    k = min(k, len(cand))
    if k <= 0:
        return []
    dist = 1.0 - x @ x[0]
    centres = [0]
    for _ in range(k - 1):
        nxt = int(np.argmax(dist))                     # np.argmax returns the first maximum
        centres.append(nxt)
        dist = np.minimum(dist, 1.0 - x @ x[nxt])
    c = x[centres].copy()
    for _ in range(iters):
        z = np.argmax(x @ c.T, axis=1)
        new = c.copy()
        for i in range(k):
            members = x[z == i]
            if len(members):
                m = members.mean(0)
                new[i] = m / max(np.linalg.norm(m), 1e-12)
        if np.array_equal(new, c):
            break
        c = new
    z = np.argmax(x @ c.T, axis=1)
    reps, clusters = [], []
    for i in range(k):
        members = np.nonzero(z == i)[0]
        if len(members):
            score = x[members] @ c[i]
            first = int(np.nonzero(score >= score.max() - TIE_TOL)[0][0])
            reps.append(cand[int(members[first])])
            clusters.append(([cand[int(m)] for m in members], score.tolist()))
    return (sorted(reps), clusters) if detail else sorted(reps)


def tie_explains(mine: list[int], theirs: list[int], clusters, tol: float = 1e-5) -> bool:
    """True when two selections differ only in medoids that tie within `tol` in the same clusters (a decision that
    floating-point rounding alone made)"""
    if len(mine) != len(theirs):
        return False
    a, b = sorted(set(mine) - set(theirs)), sorted(set(theirs) - set(mine))
    for x in a:
        cl = next((c for c in clusters if x in c[0]), None)
        if cl is None:
            return False
        members, score = cl
        alt = [m for m in b if m in members]
        if len(alt) != 1 or abs(score[members.index(alt[0])] - score[members.index(x)]) > tol:
            return False
        b.remove(alt[0])
    return not b


def scene_reads(lengths, frames, halo_frames=None) -> dict:
    """frame_memory.py:46-53 `_extra`: scene j -> the sorted frames outside scene j among `frames` (plus its fallback
    halo frames)"""
    bounds = np.cumsum([0] + list(lengths))
    out = {}
    for j, (lo, hi) in enumerate(zip(bounds[:-1], bounds[1:])):
        pool_ = set(frames) | set(halo_frames[j] if halo_frames else ())
        out[j] = sorted(int(f) for f in pool_ if not lo <= f < hi)
    return out
