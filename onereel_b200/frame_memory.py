"""Frame memory: representative frames chosen once per denoising step, read by every scene as extra key frames — the
reference's `onereel.frame_memory.FrameMemory` (src/onereel/frame_memory.py:24-132), same API and decisions.

During the conditional pass one layer's video hidden states are mean-pooled per latent frame (each rank pools its own
rows; the per-frame sums and counts are all-reduced over NCCL so every rank sees the same features). After the pass
the candidate frames are clustered by cosine k-means (farthest-point initialisation, at most `iters` Lloyd steps,
deterministic) into budget - len(sink) clusters and each cluster's medoid becomes a representative; at the next step
scene j reads the sink frames and the representatives of other scenes (SceneLayout.extra), which the scene plans
pack as shared frames. Step 0 reads the fallback halo frames instead.

The selection's steps (and so its choices) are those of the reference: the medoid ties resolve to the lowest candidate
and the loop stops when the centroids stop changing. Everything runs where the features live (the GPU); the only
host transfers are the chosen frame indices.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from onereel_b200 import dist as D
from onereel_b200.layout import SceneLayout


class FrameMemory:
    def __init__(self, budget: int = 4, candidates: str = 'all', layer: int | None = None, fallback=(2, 'adj'),
                 sink=(), per_layer: bool = False, iters: int = 20):
        if candidates not in ('all', 'boundary'):
            raise AssertionError(candidates)
        if len(sink) >= budget:
            raise AssertionError('the sink frames are part of the budget')
        self.budget, self.candidates, self.layer, self.fallback, self.iters = budget, candidates, layer, fallback, iters
        self.sink, self.per_layer = tuple(sink), per_layer
        self.layout, self.step, self.pending = None, -1, None
        self.sums, self.counts, self.history, self.extra = {}, {}, [], None

    def reset(self, layout: SceneLayout, n_layers: int):
        """frame_memory.py:34-44: a new request reads the fallback halo frames (and the sink) at step 0"""
        self.layout, self.step, self.pending, self.sums, self.counts, self.history = layout, -1, None, {}, {}, []
        self.n_layers = n_layers
        if self.layer is None:
            self.layer = n_layers // 2
        h, sides = self.fallback
        first = self._extra([], SceneLayout(layout.lengths, halo=h, sides=sides))
        layout.extra = first
        self.extra = {l: first for l in range(n_layers)} if self.per_layer else first

    def _extra(self, reps, halo=None) -> dict:
        """scene -> the sink, representatives (and fallback halo frames) that lie outside the scene, sorted"""
        res = {}
        for j, (lo, hi) in enumerate(self.layout.ranges):
            frames = set(self.sink) | set(reps)
            if halo is not None:
                frames |= set(halo.halo_frames(j))
            res[j] = sorted(f for f in frames if f < lo or f >= hi)
        return res

    def observes(self, layer: int) -> bool:
        return self.per_layer or layer == self.layer

    def begin_step(self, step: int):
        """frame_memory.py:57-69: a new step applies the representatives chosen during the previous one"""
        if step == self.step:
            return
        self.step = step
        if self.pending is None:
            return
        reps, self.pending = self.pending, None
        self.history.append(reps)
        if self.per_layer:
            self.extra = {l: self._extra(r) for l, r in reps.items()}
        else:
            self.extra = self._extra(reps)
            self.layout.extra = self.extra

    def use_layer(self, layer: int):
        """frame_memory.py:71-74: per_layer — switch SceneLayout.extra before block `layer`"""
        if self.per_layer and self.extra is not None:
            self.layout.extra = self.extra[layer]

    def collect(self, frame: torch.Tensor, hs: torch.Tensor, layer: int | None = None):
        """frame_memory.py:76-85: frame [N] latent frame of each local row (-1: not video); hs [N, C]"""
        layer = self.layer if layer is None else layer
        F_ = self.layout.n_frames
        if layer not in self.sums:
            self.sums[layer] = hs.new_zeros(F_, hs.shape[-1], dtype=torch.float32)
            self.counts[layer] = hs.new_zeros(F_, dtype=torch.float32)
        keep = frame >= 0
        idx = frame[keep]
        self.sums[layer].index_add_(0, idx, hs[keep].float())
        self.counts[layer].index_add_(0, idx, torch.ones_like(idx, dtype=torch.float32))

    @torch.no_grad()
    def finish(self):
        """frame_memory.py:87-101: all-reduce the per-frame features (one collective for every observed layer) and
        choose the next step's representatives"""
        if not self.sums:
            return
        layers = sorted(self.sums)
        sums = torch.stack([self.sums[l] for l in layers])
        counts = torch.stack([self.counts[l] for l in layers])
        D.all_reduce(sums)
        D.all_reduce(counts)
        self.sums, self.counts = {}, {}
        feats = F.normalize(sums / counts.clamp_min(1)[..., None], dim=-1)
        if self.per_layer:
            self.pending = {l: self.select(f) for l, f in zip(layers, feats)}
        else:
            self.pending = self.select(feats[0])

    def candidate_frames(self) -> list[int]:
        """frame_memory.py:103-108: every frame, or each scene's first and last frame; sink frames excluded"""
        if self.candidates == 'all':
            cand = list(range(self.layout.n_frames))
        else:
            cand = sorted({f for lo, hi in self.layout.ranges for f in (lo, hi - 1)})
        return [f for f in cand if f not in self.sink]

    def select(self, feats: torch.Tensor) -> list[int]:
        """frame_memory.py:110-132: cosine k-means over the candidates (farthest-point initialisation), the medoid of
        each non-empty cluster (the member nearest its centroid, lowest candidate on ties), sorted"""
        cand = torch.tensor(self.candidate_frames(), device=feats.device)
        x = feats[cand]
        k = min(self.budget - len(self.sink), len(cand))
        centres = [0]
        for _ in range(k - 1):
            dist = (1 - x @ x[centres].T).min(1).values          # cosine distance to the nearest chosen centre
            centres.append(int(dist.argmax()))
        c = x[centres].clone()
        for _ in range(self.iters):
            assign = (x @ c.T).argmax(1)
            new = torch.stack([F.normalize(x[assign == i].mean(0), dim=0) if (assign == i).any() else c[i]
                               for i in range(k)])
            if torch.equal(new, c):
                break
            c = new
        assign = (x @ c.T).argmax(1)
        reps = []
        for i in range(k):
            members = (assign == i).nonzero().flatten()
            if len(members):
                reps.append(int(cand[members[(x[members] @ c[i]).argmax()]]))
        return sorted(reps)
