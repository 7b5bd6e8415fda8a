"""Frame memory on B200 — the drop-in for the reference's `onereel.frame_memory.FrameMemory`
(src/onereel/frame_memory.py:24-132): same constructor, methods and decisions; the device work is two kernels.

What it does (the reference's behaviour): once per denoising step, the conditional pass pools one layer's video hidden
states per latent frame; the pooled features choose `budget - len(sink)` representative frames by cosine k-means; at
the next step every scene reads the sink frames and the representatives of other scenes as extra key frames
(SceneLayout.extra). Step 0 reads the fallback halo frames. per_layer: every layer pools and chooses for itself.

How it runs here:
  - each observed layer owns one fp32 accumulator on the device, a row per latent frame holding the C feature sums and
    then the row count; `collect` adds a layer's rows into it with one launch of orl_frame_pool (rows grouped by frame
    through a CSR table built once per row-to-frame map; fixed summation order, no atomics);
  - `finish` stacks the observed layers' accumulators, all-reduces them in ONE collective (sums and counts together)
    so every rank holds identical features, and runs the whole selection for every layer in ONE launch of
    orl_frame_select (normalised means, farthest-point start, Lloyd steps until no centroid changes bit for bit, medoid
    per cluster with the lowest candidate on ties); the chosen frames come back to the host in one copy;
  - the bookkeeping of which frames each scene reads (step / layer switching) is plain Python on the host.
"""
from __future__ import annotations

import torch

from onereel_b200 import _lib as L
from onereel_b200 import dist as D
from onereel_b200.layout import SceneLayout

_DTYPES = {torch.bfloat16: 0, torch.float32: 1}


def _scene_reads(layout: SceneLayout, frames, halo: SceneLayout | None = None) -> dict:
    """scene j -> the sorted frames outside scene j among `frames` (and halo's halo frames of scene j)"""
    chosen = set(frames)
    out = {}
    for j, (lo, hi) in enumerate(layout.ranges):
        pool = chosen | set(halo.halo_frames(j)) if halo is not None else chosen
        out[j] = sorted(f for f in pool if f < lo or f >= hi)
    return out


class _RowGroups:
    """the rows of a row-to-frame map grouped by frame (CSR, device int32), built once per map tensor"""

    def __init__(self, frame: torch.Tensor, n_frames: int):
        self.frame = frame                                   # kept: the cache is keyed on this tensor's identity
        rows = torch.nonzero(frame >= 0).flatten()
        f = frame[rows].long()
        self.rows = rows[torch.argsort(f, stable=True)].to(torch.int32).contiguous()
        self.off = torch.zeros(n_frames + 1, dtype=torch.int32, device=frame.device)
        self.off[1:] = torch.cumsum(torch.bincount(f, minlength=n_frames), 0)


class FrameMemory:
    def __init__(self, budget: int = 4, candidates: str = 'all', layer: int | None = None, fallback=(2, 'adj'),
                 sink=(), per_layer: bool = False, iters: int = 20):
        if candidates not in ('all', 'boundary'):
            raise AssertionError(candidates)
        if len(sink) >= budget:
            raise AssertionError('the sink frames are part of the budget')
        self.budget, self.candidates, self.layer, self.fallback = budget, candidates, layer, fallback
        self.sink, self.per_layer, self.iters = tuple(sink), per_layer, iters
        self.layout = None
        self.step = -1
        self.pending = None          # representatives chosen during the current step, applied at the next
        self.history = []            # per step, the representatives it read
        self.extra = None            # scene -> extra frames (per_layer: layer -> that)
        self._acc = {}               # observed layer -> fp32 [n_frames, C + 4] device accumulator
        self._groups = None

    # ---------------------------------------------------------------------------------------------- bookkeeping

    def reset(self, layout: SceneLayout, n_layers: int):
        """frame_memory.py:34-44: a new request reads the fallback halo frames (and the sink) at step 0"""
        self.layout, self.n_layers = layout, n_layers
        self.step, self.pending, self.history, self._acc = -1, None, [], {}
        if self.layer is None:
            self.layer = n_layers // 2
        h, sides = self.fallback
        start = _scene_reads(layout, self.sink, SceneLayout(layout.lengths, halo=h, sides=sides))
        layout.extra = start
        self.extra = {l: start for l in range(n_layers)} if self.per_layer else start

    def _extra(self, reps, halo=None) -> dict:
        """scene -> the sink frames, representatives (and fallback halo frames) that lie outside the scene, sorted"""
        return _scene_reads(self.layout, set(self.sink) | set(reps), halo)

    def observes(self, layer: int) -> bool:
        return self.per_layer or layer == self.layer

    def begin_step(self, step: int):
        """frame_memory.py:57-69: the first forward of a new step applies the representatives chosen in the last"""
        if step == self.step:
            return
        self.step = step
        if self.pending is None:
            return
        chosen, self.pending = self.pending, None
        self.history.append(chosen)
        if self.per_layer:
            self.extra = {l: self._extra(r) for l, r in chosen.items()}
        else:
            self.extra = self._extra(chosen)
            self.layout.extra = self.extra

    def use_layer(self, layer: int):
        """frame_memory.py:71-74: per_layer — this layer's extra frames, before its block runs"""
        if self.per_layer and self.extra is not None:
            self.layout.extra = self.extra[layer]

    def candidate_frames(self) -> list[int]:
        """frame_memory.py:103-108: every frame, or the first and last frame of each scene; sink frames left out"""
        if self.candidates == 'all':
            frames = range(self.layout.n_frames)
        else:
            frames = sorted({f for lo, hi in self.layout.ranges for f in (lo, hi - 1)})
        return [f for f in frames if f not in self.sink]

    # ---------------------------------------------------------------------------------------------- device work

    def collect(self, frame: torch.Tensor, hs: torch.Tensor, layer: int | None = None):
        """frame_memory.py:76-85: frame [N] latent frame of each local row (-1: not video), hs [N, C] (CUDA); one
        orl_frame_pool launch adds the rows into the layer's per-frame sums and counts"""
        layer = self.layer if layer is None else layer
        if not (hs.is_cuda and frame.is_cuda):
            raise TypeError('FrameMemory.collect takes CUDA tensors (the B200 path has no CPU fallback)')
        n_frames, C = self.layout.n_frames, hs.shape[-1]
        if hs.dtype not in _DTYPES:
            hs = hs.float()
        if hs.stride(-1) != 1 or (hs.stride(0) * hs.element_size()) % 16 or hs.data_ptr() % 16 or C % 8:
            hs = hs.contiguous()
        if C % 8:
            raise ValueError(f'hidden size {C} must be a multiple of 8')
        if self._groups is None or self._groups.frame is not frame or len(self._groups.off) != n_frames + 1:
            self._groups = _RowGroups(frame, n_frames)
        g = self._groups
        acc = self._acc.get(layer)
        if acc is None:
            acc = self._acc[layer] = torch.zeros(n_frames, C + 4, dtype=torch.float32, device=hs.device)
        s = torch.cuda.current_stream(hs.device).cuda_stream
        L.check(L.lib().orl_frame_pool(hs.data_ptr(), _DTYPES[hs.dtype], hs.stride(0), C, g.rows.data_ptr(),
                                       g.off.data_ptr(), n_frames, acc.data_ptr(), acc.stride(0), s), 'orl_frame_pool')

    @torch.no_grad()
    def finish(self):
        """frame_memory.py:87-101: every observed layer's sums and counts all-reduced in one collective, then every
        layer's representatives chosen in one orl_frame_select launch"""
        if not self._acc:
            return
        layers = sorted(self._acc)
        feats = torch.stack([self._acc[l] for l in layers])
        self._acc = {}
        D.all_reduce(feats)
        chosen = self._select(feats, normalized=False)
        self.pending = dict(zip(layers, chosen)) if self.per_layer else chosen[0]

    def select(self, feats: torch.Tensor) -> list[int]:
        """frame_memory.py:110-132: representatives of L2-normalised per-frame features feats [n_frames, C] (CUDA)"""
        if not feats.is_cuda:
            raise TypeError('FrameMemory.select takes a CUDA tensor (the B200 path has no CPU fallback)')
        return self._select(feats.float().contiguous()[None], normalized=True)[0]

    def _select(self, feats: torch.Tensor, normalized: bool) -> list[list[int]]:
        """feats [sets, n_frames, ld] fp32 (in place when not normalized: rows are C sums then the count)"""
        cand = self.candidate_frames()
        k = min(self.budget - len(self.sink), len(cand))
        n_sets, C = feats.shape[0], feats.shape[2] - (0 if normalized else 4)
        if k <= 0:
            return [[] for _ in range(n_sets)]
        dev = feats.device
        cand_d = torch.tensor(cand, dtype=torch.int32, device=dev)
        per_set = L.check(L.lib().orl_frame_select_scratch(C, len(cand), k), 'orl_frame_select_scratch')
        scratch = torch.empty(n_sets, per_set, dtype=torch.float32, device=dev)
        reps = torch.empty(n_sets, k + 1, dtype=torch.int32, device=dev)
        s = torch.cuda.current_stream(dev).cuda_stream
        L.check(L.lib().orl_frame_select(feats.data_ptr(), feats.stride(1), feats.stride(0), n_sets, C,
                                         0 if normalized else 1, cand_d.data_ptr(), len(cand), k, self.iters,
                                         scratch.data_ptr(), per_set, reps.data_ptr(), s), 'orl_frame_select')
        return [r[1:1 + r[0]] for r in reps.cpu().tolist()]
