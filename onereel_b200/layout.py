"""Scene layout over the latent frames of one video — the reference's `onereel.layout.SceneLayout`, same API.

src/onereel/layout.py:10-78: `lengths` latent frames per scene; a scene also reads `halo` frames of its neighbours on
`sides` ('adj' | 'prev' | 'next') and the frames in extra[j] (frame memory, replaced every denoising step). The key
order of scene j is its own frames, then its shared frames (halo: previous scene's last frames, then the next scene's
first; then its sorted extra frames not already listed and not its own) — the packed K/V order of every segment.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch


@dataclass
class SceneLayout:
    lengths: list[int]
    halo: int = 2
    sides: str = 'adj'
    extra: dict = field(default_factory=dict)

    def __post_init__(self):
        assert self.sides in ('adj', 'prev', 'next'), self.sides
        assert all(n > 0 for n in self.lengths), self.lengths

    @classmethod
    def even(cls, n_frames: int, n_scenes: int, **kw) -> 'SceneLayout':
        """scene of frame f = f * n_scenes // n_frames (layout.py:24-28)"""
        sc = np.arange(n_frames) * n_scenes // n_frames
        return cls(np.bincount(sc, minlength=n_scenes).astype(int).tolist(), **kw)

    @property
    def n_frames(self) -> int:
        return sum(self.lengths)

    @property
    def n_scenes(self) -> int:
        return len(self.lengths)

    @property
    def is_even(self) -> bool:
        return self.lengths == SceneLayout.even(self.n_frames, self.n_scenes).lengths

    @property
    def ranges(self) -> list[tuple[int, int]]:
        s = np.cumsum([0] + list(self.lengths))
        return [(int(s[j]), int(s[j + 1])) for j in range(self.n_scenes)]

    @property
    def frames(self) -> list[list[int]]:
        return [list(range(lo, hi)) for lo, hi in self.ranges]

    def scene_of_frame(self) -> torch.Tensor:
        return torch.repeat_interleave(torch.arange(self.n_scenes), torch.tensor(self.lengths))

    def halo_frames(self, j: int) -> list[int]:
        if self.halo == 0:
            return []
        lo, hi = self.ranges[j]
        before = []
        if j > 0 and self.sides in ('adj', 'prev'):
            plo, phi = self.ranges[j - 1]
            before = list(range(max(plo, phi - self.halo), phi))
        after = []
        if j + 1 < self.n_scenes and self.sides in ('adj', 'next'):
            nlo, nhi = self.ranges[j + 1]
            after = list(range(nlo, min(nhi, nlo + self.halo)))
        return before + after

    def shared_frames(self, j: int) -> list[int]:
        lo, hi = self.ranges[j]
        out = self.halo_frames(j)
        seen = set(out)
        for f in sorted(self.extra.get(j, ())):
            if not lo <= f < hi and f not in seen:
                out.append(f)
                seen.add(f)
        return out

    def key_frames(self, j: int) -> list[int]:
        return self.frames[j] + self.shared_frames(j)

    def key_range(self, j: int) -> tuple[int, int]:
        kf = self.key_frames(j)
        return min(kf), max(kf) + 1
