"""onereel_b200.frame_memory.FrameMemory against the reference's selections (tests/golden/frame_memory.json) and the
known answers of the reference's tests/test_onereel_frame_memory.py — CPU."""
import json
from pathlib import Path

import torch

from onereel_b200.frame_memory import FrameMemory
from onereel_b200.layout import SceneLayout

G = Path(__file__).resolve().parent / 'golden'


def test_selection_matches_reference_golden():
    for c in json.loads((G / 'frame_memory.json').read_text()):
        lay = SceneLayout(c['lengths'], halo=0)
        g = torch.Generator().manual_seed(c['seed'])
        frame = torch.arange(lay.n_frames).repeat_interleave(c['rows_per_frame'])
        hs = torch.randn(len(frame), c['C'], generator=g)
        fm = FrameMemory(budget=c['budget'], candidates=c['candidates'], sink=tuple(c['sink']), fallback=(1, 'adj'))
        fm.reset(lay, n_layers=4)
        assert {str(k): v for k, v in lay.extra.items()} == c['first']
        fm.begin_step(0)
        fm.collect(frame, hs)
        fm.finish()
        fm.begin_step(1)
        assert fm.history[-1] == c['reps']
        assert {str(k): v for k, v in lay.extra.items()} == c['extra']


def test_reference_known_answers():
    """tests/test_onereel_frame_memory.py:20-83 of the reference"""
    lay = SceneLayout([3, 3, 3], halo=0)
    fm = FrameMemory(budget=2, fallback=(1, 'adj'))
    fm.reset(lay, n_layers=8)
    assert fm.layer == 4 and lay.extra == {0: [3], 1: [2, 6], 2: [5]}
    fm.begin_step(0)
    g = torch.Generator().manual_seed(0)
    base = torch.randn(2, 16, generator=g)
    feats = torch.cat([base[0].expand(5, -1), base[1].expand(4, -1)]) + 0.01 * torch.randn(9, 16, generator=g)
    frame = torch.arange(9).repeat_interleave(4)
    fm.collect(frame, feats.repeat_interleave(4, 0))
    fm.finish()
    assert lay.extra == {0: [3], 1: [2, 6], 2: [5]}
    fm.begin_step(1)
    reps = fm.history[-1]
    assert len(reps) == 2 and min(reps) < 5 <= max(reps)
    for j, (lo, hi) in enumerate(lay.ranges):
        assert lay.extra[j] == [f for f in reps if not lo <= f < hi]
    lay = SceneLayout([4, 4, 4], halo=0)
    feats = torch.nn.functional.normalize(torch.randn(12, 8, generator=torch.Generator().manual_seed(1)), dim=-1)
    a, b = FrameMemory(budget=3), FrameMemory(budget=3)
    a.reset(lay, 4)
    b.reset(lay, 4)
    assert a.select(feats) == b.select(feats)
    c = FrameMemory(budget=3, candidates='boundary')
    c.reset(lay, 4)
    assert c.candidate_frames() == [0, 3, 4, 7, 8, 11] and set(c.select(feats)) <= {0, 3, 4, 7, 8, 11}
    lay = SceneLayout([3, 3, 3], halo=0)
    fm = FrameMemory(budget=3, fallback=(0, 'adj'), sink=(0,))
    fm.reset(lay, n_layers=4)
    assert lay.extra == {0: [], 1: [0], 2: [0]} and 0 not in fm.candidate_frames()
    f2 = torch.nn.functional.normalize(torch.randn(9, 8, generator=torch.Generator().manual_seed(3)), dim=-1)
    r2 = fm.select(f2)
    assert len(r2) == 2 and 0 not in r2


def test_per_layer_switches_extra():
    lay = SceneLayout([3, 3, 3], halo=0)
    fm = FrameMemory(budget=1, fallback=(0, 'adj'), per_layer=True)
    fm.reset(lay, n_layers=2)
    assert fm.observes(0) and fm.observes(1)
    fm.begin_step(0)
    frame = torch.arange(9)
    a = torch.eye(9)[[0, 0, 0, 0, 0, 0, 0, 0, 8]] + 0.01 * torch.arange(9)[:, None]
    fm.collect(frame, torch.eye(9), 0)
    fm.collect(frame, a, 1)
    fm.finish()
    fm.begin_step(1)
    r0, r1 = fm.history[-1][0], fm.history[-1][1]
    fm.use_layer(0)
    e0 = dict(lay.extra)
    fm.use_layer(1)
    e1 = dict(lay.extra)
    assert len(r0) == len(r1) == 1
    assert e0 == {j: [f for f in r0 if not lo <= f < hi] for j, (lo, hi) in enumerate(lay.ranges)}
    assert e1 == {j: [f for f in r1 if not lo <= f < hi] for j, (lo, hi) in enumerate(lay.ranges)}
