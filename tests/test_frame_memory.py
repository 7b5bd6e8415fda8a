"""Frame memory on the CPU: the oracle's selection against the reference's recorded selections
(tests/golden/frame_memory.json) and the known answers of the reference's tests/test_onereel_frame_memory.py, and the
product's host bookkeeping (which frames each scene reads, step and layer switching). The product's device kernels are
checked against the same fixtures in tests/test_gpu_frame_memory.py."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from onereel_b200.frame_memory import FrameMemory
from onereel_b200.layout import SceneLayout
from oracle import frame_memory_oracle as FO

G = Path(__file__).resolve().parent / 'golden'


def golden_cases():
    return json.loads((G / 'frame_memory.json').read_text())


def case_inputs(c):
    F = sum(c['lengths'])
    g = torch.Generator().manual_seed(c['seed'])
    frame = torch.arange(F).repeat_interleave(c['rows_per_frame'])
    hs = torch.randn(len(frame), c['C'], generator=g)
    return frame, hs


def test_oracle_selection_matches_reference_golden():
    """equal to the reference's picks, except medoids the reference's fp32 rounding chose between tied members"""
    ties = 0
    for c in golden_cases():
        frame, hs = case_inputs(c)
        x = FO.features(*FO.pool(frame.numpy(), hs.numpy(), sum(c['lengths'])))
        cand = FO.candidate_frames(c['lengths'], c['candidates'], c['sink'])
        reps, clusters = FO.select(x, cand, c['budget'] - len(c['sink']), detail=True)
        if reps != c['reps']:
            assert FO.tie_explains(reps, c['reps'], clusters), (c['seed'], reps, c['reps'])
            ties += 1
        assert {str(k): v for k, v in FO.scene_reads(c['lengths'], set(c['sink']) | set(c['reps'])).items()} == \
            c['extra']
    assert ties <= 3


def test_oracle_known_answers():
    """tests/test_onereel_frame_memory.py:20-83 of the reference, on the oracle"""
    g = torch.Generator().manual_seed(0)
    base = torch.randn(2, 16, generator=g)
    feats = torch.cat([base[0].expand(5, -1), base[1].expand(4, -1)]) + 0.01 * torch.randn(9, 16, generator=g)
    frame = torch.arange(9).repeat_interleave(4)
    x = FO.features(*FO.pool(frame.numpy(), feats.repeat_interleave(4, 0).numpy(), 9))
    reps = FO.select(x, FO.candidate_frames([3, 3, 3], 'all', ()), 2)
    assert len(reps) == 2 and min(reps) < 5 <= max(reps)
    f = torch.nn.functional.normalize(torch.randn(12, 8, generator=torch.Generator().manual_seed(1)), dim=-1).numpy()
    assert FO.candidate_frames([4, 4, 4], 'boundary', ()) == [0, 3, 4, 7, 8, 11]
    assert set(FO.select(f, [0, 3, 4, 7, 8, 11], 3)) <= {0, 3, 4, 7, 8, 11}
    f2 = torch.nn.functional.normalize(torch.randn(9, 8, generator=torch.Generator().manual_seed(3)), dim=-1).numpy()
    r2 = FO.select(f2, FO.candidate_frames([3, 3, 3], 'all', (0,)), 2)
    assert len(r2) == 2 and 0 not in r2


def test_bookkeeping_matches_reference_golden():
    """reset (fallback halo + sink) and the extra frames after a step, with the step's picks handed over as finish
    would: the product's host logic against the reference's recorded layouts"""
    for c in golden_cases():
        lay = SceneLayout(c['lengths'], halo=0)
        fm = FrameMemory(budget=c['budget'], candidates=c['candidates'], sink=tuple(c['sink']), fallback=(1, 'adj'))
        fm.reset(lay, n_layers=4)
        assert {str(k): v for k, v in lay.extra.items()} == c['first']
        assert fm.candidate_frames() == FO.candidate_frames(c['lengths'], c['candidates'], c['sink'])
        fm.begin_step(0)
        fm.pending = list(c['reps'])
        fm.begin_step(0)                      # same step: nothing applied
        assert {str(k): v for k, v in lay.extra.items()} == c['first']
        fm.begin_step(1)
        assert fm.history[-1] == c['reps']
        assert {str(k): v for k, v in lay.extra.items()} == c['extra']


def test_reference_known_answers_host_side():
    """the host-side asserts of tests/test_onereel_frame_memory.py:20-83: observed layer, fallback / sink layouts"""
    lay = SceneLayout([3, 3, 3], halo=0)
    fm = FrameMemory(budget=2, fallback=(1, 'adj'))
    fm.reset(lay, n_layers=8)
    assert fm.layer == 4 and lay.extra == {0: [3], 1: [2, 6], 2: [5]}
    assert fm.observes(4) and not fm.observes(3)
    lay = SceneLayout([3, 3, 3], halo=0)
    fm = FrameMemory(budget=3, fallback=(0, 'adj'), sink=(0,))
    fm.reset(lay, n_layers=4)
    assert lay.extra == {0: [], 1: [0], 2: [0]} and 0 not in fm.candidate_frames()
    with pytest.raises(AssertionError):
        FrameMemory(budget=1, sink=(0,))
    with pytest.raises(AssertionError):
        FrameMemory(candidates='middle')


def test_per_layer_switches_extra():
    lay = SceneLayout([3, 3, 3], halo=0)
    fm = FrameMemory(budget=1, fallback=(0, 'adj'), per_layer=True)
    fm.reset(lay, n_layers=2)
    assert fm.observes(0) and fm.observes(1)
    fm.begin_step(0)
    fm.pending = {0: [1], 1: [7]}
    fm.begin_step(1)
    fm.use_layer(0)
    assert lay.extra == {0: [], 1: [1], 2: [1]}
    fm.use_layer(1)
    assert lay.extra == {0: [7], 1: [7], 2: []}


def test_collect_refuses_cpu_tensors():
    lay = SceneLayout([2, 2], halo=0)
    fm = FrameMemory(budget=2)
    fm.reset(lay, 2)
    with pytest.raises(TypeError):
        fm.collect(torch.arange(4), torch.zeros(4, 8))
    with pytest.raises(TypeError):
        fm.select(torch.zeros(4, 8))


def test_oracle_pool_skips_unassigned_rows():
    frame = np.array([0, 1, -1, 1, 0])
    hs = np.arange(10, dtype=np.float32).reshape(5, 2)
    s, n = FO.pool(frame, hs, 3)
    assert n.tolist() == [2, 2, 0] and s[0].tolist() == [8, 10] and s[1].tolist() == [8, 10] and s[2].tolist() == [0, 0]
