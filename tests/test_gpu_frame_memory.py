"""Frame memory on the B200 kernels (orl_frame_pool, orl_frame_select) against the reference's recorded selections
(tests/golden/frame_memory.json), the CPU oracle, torch's index_add_ pooling and the known answers of the reference's
tests/test_onereel_frame_memory.py."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import frame_memory_oracle as FO

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / 'golden'


@pytest.fixture(scope='module', autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip('needs a B200')
    from onereel_b200.csrc.build import build
    build()


def test_cycle_matches_reference_golden():
    """reset -> collect (pooling kernel) -> finish (all-reduce + selection kernel) -> begin_step, per golden case;
    picks equal to the reference's except medoids its fp32 rounding chose between tied members"""
    from onereel_b200.frame_memory import FrameMemory
    from onereel_b200.layout import SceneLayout
    ties = 0
    for c in json.loads((G / 'frame_memory.json').read_text()):
        lay = SceneLayout(c['lengths'], halo=0)
        g = torch.Generator().manual_seed(c['seed'])
        frame = torch.arange(lay.n_frames).repeat_interleave(c['rows_per_frame'])
        hs = torch.randn(len(frame), c['C'], generator=g)
        fm = FrameMemory(budget=c['budget'], candidates=c['candidates'], sink=tuple(c['sink']), fallback=(1, 'adj'))
        fm.reset(lay, n_layers=4)
        assert {str(k): v for k, v in lay.extra.items()} == c['first']
        fm.begin_step(0)
        fm.collect(frame.cuda(), hs.cuda())
        fm.finish()
        fm.begin_step(1)
        got = fm.history[-1]
        x = FO.features(*FO.pool(frame.numpy(), hs.numpy(), lay.n_frames))
        cand = FO.candidate_frames(c['lengths'], c['candidates'], c['sink'])
        want, clusters = FO.select(x, cand, c['budget'] - len(c['sink']), detail=True)
        assert got == want, (c['seed'], got, want)                 # the kernel follows the oracle's rule exactly
        if got != c['reps']:
            assert FO.tie_explains(got, c['reps'], clusters), (c['seed'], got, c['reps'])
            ties += 1
        else:
            assert {str(k): v for k, v in lay.extra.items()} == c['extra']
    assert ties <= 3


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
def test_pool_kernel_matches_index_add(dtype):
    """permuted rows (the ring's row order), rows of no frame, a frame without rows; two collects accumulate"""
    from onereel_b200.frame_memory import FrameMemory
    from onereel_b200.layout import SceneLayout
    lay = SceneLayout([3, 4, 2], halo=0)
    F, C, T = lay.n_frames, 200, 37
    g = torch.Generator().manual_seed(5)
    frame = torch.arange(F).repeat_interleave(T)
    frame[frame == 4] = -1                                        # frame 4: no rows
    frame = frame[torch.randperm(len(frame), generator=g)]
    hs = torch.randn(len(frame), C, generator=g).to(dtype)
    fm = FrameMemory(budget=3)
    fm.reset(lay, 2)
    fm.collect(frame.cuda(), hs.cuda())
    fm.collect(frame.cuda(), hs.cuda())
    acc = fm._acc[fm.layer]
    keep = frame >= 0
    want = torch.zeros(F, C, dtype=torch.float64).index_add_(0, frame[keep], hs[keep].double()) * 2
    cnt = torch.bincount(frame[keep], minlength=F).double() * 2
    got = acc[:, :C].double().cpu()
    assert torch.allclose(got, want, rtol=1e-5, atol=1e-4)
    assert torch.equal(acc[:, C].double().cpu(), cnt)


def test_select_known_answers_and_layers_in_one_launch():
    """tests/test_onereel_frame_memory.py:20-83 of the reference on the kernels, and per_layer: every layer's picks from
    one selection launch equal each layer selected alone"""
    from onereel_b200.frame_memory import FrameMemory
    from onereel_b200.layout import SceneLayout
    lay = SceneLayout([3, 3, 3], halo=0)
    fm = FrameMemory(budget=2, fallback=(1, 'adj'))
    fm.reset(lay, n_layers=8)
    fm.begin_step(0)
    g = torch.Generator().manual_seed(0)
    base = torch.randn(2, 16, generator=g)
    feats = torch.cat([base[0].expand(5, -1), base[1].expand(4, -1)]) + 0.01 * torch.randn(9, 16, generator=g)
    frame = torch.arange(9).repeat_interleave(4)
    fm.collect(frame.cuda(), feats.repeat_interleave(4, 0).cuda())
    fm.finish()
    assert lay.extra == {0: [3], 1: [2, 6], 2: [5]}
    fm.begin_step(1)
    reps = fm.history[-1]
    assert len(reps) == 2 and min(reps) < 5 <= max(reps)
    for j, (lo, hi) in enumerate(lay.ranges):
        assert lay.extra[j] == [f for f in reps if not lo <= f < hi]
    lay = SceneLayout([4, 4, 4], halo=0)
    x = torch.nn.functional.normalize(torch.randn(12, 8, generator=torch.Generator().manual_seed(1)), dim=-1).cuda()
    a, b = FrameMemory(budget=3), FrameMemory(budget=3)
    a.reset(lay, 4)
    b.reset(lay, 4)
    assert a.select(x) == b.select(x) == FO.select(x.cpu().numpy().astype(np.float64), list(range(12)), 3)
    c = FrameMemory(budget=3, candidates='boundary')
    c.reset(lay, 4)
    assert c.candidate_frames() == [0, 3, 4, 7, 8, 11] and set(c.select(x)) <= {0, 3, 4, 7, 8, 11}
    # per_layer: 6 layers, one launch
    lay = SceneLayout([5, 6, 4, 5], halo=0)
    fm = FrameMemory(budget=4, per_layer=True, fallback=(0, 'adj'))
    fm.reset(lay, n_layers=6)
    fm.begin_step(0)
    frame = torch.arange(lay.n_frames).repeat_interleave(3).cuda()
    hss = [torch.randn(len(frame), 64, generator=torch.Generator().manual_seed(10 + l)).cuda() for l in range(6)]
    for l, hs in enumerate(hss):
        fm.collect(frame, hs, l)
    fm.finish()
    fm.begin_step(1)
    batched = fm.history[-1]
    for l, hs in enumerate(hss):
        x = FO.features(*FO.pool(frame.cpu().numpy(), hs.cpu().numpy(), lay.n_frames))
        assert batched[l] == FO.select(x, list(range(lay.n_frames)), 4), l
