"""The CPU oracle against the golden vectors recorded from the reference (tests/golden/make_golden.py) and the
known answers of the reference's tests/test_onereel_layout.py and tests/test_onereel_frame_memory.py."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention_oracle as AO, layout_oracle as LO

G = Path(__file__).resolve().parent / 'golden'


def lay_of(c):
    return LO.Layout(c['lengths'], c['halo'], c['sides'], {int(j): v for j, v in c['extra'].items()})


def test_layout_golden():
    data = json.loads((G / 'layout.json').read_text())
    for c in data['cases']:
        lay = lay_of(c)
        for j in range(lay.n_scenes):
            assert lay.halo_frames(j) == c['halo_frames'][j]
            assert lay.shared_frames(j) == c['shared_frames'][j]
            assert lay.key_frames(j) == c['key_frames'][j]
            assert list(lay.key_range(j)) == c['key_range'][j]
    for e in data['even']:
        assert LO.even_lengths(e['n_frames'], e['n_scenes']) == e['lengths']


def test_planner_golden():
    data = json.loads((G / 'planner.json').read_text())
    for c in data['cases']:
        lay, T, n = lay_of(c), c['T'], c['n']
        assert LO.query_cost(lay, T, c['text'], c['extra_keys']) == c['query_cost']      # bit-exact float64
        own = LO.partition(lay, n, T, 'scene', c['text'], c['extra_keys'], c['granularity'])
        assert [list(o) for o in own] == c['own']
        assert [[list(x) for x in LO.needed(lay, T, o)] for o in own] == c['needed']
        assert LO.gather_rows(lay, own, T) == c['gather_rows']
        assert LO.choose_path(lay, own, T, c['theta']) == c['eq2']
        if 'ulysses_own' in c:
            assert [list(o) for o in LO.partition(lay, n, T, 'ulysses')] == c['ulysses_own']
        for mode, want in c.get('plan', {}).items():
            if 'error' in want:
                with pytest.raises(AssertionError):
                    LO.plan_parallel(lay, n, T, mode, want['heads'], c['text'] or [0] * lay.n_scenes, c['theta'],
                                     c['granularity'])
                continue
            run_mode, own2, path = LO.plan_parallel(lay, n, T, mode, want['heads'], c['text'] or [0] * lay.n_scenes,
                                                    c['theta'], c['granularity'])
            assert run_mode == want['run_mode'] and [list(o) for o in own2] == want['own'] and path == want['path']
    for b in data['balanced_small']:
        assert [list(x) for x in LO.balanced(b['sizes'], b['cost'], b['n'])] == b['own']


def test_reference_known_answers():
    """tests/test_onereel_layout.py:17-81 and tests/test_onereel_frame_memory.py:9-16 of the reference"""
    lay = LO.Layout([3, 5, 7], halo=2)
    assert lay.halo_frames(0) == [3, 4] and lay.halo_frames(1) == [1, 2, 8, 9]
    assert lay.key_frames(1) == [3, 4, 5, 6, 7, 1, 2, 8, 9] and lay.key_range(1) == (1, 10)
    assert LO.Layout([3, 5, 7], 2, 'next').halo_frames(1) == [8, 9]
    assert LO.Layout([3, 5, 7], 2, 'prev').halo_frames(1) == [1, 2]
    T = 1590
    lay = LO.Layout([8] * 6, halo=2)
    own = LO.partition(lay, 2, T, 'scene')
    assert own == [(0, 24 * T), (24 * T, 48 * T)]
    assert LO.needed(lay, T, own[0]) == [(24 * T, 26 * T)] and LO.needed(lay, T, own[1]) == [(22 * T, 24 * T)]
    lay = LO.Layout([3, 5, 7, 9, 11, 13], halo=2)
    own = LO.partition(lay, 2, T, 'scene')
    b = own[0][1]
    assert 24 * T < b < 35 * T and b % T != 0
    assert LO.needed(lay, T, own[0]) == [(b, 37 * T)] and LO.needed(lay, T, own[1]) == [(22 * T, b)]
    assert LO.balanced([1, 1], [1.0, 100.0], 2) == [(0, 1), (1, 2)]
    many = LO.Layout([4] * 12, halo=2)
    assert LO.choose_path(many, LO.partition(many, 4, T, 'scene'), T, 1.0)['path'] == 'scene'
    one = LO.Layout([40, 2, 2, 4], halo=2)
    c = LO.choose_path(one, LO.partition(one, 4, T, 'scene'), T, 1.0)
    assert c['path'] == 'ulysses' and c['V_G'] > c['V_U']
    assert LO.merge([(5, 7), (0, 2), (2, 3), (6, 9)]) == [(0, 3), (5, 9)]
    assert LO.clip([(0, 3), (5, 9)], 2, 6) == [(2, 3), (5, 6)]
    assert LO.frame_tokens([3, 4, 1, 2], 10) == [(30, 50), (10, 30)]
    assert LO.runs([3, 4, 5, 1, 2, 8, 9]) == [(3, 6), (1, 3), (8, 10)]
    lay = LO.Layout([3, 4, 5], halo=0, extra={0: [9, 1, 5], 1: [0], 2: [10]})
    assert lay.shared_frames(0) == [5, 9] and lay.key_frames(1) == [3, 4, 5, 6, 0] and lay.shared_frames(2) == []
    assert LO.needed(lay, 10, (0, 30)) == [(50, 60), (90, 100)]


def rle(rows):
    res = []
    for r in rows:
        kind, i = ('t', r[1]) if isinstance(r, tuple) else ('v', r)
        if res and res[-1][0] == kind and res[-1][2] == i:
            res[-1][2] = i + 1
        else:
            res.append([kind, i, i + 1])
    return res


def test_segments_golden():
    """the oracle's packed segment order equals the reference processor's, call by call"""
    for c in json.loads((G / 'segments.json').read_text()):
        if c['model'] != 'hunyuan':
            continue
        lay, T = lay_of(c), c['T']
        own = c['own'][c['r']]
        mine, text_for = LO.scene_pieces(lay, T, own)
        near = [s for s in mine if LO.is_local(lay, T, own, s[0])]
        far = [s for s in mine if not LO.is_local(lay, T, own, s[0])]
        groups = [g for g in (near, far) if g]
        assert len(groups) == len(c['calls'])
        for g, call in zip(groups, c['calls']):
            segs = LO.hunyuan_segments(lay, T, c['counts'], g, text_for & {j for j, _ in g})
            assert [rle(s[2]) for s in segs] == call['q']
            assert [rle(s[3]) for s in segs] == call['k'] == call['v']
            assert LO.cu_seqlens([len(s[2]) for s in segs]).tolist() == call['cu_q']
            assert LO.cu_seqlens([len(s[3]) for s in segs]).tolist() == call['cu_k']


def cfg1_inputs():
    g = torch.Generator().manual_seed(0)
    T, H, Dh, counts = 64, 4, 64, [16, 16, 16]
    L = 12 * T
    q, k, v = (torch.randn(L, H, Dh, generator=g) for _ in range(3))
    eq, ek, ev = (torch.randn(sum(counts), H, Dh, generator=g) for _ in range(3))
    lay = LO.Layout([4, 3, 5], halo=0, extra={0: [4], 1: [0], 2: [0, 4]})
    return lay, T, counts, [x.numpy() for x in (q, k, v, eq, ek, ev)]


def test_cfg1_attention_golden():
    """the oracle's scene attention equals the reference processor run on the CPU (fp32 SDPA in place of FA)"""
    lay, T, counts, (q, k, v, eq, ek, ev) = cfg1_inputs()
    gold = np.load(G / 'cfg1.npz')
    ov, ot, valid = AO.hunyuan_scene(lay, T, counts, q, k, v, eq, ek, ev)
    assert valid.all()
    assert np.abs(ov[::4] - gold['ov']).max() < 2e-5 and np.abs(ot - gold['ot']).max() < 2e-5
    segs = LO.hunyuan_segments(lay, T, counts, LO.scene_pieces(lay, T, (0, 12 * T))[0], {0, 1, 2})
    assert LO.cu_seqlens([len(s[2]) for s in segs]).tolist() == gold['cu_q'].tolist() == [0, 256, 272, 464, 480, 800, 816]
    assert LO.cu_seqlens([len(s[3]) for s in segs]).tolist() == gold['cu_k'].tolist() == [0, 336, 608, 880, 1088, 1552, 1888]
    # BASELINE cfg1's own check: dense SDPA with the scene block mask
    dv, dt = AO.masked_dense(lay, T, counts, q, k, v, eq, ek, ev)
    assert np.abs(dv - ov).max() < 1e-9 and np.abs(dt - ot).max() < 1e-9


def test_lse_merge_is_exact_split():
    rng = np.random.default_rng(0)
    q, k, v = rng.standard_normal((5, 2, 8)), rng.standard_normal((13, 2, 8)), rng.standard_normal((13, 2, 8))
    o, l = AO.attend(q, k, v)
    o1, l1 = AO.attend(q, k[:6], v[:6])
    o2, l2 = AO.attend(q, k[6:], v[6:])
    om, lm = AO.lse_merge(o1, l1, o2, l2)
    assert np.abs(om - o).max() < 1e-12 and np.abs(lm - l).max() < 1e-12
