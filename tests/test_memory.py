"""Bounded cross-scene memory, host side (CPU): candidate frames and BoundaryMemory.select against the reference's own
outputs (tests/golden/memory.json, src/onereel/memory.py:31-105), the compiled pieces against the reference's
frame_plan (memory.py:118-140 as hunyuan15.Processor.memory builds it, 305-333), and the selection properties the
reference's tests/test_onereel_memory.py checks (every candidate kept when the budget covers them; each
representative is the member nearest its centroid)."""
import json
from pathlib import Path

import torch

from onereel_b200 import comm
from onereel_b200 import memory as MEM
from onereel_b200 import scene as S
from onereel_b200.layout import SceneLayout

G = Path(__file__).resolve().parent / 'golden'


def test_candidates_and_selection_match_reference():
    cases = json.loads((G / 'memory.json').read_text())['select']
    for c in cases:
        lay = SceneLayout(c['lengths'], halo=0)
        assert MEM.candidate_frames(lay) == (c['frames'], c['owner'])
        B = len(c['frames']) * c['T']
        g = torch.Generator().manual_seed(c['seed'])
        kc = torch.randn(B, c['H'], c['D'], generator=g)
        kc2 = kc + 0.3 * torch.randn(B, c['H'], c['D'], generator=g)
        mem = MEM.BoundaryMemory(c['M'])
        rep, valid = mem.select('k', kc)
        assert rep.tolist() == c['rep'] and valid.tolist() == c['valid'], c
        rep, valid = mem.select('k', kc2)                      # warm-started from the first call's centroids
        assert rep.tolist() == c['rep2'] and valid.tolist() == c['valid2'], c


def _decode(plan, seg, own, remote_index):
    """a compiled segment's key sources -> video tokens (t >= 0) and text rows (-(i + 1)), in key order"""
    out = []
    for src, lo, hi in seg.kv:
        for row in range(lo, hi):
            if src == S.VIDEO:
                out.append(own[0] + row)
            elif src == S.TEXT:
                out.append(-(row + 1))
            else:
                x, y, r = next(t for t in remote_index if t[2] <= row < t[2] + t[1] - t[0])
                out.append(x + row - r)
    return out


def test_pieces_match_reference_frame_plan():
    cases = json.loads((G / 'memory.json').read_text())['plans']
    for c in cases:
        lay = SceneLayout(c['lengths'], halo=0)
        T, counts, n = c['T'], c['counts'], c['n']
        own_all = [tuple(r['own']) for r in c['ranks']]
        cand = MEM.candidate_frames(lay)[0]
        for r, rk in enumerate(c['ranks']):
            own = own_all[r]
            if n == 1:
                remote_index = []
                scenes = [(j, (lo * T, hi * T)) for j, (lo, hi) in enumerate(lay.ranges)]
                text_for = set(range(lay.n_scenes))
            else:
                remote_index = S.remote_index_of(lay, T, own_all, r, lambda l, t, o: comm.needed(l, t, o, cand))
                scenes, text_for = S.pieces(lay, T, own)
            plan = MEM.MemoryPlan.for_rank(lay, T, counts, own, remote_index, scenes, text_for, 'cpu')
            plan.compile(2, 64, 8)
            mine, Sq = {}, own[1] - own[0]
            for seg in plan.segs:
                if seg.lq == 0:                 # the reference drops pieces without queries (memory.py:121)
                    continue
                off = 0 if seg.kind == 'v' else Sq                 # text queries follow the video rows
                mine[(seg.kind == 'v', seg.scene)] = ([off + seg.q[1], off + seg.q[2]],
                                                      _decode(plan, seg, own, remote_index))
            ref = {(p['mem'], p['scene']): (p['q'], p['keys']) for p in rk['pieces']}
            assert mine == ref, (c['lengths'], r)
            # candidates: every boundary frame's tokens, frame by frame
            assert rk['cand'] == [f * T + t for f in cand for t in range(T)]
            # the packed layout: each video segment's local keys, then min(M, B) representative slots
            for i, seg in enumerate(plan.segs):
                nxt = plan.base[i] + plan.n_local[i] + (plan.M if seg.kind == 'v' else 0)
                assert nxt == (plan.base[i + 1] if i + 1 < len(plan.segs) else plan.spare)


def test_all_candidates_kept_when_budget_covers_them():
    """tests/test_onereel_memory.py:57-66 of the reference"""
    torch.manual_seed(1)
    lay = SceneLayout([3, 4, 2], halo=0)
    T, H, Dh = 8, 2, 32
    rows, owner = MEM.candidates(lay, T, 'cpu')
    k = torch.randn(lay.n_frames * T, H, Dh)
    rep, valid = MEM.BoundaryMemory(len(rows)).select('x', k[rows])
    for h in range(H):
        assert sorted(rep[h][valid[h]].tolist()) == list(range(len(rows)))


def test_representative_is_nearest_member():
    """tests/test_onereel_memory.py:69-83 of the reference"""
    torch.manual_seed(2)
    x = torch.randn(300, 3, 16)
    mem = MEM.BoundaryMemory(12)
    rep, valid = mem.select('y', x)
    c = mem.centroids['y']
    xn = torch.nn.functional.normalize(x.float().transpose(0, 1), dim=-1)
    for h in range(3):
        z = torch.cdist(xn[h], c[h]).argmin(-1)
        for r in rep[h][valid[h]].tolist():
            members = (z == z[r]).nonzero().flatten()
            d = (xn[h, members] - c[h, z[r]]).pow(2).sum(-1)
            assert d.min() >= (xn[h, r] - c[h, z[r]]).pow(2).sum() - 1e-6


def test_frame_plan_matches_reference_at_world_1():
    """the reference-style frame_plan (memory.py:126-140) on one rank: same pieces, keys and candidates"""
    cases = [c for c in json.loads((G / 'memory.json').read_text())['plans'] if c['n'] == 1]
    assert cases
    for c in cases:
        lay = SceneLayout(c['lengths'], halo=0)
        T, counts = c['T'], c['counts']
        L_ = lay.n_frames * T
        tr = S.text_ranges(counts)
        plan = MEM.frame_plan(lay, T, torch.arange(L_), L_, [(j, lo * T, hi * T) for j, (lo, hi) in
                                                           enumerate(lay.ranges)], tr, set(range(lay.n_scenes)), L_,
                              'cpu')
        mine = {}
        for seg in plan.segs:
            keys = [row if row < L_ else -(row - L_ + 1) for _, lo, hi in seg.kv for row in range(lo, hi)]
            mine[(seg.kind == 'v', seg.scene)] = ([seg.q[1], seg.q[2]], keys)
        ref = {(p['mem'], p['scene']): (p['q'], p['keys']) for p in c['ranks'][0]['pieces']}
        assert mine == ref, c['lengths']
        assert plan.cand_local_rows.tolist() == c['ranks'][0]['cand']
