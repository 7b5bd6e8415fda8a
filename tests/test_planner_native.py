"""The native planner (csrc/planner.cpp via onereel_b200.comm) and the processors' compiled segment plans against the
reference's golden vectors and the CPU oracle — no GPU needed."""
import json
import random
from pathlib import Path

import pytest

from oracle import layout_oracle as LO

G = Path(__file__).resolve().parent / 'golden'


@pytest.fixture(scope='module', autouse=True)
def _built():
    from onereel_b200.csrc.build import build
    build()


def lay_of(c):
    from onereel_b200.layout import SceneLayout
    return SceneLayout(c['lengths'], c['halo'], c['sides'], {int(j): v for j, v in c['extra'].items()})


def test_planner_matches_golden_bit_exact():
    from onereel_b200 import comm
    data = json.loads((G / 'planner.json').read_text())
    for c in data['cases']:
        lay, T, n = lay_of(c), c['T'], c['n']
        assert comm.query_cost(lay, T, c['text'], c['extra_keys']) == c['query_cost']
        own = comm.partition(lay, n, T, 'scene', c['text'], c['extra_keys'], c['granularity'])
        assert [list(o) for o in own] == c['own'], c
        assert [[list(x) for x in comm.needed(lay, T, o)] for o in own] == c['needed']
        assert comm.gather_rows(lay, own, T) == c['gather_rows']
        assert comm.choose_path(lay, own, T, c['theta']) == c['eq2']
        if 'ulysses_own' in c:
            assert [list(o) for o in comm.partition(lay, n, T, 'ulysses')] == c['ulysses_own']
    for b in data['balanced_small']:
        assert [list(x) for x in comm.balanced(b['sizes'], b['cost'], b['n'])] == b['own']


def test_plan_parallel_matches_golden():
    """hunyuan15._plan_parallel decisions (run_mode, own, path) for n ranks, recorded from the reference"""
    from onereel_b200 import dist as D, hunyuan15 as HY
    data = json.loads((G / 'planner.json').read_text())
    saved = D.world
    try:
        for c in data['cases']:
            for mode, want in c.get('plan', {}).items():
                lay = lay_of(c)
                ctx = HY.Context(lay, mode=mode, partition=c['granularity'], theta=c['theta'], T=c['T'],
                                 counts={True: c['text'] or [0] * lay.n_scenes})
                D.world = lambda n=c['n']: n
                if 'error' in want:
                    with pytest.raises(AssertionError):
                        HY.plan_parallel(ctx, want['heads'])
                    continue
                HY.plan_parallel(ctx, want['heads'])
                assert ctx.run_mode == want['run_mode'] and [list(o) for o in ctx.own] == want['own']
                assert ctx.path == want['path']
    finally:
        D.world = saved


def test_planner_random_against_oracle():
    from onereel_b200 import comm
    from onereel_b200.layout import SceneLayout
    rng = random.Random(7)
    for _ in range(300):
        n_s = rng.randint(1, 12)
        lengths = [rng.randint(1, 20) for _ in range(n_s)]
        F = sum(lengths)
        extra = {j: rng.sample(range(F), rng.randint(0, 3)) for j in range(n_s)} if rng.random() < 0.5 else {}
        halo, sides = rng.choice([0, 1, 2, 4]), rng.choice(['adj', 'prev', 'next'])
        T = rng.choice([1, 7, 880, 1590, 3600])
        n = rng.choice([2, 3, 4, 5, 8])
        text = [rng.randint(0, 512) for _ in range(n_s)] if rng.random() < 0.5 else None
        if F * T < n:
            continue
        lay, olay = SceneLayout(lengths, halo, sides, extra), LO.Layout(lengths, halo, sides, extra)
        own = comm.partition(lay, n, T, 'scene', text)
        assert own == LO.partition(olay, n, T, 'scene', text)
        for o in own:
            assert comm.needed(lay, T, o) == LO.needed(olay, T, o)
        assert comm.choose_path(lay, own, T, 1.0) == LO.choose_path(olay, own, T, 1.0)


def _decode(plan, remote_index, a):
    """a compiled ScenePlan's K/V run table -> per segment the token rows it packs (video t, text ('t', i))"""
    from onereel_b200 import scene as S
    res = []
    for s in plan.segs:
        rows = []
        for src, lo, hi in s.kv:
            if src == S.VIDEO:
                rows += list(range(a + lo, a + hi))
            elif src == S.TEXT:
                rows += [('t', i) for i in range(lo, hi)]
            else:
                for r in range(lo, hi):
                    x, y, off = next(t for t in remote_index if t[2] <= r < t[2] + t[1] - t[0])
                    rows.append(x + r - off)
        res.append(rows)
    return res


def _rle(rows):
    out = []
    for r in rows:
        kind, i = ('t', r[1]) if isinstance(r, tuple) else ('v', r)
        if out and out[-1][0] == kind and out[-1][2] == i:
            out[-1][2] = i + 1
        else:
            out.append([kind, i, i + 1])
    return out


def test_rank_plans_match_reference_calls():
    """for every rank of n in {1, 2, 3}: the processor's near / far plans reproduce the reference processor's packed
    calls (segment order, query rows, key rows including received ones, cu_seqlens)"""
    from onereel_b200 import comm, dist as D, hunyuan15 as HY
    saved = D.world, D.rank
    checked = 0
    try:
        for c in json.loads((G / 'segments.json').read_text()):
            if c['model'] != 'hunyuan':
                continue
            lay = lay_of(c)
            n, r = c['n'], c['r']
            D.world, D.rank = (lambda: n), (lambda: r)
            ctx = HY.Context(lay, T=c['T'], own=[tuple(o) for o in c['own']], counts={True: c['counts']}, fwd=1)
            plan = HY._RankPlan(ctx, 2, 64, 'cpu', False)
            groups = [p for p in (plan.near, plan.far) if p is not None]
            assert len(groups) == len(c['calls'])
            a = ctx.own[r][0]
            for p, call in zip(groups, c['calls']):
                assert [[['v' if s.kind == 'v' else 't', s.q[1] + (a if s.kind == 'v' else 0),
                          s.q[2] + (a if s.kind == 'v' else 0)]] for s in p.segs] == call['q']
                assert [_rle(rows) for rows in _decode(p, plan.remote_index, a)] == call['k']
                assert p.cu_q == call['cu_q'] and p.cu_k == call['cu_k']
            checked += 1
    finally:
        D.world, D.rank = saved
    assert checked > 100


def test_ring_plan_matches_reference():
    """onereel_b200.ring.RingPlan against the reference's RingPlan (chunks, permutation, rows, volume, key sets)"""
    from onereel_b200.ring import RingPlan
    for c in json.loads((G / 'ring.json').read_text()):
        plan = RingPlan(lay_of(c), c['n'], c['T'], device='cpu')
        assert [[list(x) for x in ch] for ch in plan.chunks] == c['chunks']
        assert plan.perm.tolist() == c['perm'] and plan.inv.tolist() == c['inv']
        assert [list(o) for o in plan.own] == c['own'] and [[list(x) for x in l] for l in plan.local] == c['local']
        assert plan.volume() == c['volume']
        for src in range(c['n']):
            got = {str(j): (None if x is None else x.tolist()) for j, x in plan.keys(src, 'tag').items()}
            assert got == c['keys'][str(src)]


def test_exchange_plan_covers_every_read_once():
    """the K/V exchange's operation lists (broadcast of rows every other rank reads, point to point for the rest) on
    random layouts for 2..8 ranks: every rank receives exactly the tokens it reads outside its range, each once, and
    both sides of every point-to-point pair list the same intervals"""
    import random
    from onereel_b200 import comm
    from onereel_b200.layout import SceneLayout
    rng = random.Random(3)
    for case in range(120):
        lengths = [rng.randint(1, 9) for _ in range(rng.randint(1, 9))]
        lay = SceneLayout(lengths, halo=rng.choice([0, 1, 2]), sides=rng.choice(['adj', 'prev', 'next']))
        F = lay.n_frames
        if rng.random() < 0.7:
            shared = rng.sample(range(F), min(F, rng.randint(1, 3)))        # frame-memory-like: read by every scene
            lay.extra = {j: sorted(shared) for j in range(lay.n_scenes)}
        T = rng.choice([2, 4, 7])
        n = rng.randint(2, 8)
        if F * T < 2 * n:
            continue
        own = comm.partition(lay, n, T, 'scene', [rng.randint(0, 4) for _ in lengths])
        extra = sorted({f for v in lay.extra.values() for f in v}) if rng.random() < 0.3 else ()
        need, common, p2p = comm.exchange_plan(lay, own, T, extra)
        for r in range(n):
            got = []
            for p in range(n):
                if p != r:
                    got += [iv for iv in common[p]] + p2p[(p, r)]
            toks = sorted(t for lo, hi in got for t in range(lo, hi))
            want = sorted(t for lo, hi in need[r] for t in range(lo, hi))
            assert toks == want, (case, lengths, n, r)
            for p in range(n):                       # what p broadcasts lies in its own range
                assert all(own[p][0] <= lo and hi <= own[p][1] for lo, hi in common[p])
        if n == 2:
            assert all(not c for c in common)
