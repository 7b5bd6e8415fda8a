"""Generate the golden fixtures of tests/golden/ by running the OneReel reference's own Python code on the CPU.

Run where the reference is checked out (next to this repository by default, or ONEREEL_REF=<repo root>):
    python tests/golden/make_golden.py
Writes layout.json, planner.json, segments.json and cfg1.npz next to this file. The fixtures pin both the CPU oracle
(oracle/) and the product's native planner / pack plan; the GPU box never needs the reference.

What is recorded (reference file:line in brackets):
  layout.json    SceneLayout halo/shared/key frames and key ranges (src/onereel/layout.py:54-78), even() splits (24-28)
  planner.json   partition / needed / gather_rows / eq2 / _plan_parallel (src/onereel/parallel/comm.py:18-112,
                 src/onereel/models/hunyuan15.py:553-573) on seeded random layouts, n in {2, 3, 4, 8}
  segments.json  the packed segment order of hunyuan15.Processor.scene (212-251, _segments 153-170) per rank, and of
                 wan.Processor.ranges/scene (110-152): per packed call, each segment's query and key source rows and
                 the call's cu_seqlens (attention.py:28-29, 65-71). Rows are recorded by running the processor on index
                 tensors (video token t -> t, text row i -> -(i + 1)); the collectives are replaced by row lookups.
  frame_memory.json  FrameMemory selections and extra frames (src/onereel/frame_memory.py:24-132) on seeded features
  ring.json      RingPlan chunks / permutation / per-rank rows / key sets (src/onereel/parallel/ring.py:23-60)
  memory.json    bounded memory (src/onereel/memory.py): candidate frames (31-38), BoundaryMemory.select (58-105) on
                 seeded candidate keys — a first selection and a warm-started one — and the pieces of frame_plan
                 (118-140) as built by hunyuan15.Processor.memory (305-333) at world 1 and per rank of gathering
                 partitions (query rows and local key tokens of each piece)
  cfg1.npz       BASELINE cfg1 run through hunyuan15.Processor.scene at world 1 in fp32 on the CPU, with the FA varlen
                 call replaced by per-segment fp32 softmax attention: inputs are regenerated from seed 0 by the tests,
                 outputs stored as float32 (every 4th video row, every text row).
"""
from __future__ import annotations

import json
import os
import random
import sys
from pathlib import Path

import numpy as np
import torch

REF = Path(os.environ.get('ONEREEL_REF', Path(__file__).resolve().parents[3] / 'reference'))
sys.path.insert(0, str(REF / 'src'))
HERE = Path(__file__).resolve().parent

from onereel import attention as A                          # noqa: E402
from onereel.layout import SceneLayout                        # noqa: E402
from onereel.models import hunyuan15 as HY, wan as WN         # noqa: E402
from onereel.parallel import comm, dist as D                  # noqa: E402
from onereel.parallel import ring as RG                       # noqa: E402
from onereel.frame_memory import FrameMemory                  # noqa: E402
from onereel import memory as MEMR                            # noqa: E402


def rand_layout(rng, max_scenes=8, max_len=12):
    n = rng.randint(1, max_scenes)
    lengths = [rng.randint(1, max_len) for _ in range(n)]
    halo = rng.choice([0, 0, 1, 2, 3])
    sides = rng.choice(['adj', 'prev', 'next'])
    F = sum(lengths)
    extra = {}
    if rng.random() < 0.6:
        for j in range(n):
            extra[j] = sorted(rng.sample(range(F), min(F, rng.randint(0, 4))))
    return dict(lengths=lengths, halo=halo, sides=sides, extra=extra)


def make(case):
    lay = SceneLayout(case['lengths'], halo=case['halo'], sides=case['sides'])
    lay.extra = {int(j): list(v) for j, v in case['extra'].items()}
    return lay


def gen_layout(rng):
    cases = []
    for _ in range(300):
        c = rand_layout(rng)
        lay = make(c)
        c['halo_frames'] = [lay.halo_frames(j) for j in range(lay.n_scenes)]
        c['shared_frames'] = [lay.shared_frames(j) for j in range(lay.n_scenes)]
        c['key_frames'] = [lay.key_frames(j) for j in range(lay.n_scenes)]
        c['key_range'] = [list(lay.key_range(j)) for j in range(lay.n_scenes)]
        cases.append(c)
    even = [dict(n_frames=F, n_scenes=S, lengths=SceneLayout.even(F, S).lengths)
            for F in (7, 20, 21, 31, 84, 124) for S in (1, 2, 3, 4, 5, 7) if S <= F]
    return dict(cases=cases, even=even)


class _World:
    """D.world / D.rank stand-ins so the reference planner runs for n ranks without a process group"""

    def __init__(self, n, r=0):
        self.n, self.r = n, r

    def __enter__(self):
        self.saved = D.world, D.rank
        D.world, D.rank = (lambda: self.n), (lambda: self.r)

    def __exit__(self, *a):
        D.world, D.rank = self.saved


def gen_planner(rng):
    cases = []
    for i in range(400):
        c = rand_layout(rng, max_scenes=10, max_len=14)
        lay = make(c)
        T = rng.choice([1, 3, 16, 64, 880, 1590])
        n = rng.choice([2, 3, 4, 8])
        if lay.n_frames * T < n:
            continue
        text = [rng.randint(0, 300) for _ in lay.lengths] if rng.random() < 0.6 else None
        extra_keys = rng.choice([0, 0, 4, 128])
        gran = rng.choice(['balanced', 'balanced', 'tokens', 'scenes'])
        theta = rng.choice([0.5, 1.0, 2.0])
        if gran == 'scenes' and lay.n_scenes < n:
            gran = 'balanced'
        c.update(T=T, n=n, text=text, extra_keys=extra_keys, granularity=gran, theta=theta)
        own = comm.partition(lay, n, T, 'scene', text, extra_keys, gran)
        c['query_cost'] = comm.query_cost(lay, T, text, extra_keys)
        c['own'] = [list(o) for o in own]
        c['needed'] = [[list(x) for x in comm.needed(lay, T, o)] for o in own]
        c['gather_rows'] = comm.gather_rows(lay, own, T)
        c['eq2'] = comm.choose_path(lay, own, T, theta)
        if lay.n_frames * T % n == 0:
            c['ulysses_own'] = [list(o) for o in comm.partition(lay, n, T, 'ulysses')]
        heads = rng.choice([16, 24, 6])
        for mode in ('scene', 'auto', 'ulysses'):
            ctx = HY.Context(lay, mode=mode, partition=gran, theta=theta, T=T, counts={True: text or [0] * lay.n_scenes})
            with _World(n):
                try:
                    HY._plan_parallel(ctx, heads)
                    c.setdefault('plan', {})[mode] = dict(heads=heads, run_mode=ctx.run_mode,
                                                          own=[list(o) for o in ctx.own], path=ctx.path)
                except AssertionError:
                    c.setdefault('plan', {})[mode] = dict(heads=heads, error='AssertionError')
        cases.append(c)
    # the exact-answer tests of the reference (tests/test_onereel_layout.py) restated as data
    extra_cases = []
    for lengths, n, T in (([8] * 6, 2, 1590), ([3, 5, 7, 9, 11, 13], 2, 1590), ([3, 5, 7, 9, 11, 13, 2, 6], 3, 1590),
                          ([3, 5, 7, 9, 11, 13, 2, 6], 8, 1590), ([4] * 12, 4, 1590), ([40, 2, 2, 4], 4, 1590)):
        lay = SceneLayout(lengths, halo=2)
        own = comm.partition(lay, n, T, 'scene')
        extra_cases.append(dict(lengths=lengths, halo=2, sides='adj', extra={}, T=T, n=n, text=None, extra_keys=0,
                                granularity='balanced', theta=1.0, own=[list(o) for o in own],
                                needed=[[list(x) for x in comm.needed(lay, T, o)] for o in own],
                                gather_rows=comm.gather_rows(lay, own, T), eq2=comm.choose_path(lay, own, T, 1.0),
                                query_cost=comm.query_cost(lay, T)))
    return dict(cases=cases + extra_cases, balanced_small=[dict(sizes=[1, 1], cost=[1.0, 100.0], n=2,
                                                               own=[list(x) for x in comm.balanced([1, 1], [1.0, 100.0], 2)])])


def _row_tensor(vals):
    return torch.tensor(vals, dtype=torch.float64)[:, None, None]


def _decode(t):
    """index tensor -> run-length rows [[kind, lo, hi], ...]: kind 'v' video tokens lo..hi-1, 't' text rows"""
    res = []
    for x in t[:, 0, 0].tolist():
        kind, i = ('v', int(x)) if x >= 0 else ('t', int(-x - 1))
        if res and res[-1][0] == kind and res[-1][2] == i:
            res[-1][2] = i + 1
        else:
            res.append([kind, i, i + 1])
    return res


def gen_segments(rng):
    """segment order per packed call of the reference processors, on index tensors"""
    out = []
    layouts = [dict(lengths=[4, 3, 5], halo=0, sides='adj', extra={0: [4], 1: [0], 2: [0, 4]}, T=64, counts=[16] * 3),
               dict(lengths=[8, 6, 10, 7], halo=0, sides='adj', extra={0: [8, 14, 24], 1: [0, 14, 24], 2: [0, 8, 24],
                                                                       3: [0, 8, 14]}, T=10, counts=[5] * 4)]
    for _ in range(40):
        c = rand_layout(rng, max_scenes=7, max_len=8)
        c['T'] = rng.choice([2, 5, 16])
        c['counts'] = [rng.randint(1, 9) for _ in c['lengths']]
        layouts.append(c)
    calls = []

    def rec_packed(segs):
        calls.append(dict(q=[_decode(s[0]) for s in segs], k=[_decode(s[1]) for s in segs],
                          v=[_decode(s[2]) for s in segs],
                          cu_q=A.cu_seqlens([s[0].shape[0] for s in segs], 'cpu').tolist(),
                          cu_k=A.cu_seqlens([s[1].shape[0] for s in segs], 'cpu').tolist()))
        return [s[0].clone() for s in segs]

    class FakeExchange:
        """HaloExchange without a process group: rows(i)(frames) = the rows of the frame list, from the full tensor"""
        full = None

        def __init__(self, layout, own, T, k, v, extra=(), heads=None):
            self.T = T

        def wait(self):
            pass

        def rows(self, i, side=None):
            full, T = FakeExchange.full[i], self.T
            return lambda fl: torch.cat([full[lo:hi] for lo, hi in comm.frame_tokens(fl, T)])

    saved = A.packed, comm.HaloExchange, comm.send_text_rows, D.all_reduce
    A.packed, comm.HaloExchange = rec_packed, FakeExchange
    comm.send_text_rows = lambda *a, **k: None
    D.all_reduce = lambda x: None
    try:
        for c in layouts:
            lay = make(c)
            T, counts = c['T'], c['counts']
            L = lay.n_frames * T
            full = _row_tensor(list(range(L)))
            text = _row_tensor([-(i + 1) for i in range(sum(counts))])
            FakeExchange.full = (full, full)
            for n in (1, 2, 3):
                if L < n:
                    continue
                own = comm.partition(lay, n, T, 'scene', counts)
                for r in range(n):
                    a, b = own[r]
                    calls.clear()
                    with _World(n, r):
                        ctx = HY.Context(lay, T=T, own=own, counts={True: counts}, fwd=1)
                        HY.Processor(ctx, 0).scene(full[a:b], full[a:b], full[a:b], text, text, text)
                    out.append(dict(model='hunyuan', lengths=c['lengths'], halo=c['halo'], sides=c['sides'],
                                    extra={str(j): v for j, v in c['extra'].items()}, T=T, counts=counts, n=n, r=r,
                                    own=[list(o) for o in own], calls=list(calls)))
            # Wan at world 1: contiguous ranges (overlapping_ranges) or the packed path when extra frames are read
            ranges_calls = []
            A.overlapping_ranges = lambda q, k, v, qr, kr: (ranges_calls.append(dict(q_ranges=[list(x) for x in qr],
                                                                                       k_ranges=[list(x) for x in kr])), q)[1]
            calls.clear()
            wc = WN.Context(lay, T=T, own=[(0, L)])
            try:
                WN.Processor.ranges(type('P', (), {'ctx': wc})(), full, full, full)
                out.append(dict(model='wan', lengths=c['lengths'], halo=c['halo'], sides=c['sides'],
                                extra={str(j): v for j, v in c['extra'].items()}, T=T, n=1, r=0,
                                calls=list(calls), ranges=ranges_calls))
            except AssertionError:
                out.append(dict(model='wan', lengths=c['lengths'], halo=c['halo'], sides=c['sides'],
                                extra={str(j): v for j, v in c['extra'].items()}, T=T, n=1, r=0,
                                error='AssertionError'))
    finally:
        A.packed, comm.HaloExchange, comm.send_text_rows, D.all_reduce = saved
    return out


def sdpa_varlen(q, k, v, cu_q, cu_k, max_q, max_k):
    """the FA varlen call replaced by per-segment fp32 softmax attention on the CPU"""
    outs = []
    for i in range(len(cu_q) - 1):
        a, b, c, d = (int(x) for x in (cu_q[i], cu_q[i + 1], cu_k[i], cu_k[i + 1]))
        qq, kk, vv = (x.transpose(0, 1)[None] for x in (q[a:b], k[c:d], v[c:d]))
        outs.append(torch.nn.functional.scaled_dot_product_attention(qq, kk, vv)[0].transpose(0, 1))
    return torch.cat(outs)


def gen_cfg1():
    """BASELINE cfg1: lengths [4,3,5], T = 64, 16 text tokens per scene, frame memory = first latent frame of scenes 0
    and 1 (frames {0, 4}), H = 4, D = 64, q/k/v ~ N(0, 1) from seed 0 drawn in the order q, k, v, eq, ek, ev"""
    lay = SceneLayout([4, 3, 5], halo=0)
    mem = [0, 4]
    lay.extra = {j: [f for f in mem if not lo <= f < hi] for j, (lo, hi) in enumerate(lay.ranges)}
    T, H, Dh, counts = 64, 4, 64, [16, 16, 16]
    g = torch.Generator().manual_seed(0)
    L, Nt = lay.n_frames * T, sum(counts)
    q, k, v = (torch.randn(L, H, Dh, generator=g) for _ in range(3))
    eq, ek, ev = (torch.randn(Nt, H, Dh, generator=g) for _ in range(3))
    rec = {}
    saved_varlen, saved_cu = A.varlen, A.cu_seqlens

    def varlen(q_, k_, v_, cu_q, cu_k, max_q, max_k):
        rec.update(cu_q=cu_q.tolist(), cu_k=cu_k.tolist(), max_q=max_q, max_k=max_k)
        return sdpa_varlen(q_, k_, v_, cu_q, cu_k, max_q, max_k)
    A.varlen = varlen
    A.cu_seqlens = lambda lengths, device='cpu': saved_cu(lengths, 'cpu')
    try:
        ctx = HY.Context(lay, T=T, own=[(0, L)], counts={True: counts}, fwd=1)
        ov, ot = HY.Processor(ctx, 0).scene(q, k, v, eq, ek, ev)
    finally:
        A.varlen, A.cu_seqlens = saved_varlen, saved_cu
    np.savez_compressed(HERE / 'cfg1.npz', ov=ov.numpy()[::4].astype(np.float32), ot=ot.numpy().astype(np.float32),
                        cu_q=np.array(rec['cu_q'], np.int32), cu_k=np.array(rec['cu_k'], np.int32),
                        max_q=rec['max_q'], max_k=rec['max_k'], extra=json.dumps({str(j): v for j, v in lay.extra.items()}))
    return rec


def gen_ring(rng):
    """RingPlan (src/onereel/parallel/ring.py:23-60) on seeded layouts: chunks, perm, own, local, volume, keys"""
    out = []
    for _ in range(40):
        c = rand_layout(rng, max_scenes=6, max_len=6)
        lay = make(c)
        T = rng.choice([3, 7, 16])
        n = rng.choice([1, 2, 3, 4])
        plan = RG.RingPlan(lay, n, T, device='cpu')
        keys = {str(src): {str(j): (None if x is None else x.tolist()) for j, x in plan.keys(src, 'tag').items()}
                for src in range(n)}
        out.append(dict(c, T=T, n=n, chunks=plan.chunks, perm=plan.perm.tolist(), inv=plan.inv.tolist(),
                        own=[list(o) for o in plan.own], local=plan.local, volume=plan.volume(), keys=keys))
    return out


def gen_frame_memory(rng):
    """FrameMemory (src/onereel/frame_memory.py:24-132): selections on seeded per-frame features (CPU fp32), and the
    extra frames a full reset / collect / finish / begin_step cycle produces"""
    out = []
    for i in range(30):
        c = rand_layout(rng, max_scenes=6, max_len=10)
        lay = make(c)
        budget = rng.randint(2, 6)
        cands = rng.choice(['all', 'boundary'])
        sink = tuple(sorted(rng.sample(range(lay.n_frames), min(rng.randint(0, 1), lay.n_frames))))
        if len(sink) >= budget:
            sink = ()
        C = rng.choice([8, 32])
        g = torch.Generator().manual_seed(100 + i)
        rows_per_frame = rng.randint(1, 4)
        frame = torch.arange(lay.n_frames).repeat_interleave(rows_per_frame)
        hs = torch.randn(len(frame), C, generator=g)
        fm = FrameMemory(budget=budget, candidates=cands, sink=sink, fallback=(1, 'adj'))
        lay.extra = {}
        fm.reset(lay, n_layers=4)
        first = dict(lay.extra)
        fm.begin_step(0)
        fm.collect(frame, hs)
        fm.finish()
        fm.begin_step(1)
        out.append(dict(lengths=c['lengths'], budget=budget, candidates=cands, sink=list(sink), C=C, seed=100 + i,
                        rows_per_frame=rows_per_frame, first={str(k): v for k, v in first.items()},
                        reps=fm.history[-1], extra={str(k): v for k, v in lay.extra.items()}))
    return out


def gen_memory(rng):
    """bounded memory: candidate_frames, select (init + warm-started update), frame_plan pieces"""
    sel = []
    for i in range(24):
        lengths = [rng.randint(1, 6) for _ in range(rng.randint(1, 5))]
        lay = SceneLayout(lengths, halo=0)
        T, H, Dh = rng.choice([2, 4, 8]), rng.choice([1, 3]), rng.choice([8, 16, 32])
        M = rng.choice([1, 3, 7, 12, 1000])
        frames, owner = MEMR.candidate_frames(lay)
        B = len(frames) * T
        g = torch.Generator().manual_seed(500 + i)
        kc = torch.randn(B, H, Dh, generator=g)
        kc2 = kc + 0.3 * torch.randn(B, H, Dh, generator=g)
        mem = MEMR.BoundaryMemory(M)
        rep, valid = mem.select('k', kc)
        rep2, valid2 = mem.select('k', kc2)
        sel.append(dict(lengths=lengths, T=T, H=H, D=Dh, M=M, seed=500 + i, frames=frames, owner=owner,
                        rep=rep.tolist(), valid=valid.tolist(), rep2=rep2.tolist(), valid2=valid2.tolist()))
    plans = []
    for i in range(16):
        lengths = [rng.randint(1, 7) for _ in range(rng.randint(1, 6))]
        lay = SceneLayout(lengths, halo=0)
        T = rng.choice([2, 3, 4])
        counts = [rng.randint(0, 5) for _ in lengths]
        n = rng.choice([1, 2, 3, 4])
        L_ = lay.n_frames * T
        if L_ < 2 * n:
            n = 1
        own = comm.partition(lay, n, T, 'scene', counts, 8) if n > 1 else [(0, L_)]
        tr, c = [], 0
        for m in counts:
            tr.append((c, c + m))
            c += m
        ranks = []
        for r, (a, b) in enumerate(own):
            cand = MEMR.candidate_frames(lay)[0]
            if n == 1:
                token_row = torch.arange(L_)
                pieces = [(j, lo * T, hi * T) for j, (lo, hi) in enumerate(lay.ranges)]
                text_for = set(range(lay.n_scenes))
                Lv = L_
            else:
                need = comm.needed(lay, T, (a, b), cand)
                held = [(a, b)] + [(lo, hi) for lo, hi in need]
                token_row = torch.full((L_,), -1, dtype=torch.long)
                row = 0
                for lo, hi in held:
                    token_row[lo:hi] = torch.arange(row, row + hi - lo)
                    row += hi - lo
                Lv = row
                pieces = [(j, lo - a, hi - a) for j, (lo, hi) in
                          [(j, (max(lo * T, a), min(hi * T, b))) for j, (lo, hi) in enumerate(lay.ranges)
                           if lo * T < b and hi * T > a]]
                text_for = {j for j, (lo, _) in enumerate(lay.ranges) if a <= lo * T < b}
            Sq = (b - a) if n > 1 else L_
            plan = MEMR.frame_plan(lay, T, token_row, Lv, pieces, tr, text_for, Sq, 'cpu')
            inv = {int(rw): t for t, rw in enumerate(token_row.tolist()) if rw >= 0}
            dec = lambda rw: inv[rw] if rw < Lv else -(rw - Lv + 1)
            qoff = 0
            out_pieces = []
            for pi in range(len(plan.qlen)):
                ql = int(plan.qlen[pi])
                qr = plan.qrows[qoff:qoff + ql].tolist()
                qoff += ql
                keys = [dec(int(x)) for x in plan.pad[pi, :int(plan.lens[pi])].tolist()]
                out_pieces.append(dict(scene=int(plan.scene[pi]), q=[qr[0], qr[-1] + 1], keys=keys,
                                       mem=bool(plan.mem[pi])))
            ranks.append(dict(own=[a, b], pieces=out_pieces, cand=[dec(int(x)) for x in plan.cand.tolist()]))
        plans.append(dict(lengths=lengths, T=T, counts=counts, n=n, ranks=ranks))
    return dict(select=sel, plans=plans)


def main():
    (HERE / 'ring.json').write_text(json.dumps(gen_ring(random.Random(7))))
    (HERE / 'frame_memory.json').write_text(json.dumps(gen_frame_memory(random.Random(11))))
    (HERE / 'memory.json').write_text(json.dumps(gen_memory(random.Random(13))))
    rng = random.Random(20261201)
    torch.set_num_threads(os.cpu_count())
    (HERE / 'layout.json').write_text(json.dumps(gen_layout(rng)))
    (HERE / 'planner.json').write_text(json.dumps(gen_planner(rng)))
    (HERE / 'segments.json').write_text(json.dumps(gen_segments(rng)))
    rec = gen_cfg1()
    print('cfg1 cu_q', rec['cu_q'], 'cu_k', rec['cu_k'])
    for f in sorted(HERE.iterdir()):
        print(f.name, f.stat().st_size)


if __name__ == '__main__':
    main()
