"""Bounded cross-scene memory on the B200 kernels (hunyuan15.Processor.memory at world 1) against a per-head fp32
reference — the reference's tests/test_onereel_memory.py:20-54: every scene's video queries read their frames, their
sentence and the valid representatives of other scenes; sentence queries read the scene's frames and the sentence.
Two calls in a row: the second selection is warm-started from the first one's centroids (B200 only)."""
import pytest
import torch

from onereel_b200 import memory as MEM

pytestmark = pytest.mark.gpu


def _reference(q, k, v, eq, ek, ev, lay, T, rep_row, rep_scene, valid, text_ranges):
    S, H, Dh = q.shape
    ov, ot = torch.zeros(S, H, Dh, device=q.device), torch.zeros(ek.shape[0], H, Dh, device=q.device)
    kk, vv = torch.cat([k, ek]).float(), torch.cat([v, ev]).float()
    for h in range(H):
        for j, (lo, hi) in enumerate(lay.ranges):
            t0, t1 = text_ranges[j]
            fr = [r for r, s, ok in zip(rep_row[h].tolist(), rep_scene[h].tolist(), valid[h].tolist()) if ok and s != j]
            keys = list(range(lo * T, hi * T)) + [S + t for t in range(t0, t1)] + fr
            a = torch.softmax(q[lo * T:hi * T, h].float() @ kk[keys, h].T / Dh ** 0.5, -1)
            ov[lo * T:hi * T, h] = a @ vv[keys, h]
            tkeys = list(range(lo * T, hi * T)) + [S + t for t in range(t0, t1)]
            if t1 > t0:
                a = torch.softmax(eq[t0:t1, h].float() @ kk[tkeys, h].T / Dh ** 0.5, -1)
                ot[t0:t1, h] = a @ vv[tkeys, h]
    return ov, ot


@pytest.mark.parametrize('lengths,M,counts', [([3, 5, 2, 4], 8, [5, 7, 3, 6]), ([2, 2, 2], 1000, [5, 0, 3]),
                                              ([6, 1, 3], 5, [4, 4, 4]), ([7], 3, [2])])
def test_memory_attention_matches_reference(lengths, M, counts):
    if not torch.cuda.is_available():
        pytest.skip('needs a B200')
    from onereel_b200 import attention as A, hunyuan15 as HY
    from onereel_b200.layout import SceneLayout
    torch.manual_seed(0)
    T, H, Dh = 16, 4, 64
    lay = SceneLayout(lengths, halo=0)
    S = lay.n_frames * T
    tr = HY.S.text_ranges(counts)
    ctx = HY.Context(lay, T=T, counts={True: counts}, fwd=1, own=[(0, S)], memory=M)
    proc = HY.Processor(ctx, 0)
    rows, owner = MEM.candidates(lay, T, 'cuda')
    shadow = MEM.BoundaryMemory(M)                  # the same (deterministic) selections as the processor's memory
    rel = lambda a, b: ((a.float() - b).norm() / b.norm()).item()
    for call in range(2):
        q, k, v = (torch.randn(S, H, Dh, device='cuda', dtype=torch.bfloat16) for _ in range(3))
        eq, ek, ev = (torch.randn(sum(counts), H, Dh, device='cuda', dtype=torch.bfloat16) for _ in range(3))
        ov, ot = proc.memory(q, k, v, eq, ek, ev)
        torch.cuda.synchronize()
        A.check()
        rep, valid = shadow.select((0, True), k[rows])
        ref_v, ref_t = _reference(q, k, v, eq, ek, ev, lay, T, rows[rep], owner[rep], valid, tr)
        assert rel(ov, ref_v) < 2e-2, (call, rel(ov, ref_v))
        assert rel(ot, ref_t) < 2e-2, (call, rel(ot, ref_t))


def test_wan_memory_matches_reference():
    """Wan self-attention with the bounded memory (no joint text): scene frames plus foreign representatives"""
    if not torch.cuda.is_available():
        pytest.skip('needs a B200')
    from onereel_b200 import attention as A, wan as WN
    from onereel_b200.layout import SceneLayout
    torch.manual_seed(3)
    T, H, Dh, M = 16, 4, 128, 6
    lay = SceneLayout([4, 3, 5], halo=0)
    S = lay.n_frames * T
    ctx = WN.Context(lay, T=T, own=[(0, S)], memory=M, fwd=1)
    q, k, v = (torch.randn(S, H, Dh, device='cuda', dtype=torch.bfloat16) for _ in range(3))
    o = WN.Processor(ctx, 'self', None, 0).memory(q, k, v)
    torch.cuda.synchronize()
    A.check()
    rows, owner = MEM.candidates(lay, T, 'cuda')
    rep, valid = MEM.BoundaryMemory(M).select((0, True), k[rows])
    empty = torch.zeros(0, H, Dh, device='cuda', dtype=torch.bfloat16)
    ref, _ = _reference(q, k, v, empty, empty, empty, lay, T, rows[rep], owner[rep], valid, [(0, 0)] * lay.n_scenes)
    rel = ((o.float() - ref).norm() / ref.norm()).item()
    assert rel < 2e-2, rel


def test_reference_style_frame_plan_call():
    """the reference's own call shape (tests/test_onereel_memory.py:11-17): frame_plan over concatenated video+text
    buffers, MemoryAttention(BoundaryMemory(M))(key, q, k, v, plan) -> [Sq + text, H, D]"""
    if not torch.cuda.is_available():
        pytest.skip('needs a B200')
    from onereel_b200 import attention as A
    from onereel_b200.layout import SceneLayout
    torch.manual_seed(4)
    lengths, M, counts = [3, 5, 2, 4], 8, [5, 7, 3, 6]
    T, H, Dh = 16, 4, 64
    lay = SceneLayout(lengths, halo=0)
    S = lay.n_frames * T
    tr, c = [], 0
    for m in counts:
        tr.append((c, c + m))
        c += m
    q, k, v = (torch.randn(S, H, Dh, device='cuda', dtype=torch.bfloat16) for _ in range(3))
    eq, ek, ev = (torch.randn(c, H, Dh, device='cuda', dtype=torch.bfloat16) for _ in range(3))
    plan = MEM.frame_plan(lay, T, torch.arange(S), S, [(j, lo * T, hi * T) for j, (lo, hi) in enumerate(lay.ranges)],
                          tr, set(range(lay.n_scenes)), S, 'cuda')
    out = MEM.MemoryAttention(MEM.BoundaryMemory(M))(('l0', True), torch.cat([q, eq]), torch.cat([k, ek]),
                                                    torch.cat([v, ev]), plan)
    torch.cuda.synchronize()
    A.check()
    rows, owner = MEM.candidates(lay, T, 'cuda')
    rep, valid = MEM.BoundaryMemory(M).select(('l0', True), k[rows])
    ref_v, ref_t = _reference(q, k, v, eq, ek, ev, lay, T, rows[rep], owner[rep], valid, tr)
    rel = lambda a, b: ((a.float() - b).norm() / b.norm()).item()
    assert rel(out[:S], ref_v) < 2e-2 and rel(out[S:], ref_t) < 2e-2
