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
