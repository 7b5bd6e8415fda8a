"""The gather/pack kernel (orl_pack) and the LSE merge kernels (orl_lse_merge, orl_lse_merge_acc) on the GPU: the
pack bit-exact against a byte gather for run tables with tiny, empty and tile-straddling runs, several planes and
more runs than a tile holds; the cu_seqlens it writes against the reference's recorded packed calls; the merges
against the CPU oracle's merge (B200 only)."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention_oracle as AO

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope='module', autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip('needs a B200')
    from onereel_b200.csrc.build import build
    build()


def gather_reference(srcs, runs, total_bytes):
    """the copy a run table describes, done with torch indexing on raw bytes"""
    out = torch.zeros(total_bytes, dtype=torch.uint8, device='cuda')
    for s_slot, s_off, d_off, nb in runs:
        out[d_off:d_off + nb] = srcs[s_slot][s_off:s_off + nb]
    return out


@pytest.mark.parametrize('n_planes', [1, 2, 3])
@pytest.mark.parametrize('kind', ['tiny', 'mixed', 'many'])
def test_pack_run_tables_bit_exact(n_planes, kind):
    from onereel_b200.pack import RunTable
    rng = np.random.default_rng(10 * n_planes + ['tiny', 'mixed', 'many'].index(kind))
    n_runs = {'tiny': 300, 'mixed': 60, 'many': 5000}[kind]
    if kind == 'tiny':                           # 0 to 3 vectors per run, many runs inside one 2048-vector tile
        nvec = rng.integers(0, 4, n_runs)
    elif kind == 'mixed':                        # empty runs, single vectors, runs longer than a tile
        nvec = rng.choice([0, 1, 7, 256, 2047, 2048, 2049, 9000], n_runs)
    else:                                        # more runs than fit any fixed staging
        nvec = rng.integers(1, 40, n_runs)
    nbytes = (nvec * 16).astype(np.int64)
    n_slots = 3
    src_size = [int(nbytes.sum()) + 4096] * n_slots
    srcs = [[torch.randint(0, 256, (sz,), dtype=torch.uint8, device='cuda') for sz in src_size]
            for _ in range(n_planes)]
    src_slot = rng.integers(0, n_slots, n_runs).astype(np.int32)
    src_off = np.array([16 * rng.integers(0, (src_size[0] - nb) // 16 + 1) for nb in nbytes], dtype=np.int64)
    order = rng.permutation(n_runs)              # destination order differs from the table's order
    dst_off = np.empty(n_runs, dtype=np.int64)
    dst_off[order] = np.concatenate([[0], np.cumsum(nbytes[order])[:-1]])
    total = int(nbytes.sum())
    t = RunTable(src_slot, np.full(n_runs, n_slots, np.int32), src_off, dst_off, nbytes, 'cuda')
    dsts = [torch.full((total + 16,), 7, dtype=torch.uint8, device='cuda') for _ in range(n_planes)]
    src_b, dst_b = [], []
    for p in range(n_planes):
        src_b += [x.data_ptr() for x in srcs[p]] + [0]
        dst_b += [0] * n_slots + [dsts[p].data_ptr()]
    t.run(src_b, dst_b, n_planes=n_planes)
    torch.cuda.synchronize()
    for p in range(n_planes):
        runs = list(zip(src_slot.tolist(), src_off.tolist(), dst_off.tolist(), nbytes.tolist()))
        want = gather_reference(srcs[p], runs, total)
        assert torch.equal(dsts[p][:total], want)
        assert torch.equal(dsts[p][total:], torch.full((16,), 7, dtype=torch.uint8, device='cuda'))


def test_pack_writes_cu_seqlens_of_the_reference():
    """ScenePlan.pack_kv's launch writes cu_seqlens_k on the device; it equals the reference's recorded cu_k for
    every one-rank Hunyuan layout of the golden set"""
    from onereel_b200 import scene as S
    from onereel_b200.layout import SceneLayout
    cases = json.loads((ROOT / 'tests' / 'golden' / 'segments.json').read_text())
    checked = 0
    H, Dh = 2, 64
    for c in cases:
        if c['model'] != 'hunyuan' or c['n'] != 1:
            continue
        lay = SceneLayout(c['lengths'], c['halo'], c['sides'], {int(j): v for j, v in c['extra'].items()})
        T, counts = c['T'], c['counts']
        L = lay.n_frames * T
        mine = [(j, (lo * T, hi * T)) for j, (lo, hi) in enumerate(lay.ranges)]
        segs = S.scene_segments(lay, T, counts, mine, set(range(lay.n_scenes)), (0, L))
        plan = S.ScenePlan(segs, H * Dh * 2, H, torch.device('cuda'))
        k = torch.randn(L, H, Dh, device='cuda').to(torch.bfloat16)
        ek = torch.randn(sum(counts), H, Dh, device='cuda').to(torch.bfloat16)
        plan.cu_k_dev.fill_(-1)
        kp, vp = plan.pack_kv(k, k, ek, ek)
        (call,) = c['calls']
        assert plan.cu_k_dev.tolist() == call['cu_k']
        checked += 1
        if checked >= 12:
            break
    assert checked >= 12


@pytest.mark.parametrize('Dh', [64, 128])
def test_lse_merge_kernels_match_oracle(Dh):
    from onereel_b200 import attention as A
    g = torch.Generator().manual_seed(Dh)
    n, H = 333, 3
    o1 = torch.randn(n, H, Dh, generator=g).to(torch.bfloat16)
    o2 = torch.randn(n, H, Dh, generator=g).to(torch.bfloat16)
    l1 = torch.randn(H, n, generator=g) * 4
    l2 = torch.randn(H, n, generator=g) * 4
    l2[0, :5] = -float('inf')                      # a partial without keys
    l1[1, 7:9] = -float('inf')
    l1[2, 11], l2[2, 11] = -float('inf'), -float('inf')
    want_o, want_l = AO.lse_merge(o1.float().numpy(), l1.numpy(), o2.float().numpy(), l2.numpy())
    d = lambda x: x.to('cuda')
    g1, gl1 = d(o1).contiguous(), d(l1).contiguous()
    A.lse_merge(g1, gl1, d(o2).contiguous(), d(l2).contiguous())
    acc, lacc = d(o1).float().contiguous(), d(l1).contiguous()
    A.lse_merge_acc(acc, lacc, d(o2).contiguous(), d(l2).contiguous())
    torch.cuda.synchronize()
    # a row where neither part has keys merges to zeros with lse -inf (as a segment without keys)
    assert torch.equal(g1[11, 2].float().cpu(), torch.zeros(Dh)) and gl1[2, 11].item() == -float('inf')
    fin = ~np.isnan(want_o)
    # bf16 result: within one bf16 rounding (2^-8 relative) of the fp64 merge
    err = np.abs(g1.float().cpu().numpy() - want_o)[fin]
    assert (err <= np.abs(want_o[fin]) * 2.0 ** -8 + 1e-3).all(), err.max()
    assert np.abs(acc.cpu().numpy() - want_o)[fin].max() < 1e-4
    for got in (gl1, lacc):
        gl = got.cpu().numpy()
        both = np.isfinite(want_l)
        assert np.abs(gl[both] - want_l[both]).max() < 1e-4


def test_peer_gather_all_to_all_layouts():
    """orl_peer_gather (the Ulysses all-to-alls over peer memory) on buffers of this one GPU standing for the peers'
    symmetric buffers: both directions land every row segment where the NCCL all-to-all puts it"""
    import ctypes
    from onereel_b200 import _lib as L
    n, rows, H, Dh = 4, 37, 8, 64
    Hl, es = H // n, 2
    g = torch.Generator(device='cuda').manual_seed(5)
    src = [torch.randn(3, rows, H * Dh, generator=g, device='cuda').to(torch.bfloat16) for _ in range(n)]
    s = torch.cuda.current_stream().cuda_stream
    for r in range(n):
        outs = [torch.empty(n * rows, Hl, Dh, dtype=torch.bfloat16, device='cuda') for _ in range(3)]
        seg = Hl * Dh * es
        S = (ctypes.c_void_p * (3 * n))(*[src[p][pl].data_ptr() for pl in range(3) for p in range(n)])
        Dd = (ctypes.c_void_p * 3)(*[o.data_ptr() for o in outs])
        assert L.lib().orl_peer_gather(S, Dd, 3, n, rows, seg, r * seg, H * Dh * es, rows * seg, seg, s) == 0
        for pl in range(3):
            want = torch.cat([src[p][pl].view(rows, H, Dh)[:, r * Hl:(r + 1) * Hl] for p in range(n)])
            assert torch.equal(outs[pl], want)
    ov = [torch.randn(n * rows, Hl, Dh, generator=g, device='cuda').to(torch.bfloat16) for _ in range(n)]
    for r in range(n):
        out = torch.empty(rows, H, Dh, dtype=torch.bfloat16, device='cuda')
        seg = Hl * Dh * es
        S = (ctypes.c_void_p * n)(*[x.data_ptr() for x in ov])
        Dd = (ctypes.c_void_p * 1)(out.data_ptr())
        assert L.lib().orl_peer_gather(S, Dd, 1, n, rows, seg, r * rows * seg, seg, seg, H * Dh * es, s) == 0
        want = torch.cat([ov[p][r * rows:(r + 1) * rows] for p in range(n)], dim=1)
        assert torch.equal(out, want)
    torch.cuda.synchronize()
