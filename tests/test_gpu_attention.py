"""The sm_100a varlen attention kernel and the pack kernel against the fp32 reference and the CPU oracle (B200 only)."""
import numpy as np
import pytest
import torch

from oracle import attention_oracle as AO, layout_oracle as LO
from tests.gpu_ref import MAX_ABS, MEAN_ABS, compare, ref_attention

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module', autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip('needs a B200')
    from onereel_b200.csrc.build import build
    build()


def rand(*shape, seed=0, dev='cuda'):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dev, torch.bfloat16)


def run_case(segs, H, Dh, seed=0, lse=True):
    from onereel_b200 import attention as A
    lq, lk = [a for a, _ in segs], [b for _, b in segs]
    q = rand(max(sum(lq), 1), H, Dh, seed=seed)
    k = rand(max(sum(lk), 1), H, Dh, seed=seed + 1)
    v = rand(max(sum(lk), 1), H, Dh, seed=seed + 2)
    qs = np.cumsum([0] + lq)[:-1].tolist()
    ks = np.cumsum([0] + lk)[:-1].tolist()
    out, l = A.attend(q, k, v, qs, lq, ks, lk, lse=lse)
    torch.cuda.synchronize()
    A.check()
    return q, k, v, qs, lq, ks, lk, out, l


CASES = [
    [(1, 1)],
    [(128, 128)],
    [(127, 129), (128, 128), (129, 127)],
    [(256, 300), (257, 1), (300, 2000)],
    [(16, 336), (256, 336), (1, 4096), (600, 77)],
    [(1000, 513), (3, 1000), (512, 512)],
]


@pytest.mark.parametrize('Dh', [128, 64])
@pytest.mark.parametrize('H', [1, 4])
@pytest.mark.parametrize('ci', range(len(CASES)))
def test_varlen_matches_fp32(ci, H, Dh):
    q, k, v, qs, lq, ks, lk, out, l = run_case(CASES[ci], H, Dh, seed=ci)
    ref = ref_attention(q, k, v, qs, lq, ks, lk)
    mx, mean, lmx = compare(out, l, ref, qs)
    assert mx < MAX_ABS and mean < MEAN_ABS, (mx, mean)
    assert lmx < 1e-3, lmx


def test_heads_16_and_24():
    for H in (16, 24):
        q, k, v, qs, lq, ks, lk, out, l = run_case([(700, 1500), (130, 260)], H, 128, seed=H)
        mx, mean, lmx = compare(out, l, ref_attention(q, k, v, qs, lq, ks, lk), qs)
        assert mx < MAX_ABS and mean < MEAN_ABS and lmx < 1e-3, (H, mx, mean, lmx)


def test_zero_keys_gives_zero_output():
    q, k, v, qs, lq, ks, lk, out, l = run_case([(5, 0), (64, 64)], 2, 64, seed=3)
    assert torch.all(out[:5] == 0)
    assert torch.all(torch.isinf(l[:, :5]))
    mx, mean, _ = compare(out, None, ref_attention(q, k, v, qs[1:], lq[1:], ks[1:], lk[1:]), qs[1:])
    assert mx < MAX_ABS


def test_deterministic_bitwise():
    a = run_case(CASES[4], 4, 128, seed=9)[7]
    b = run_case(CASES[4], 4, 128, seed=9)[7]
    assert torch.equal(a, b)


def test_varlen_api_and_packed_match_reference_semantics():
    """the drop-in functions: varlen / varlen_lse on cu_seqlens, packed / packed_lse on segment lists"""
    from onereel_b200 import attention as A
    H, Dh = 4, 64
    segs = [(rand(200, H, Dh, seed=1), rand(333, H, Dh, seed=2), rand(333, H, Dh, seed=3)),
            (rand(17, H, Dh, seed=4), rand(50, H, Dh, seed=5), rand(50, H, Dh, seed=6))]
    outs = A.packed(segs)
    outs_l = A.packed_lse(segs)
    for (qq, kk, vv), o, (o2, l2) in zip(segs, outs, outs_l):
        want, wl = AO.attend(qq.float().cpu().numpy(), kk.float().cpu().numpy(), vv.float().cpu().numpy())
        assert np.abs(o.float().cpu().numpy() - want).max() < MAX_ABS
        assert torch.equal(o, o2)
        assert np.abs(l2.cpu().numpy() - wl).max() < 1e-3
    q = torch.cat([s[0] for s in segs])
    k = torch.cat([s[1] for s in segs])
    v = torch.cat([s[2] for s in segs])
    cq, ck = A.cu_seqlens([200, 17]), A.cu_seqlens([333, 50])
    o = A.varlen(q, k, v, cq, ck, 200, 333)
    assert torch.equal(o, torch.cat(outs))
    o3, l3 = A.varlen_lse(q, k, v, cq, ck, 200, 333)
    assert torch.equal(o3, o) and l3.shape == (H, 217)
    A.check()


def test_overlapping_ranges_reads_in_place():
    from onereel_b200 import attention as A
    T, H, Dh = 32, 2, 128
    lay = LO.Layout([3, 5, 4], halo=2, sides='next')
    L = lay.n_frames * T
    q, k, v = rand(L, H, Dh, seed=1), rand(L, H, Dh, seed=2), rand(L, H, Dh, seed=3)
    qr = [(lo * T, hi * T) for lo, hi in lay.ranges()]
    kr = [(a * T, b * T) for a, b in (lay.key_range(j) for j in range(lay.n_scenes))]
    o = A.overlapping_ranges(q, k, v, qr, kr)
    want = AO.wan_scene(lay, T, *(x.float().cpu().numpy() for x in (q, k, v)))
    d = np.abs(o.float().cpu().numpy() - want)
    assert d.max() < MAX_ABS and d.mean() < MEAN_ABS


def test_dense():
    from onereel_b200 import attention as A
    B, S, H, Dh = 2, 300, 2, 64
    q, k, v = rand(B, S, H, Dh, seed=1), rand(B, S, H, Dh, seed=2), rand(B, S, H, Dh, seed=3)
    o = A.dense(q, k, v)
    ref = torch.nn.functional.scaled_dot_product_attention(*(x.float().transpose(1, 2) for x in (q, k, v)))
    assert (o.float() - ref.transpose(1, 2)).abs().max().item() < MAX_ABS


def test_pack_rows_bit_exact():
    from onereel_b200.pack import pack_rows
    parts = [rand(n, 3, 64, seed=n) for n in (5, 0, 17, 1, 200)]
    dst = torch.empty(sum(p.shape[0] for p in parts), 3, 64, dtype=torch.bfloat16, device='cuda')
    pack_rows(parts, dst)
    assert torch.equal(dst, torch.cat(parts))


def test_lse_merge_matches_oracle():
    from onereel_b200 import attention as A
    H, Dh = 4, 128
    q, k, v = rand(100, H, Dh, seed=1), rand(500, H, Dh, seed=2), rand(500, H, Dh, seed=3)
    o1, l1 = A.attend(q, k[:200].contiguous(), v[:200].contiguous(), [0], [100], [0], [200], lse=True)
    o2, l2 = A.attend(q, k[200:].contiguous(), v[200:].contiguous(), [0], [100], [0], [300], lse=True)
    A.lse_merge(o1, l1, o2, l2)
    want, wl = AO.attend(*(x.float().cpu().numpy() for x in (q, k, v)))
    assert np.abs(o1.float().cpu().numpy() - want).max() < MAX_ABS
    assert np.abs(l1.cpu().numpy() - wl).max() < 1e-3


def test_cfg1_layout_on_gpu():
    """BASELINE cfg1 (bf16 on the GPU) through the packed path against the reference's own output (golden)"""
    from pathlib import Path
    from onereel_b200 import attention as A
    g = torch.Generator().manual_seed(0)
    T, H, Dh, counts = 64, 4, 64, [16, 16, 16]
    q, k, v = (torch.randn(12 * T, H, Dh, generator=g) for _ in range(3))
    eq, ek, ev = (torch.randn(48, H, Dh, generator=g) for _ in range(3))
    lay = LO.Layout([4, 3, 5], halo=0, extra={0: [4], 1: [0], 2: [0, 4]})
    segs = LO.hunyuan_segments(lay, T, counts, LO.scene_pieces(lay, T, (0, 12 * T))[0], {0, 1, 2})
    dev = lambda x: x.to('cuda', torch.bfloat16)
    vid = [dev(x) for x in (q, k, v)]
    txt = [dev(x) for x in (eq, ek, ev)]
    rows = lambda rs, i: torch.stack([txt[i][r[1]] if isinstance(r, tuple) else vid[i][r] for r in rs])
    outs = A.packed([(rows(s[2], 0), rows(s[3], 1), rows(s[3], 2)) for s in segs])
    gold = np.load(Path(__file__).resolve().parent / 'golden' / 'cfg1.npz')
    ov = torch.cat([o for s, o in zip(segs, outs) if s[0] == 'v']).float().cpu().numpy()
    ot = torch.cat([o for s, o in zip(segs, outs) if s[0] == 't']).float().cpu().numpy()
    d = np.concatenate([np.abs(ov[::4] - gold['ov']).ravel(), np.abs(ot - gold['ot']).ravel()])
    assert d.max() < MAX_ABS and d.mean() < MEAN_ABS, (d.max(), d.mean())


def test_cfg2_full_size_sampled_rows():
    """BASELINE cfg2 packed shapes (Σq 49 802, Σk 118 684, H 16, D 128), every 13th query row against fp32"""
    lay = LO.Layout([8, 6, 10, 7], halo=0, extra={j: [f for f in (0, 8, 14, 24) if not lo <= f < hi]
                                                  for j, (lo, hi) in enumerate([(0, 8), (8, 14), (14, 24), (24, 31)])})
    T, counts = 1590, [128] * 4
    segs = LO.hunyuan_segments(lay, T, counts, LO.scene_pieces(lay, T, (0, 31 * T))[0], {0, 1, 2, 3})
    segs_l = [(len(s[2]), len(s[3])) for s in segs]
    assert sum(a for a, _ in segs_l) == 49802 and sum(b for _, b in segs_l) == 118684
    from onereel_b200 import attention as A
    lq, lk = [a for a, _ in segs_l], [b for _, b in segs_l]
    q, k, v = rand(sum(lq), 16, 128, seed=1), rand(sum(lk), 16, 128, seed=2), rand(sum(lk), 16, 128, seed=3)
    qs, ks = np.cumsum([0] + lq)[:-1].tolist(), np.cumsum([0] + lk)[:-1].tolist()
    out, l = A.attend(q, k, v, qs, lq, ks, lk, lse=True)
    torch.cuda.synchronize()
    A.check()
    rows = [torch.arange(0, n, 13) for n in lq]
    mx, mean, lmx = compare(out, l, ref_attention(q, k, v, qs, lq, ks, lk, rows=rows), qs)
    assert mx < MAX_ABS and mean < MEAN_ABS and lmx < 1e-3, (mx, mean, lmx)


def test_ring_single_rank_matches_oracle():
    """the Scene-Ring path on one rank (one step: pack, attention with LSE, LSE merge into the fp32 accumulator)
    against the CPU oracle of the reference's scene attention (hunyuan15.Processor.scene), within the kernel
    tolerance"""
    from onereel_b200 import hunyuan15 as HY, ring as R
    from onereel_b200.layout import SceneLayout
    lay = SceneLayout([3, 5, 2], halo=1, extra={0: [7], 2: [0]})
    T, H, Dh, counts = 32, 4, 128, [5, 9, 3]
    L = lay.n_frames * T
    q, k, v = rand(L, H, Dh, seed=1), rand(L, H, Dh, seed=2), rand(L, H, Dh, seed=3)
    eq, ek, ev = rand(17, H, Dh, seed=4), rand(17, H, Dh, seed=5), rand(17, H, Dh, seed=6)
    ctx = HY.Context(lay, T=T, counts={True: counts}, fwd=1, own=[(0, L)])
    plan = R.RingPlan(lay, 1, T)
    rows = plan.perm
    ov, ot = R.attention(plan, q[rows].contiguous(), k[rows].contiguous(), v[rows].contiguous(), eq, ek, ev,
                         ctx.text_ranges(), id(lay.extra))
    torch.cuda.synchronize()
    olay = LO.Layout([3, 5, 2], halo=1, extra={0: [7], 2: [0]})
    want_v, want_t, _ = AO.hunyuan_scene(olay, T, counts, *(x.float().cpu().numpy() for x in (q, k, v, eq, ek, ev)))
    dv = np.abs(ov.float().cpu().numpy() - want_v[rows.cpu().numpy()])
    dt = np.abs(ot.float().cpu().numpy() - want_t)
    d = np.concatenate([dv.ravel(), dt.ravel()])
    assert d.max() < MAX_ABS and d.mean() < MEAN_ABS, (d.max(), d.mean())


@pytest.mark.parametrize('Dh', [128, 64])
def test_varlen_device_cu_seqlens_plan_on_gpu(Dh):
    """varlen with cu_seqlens on the device (orl_attn_fwd_cu: work list planned on the GPU) gives the same bits as
    the host-planned call, for segments with no query rows, no keys, ragged lengths and equal key counts (the stable
    order), and rejects decreasing cu_seqlens through the error word"""
    from onereel_b200 import _lib as L, attention as A
    H = 3
    lq = [0, 300, 1, 257, 128, 0, 45, 600]
    lk = [10, 129, 0, 400, 129, 7, 2000, 129]
    q = rand(sum(lq), H, Dh, seed=11)
    k = rand(sum(lk), H, Dh, seed=12)
    v = rand(sum(lk), H, Dh, seed=13)
    cq = torch.tensor(np.cumsum([0] + lq), dtype=torch.int32, device='cuda')
    ck = torch.tensor(np.cumsum([0] + lk), dtype=torch.int32, device='cuda')
    qs, ks = np.cumsum([0] + lq)[:-1].tolist(), np.cumsum([0] + lk)[:-1].tolist()
    want, wl = A.attend(q, k, v, qs, lq, ks, lk, lse=True)
    for _ in range(2):                                  # the scratch is reused by the second call
        o, l = A.varlen_lse(q, k, v, cq, ck, max(lq), max(lk))
        torch.cuda.synchronize()
        A.check()
        assert torch.equal(o, want)
        assert torch.equal(l, wl)
    bad = torch.tensor([0, 300, 200, sum(lq)], dtype=torch.int32, device='cuda')
    A.varlen(q, k, v, bad, ck[:4].contiguous(), 300, 400)
    torch.cuda.synchronize()
    with pytest.raises(L.OrlError, match='cu_seqlens rejected'):
        A.check()


def test_key_split_of_coarse_launches():
    """attend(split_keys=True) on a launch of less than a few waves with long segments: the two key halves run on two
    streams and merge by log-sum-exp — exact attention within the kernel tolerance of fp32 and of the unsplit call;
    segments too short to split, and a segment without keys, come out as unsplit"""
    from onereel_b200 import attention as A
    H, Dh = 2, 128
    lq, lk = [256, 200, 5, 64], [5000, 2300, 100, 0]
    q, k, v = rand(sum(lq), H, Dh, seed=21), rand(sum(lk), H, Dh, seed=22), rand(sum(lk), H, Dh, seed=23)
    qs, ks = np.cumsum([0] + lq)[:-1].tolist(), np.cumsum([0] + lk)[:-1].tolist()
    splits = A.SPLITS
    o, l = A.attend(q, k, v, qs, lq, ks, lk, lse=True, split_keys=True)
    torch.cuda.synchronize()
    A.check()
    assert A.SPLITS == splits + 1
    o1, l1 = A.attend(q, k, v, qs, lq, ks, lk, lse=True)
    mx, mean, lmx = compare(o, l, ref_attention(q, k, v, qs, lq, ks, lk), qs)
    assert mx < MAX_ABS and mean < MEAN_ABS and lmx < 1e-3, (mx, mean, lmx)
    assert (o.float() - o1.float()).abs().max().item() < MAX_ABS
    assert torch.equal(o[sum(lq[:3]):], torch.zeros_like(o[sum(lq[:3]):]))
    assert torch.isinf(l[:, sum(lq[:3]):]).all()
