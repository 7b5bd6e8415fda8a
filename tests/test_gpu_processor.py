"""The attention processor end to end (hunyuan15.Processor.__call__: projections, q/k RMSNorm, RoPE, scene attention
on the B200 kernels, output projections) inside the random-init DiT stand-in, against the same model whose processor
computes the scene attention in fp32 torch from the oracle's segment list (B200 only)."""
import pytest
import torch

from oracle import layout_oracle as LO

pytestmark = pytest.mark.gpu


class _RefProcessor:
    """hunyuan15.Processor with scene() replaced by fp32 softmax attention per oracle segment"""

    def __init__(self, inner):
        self.inner = inner

    def __call__(self, *a, **k):
        from onereel_b200 import hunyuan15 as HY
        proc = self.inner
        ctx = proc.ctx

        def scene(q, k, v, eq, ek, ev):
            olay = LO.Layout(ctx.layout.lengths, ctx.layout.halo, ctx.layout.sides, ctx.layout.extra)
            T, L = ctx.T, ctx.layout.n_frames * ctx.T
            segs = LO.hunyuan_segments(olay, T, ctx.counts[ctx.cond()], LO.scene_pieces(olay, T, (0, L))[0],
                                       set(range(olay.n_scenes)))
            Q, K, V = (torch.cat([x, e]).float() for x, e in ((q, eq), (k, ek), (v, ev)))
            idx = lambda rows: torch.tensor([L + r[1] if isinstance(r, tuple) else r for r in rows], device=q.device)
            out = torch.zeros_like(Q)
            for kind, j, qr, kr in segs:
                qi, ki = idx(qr), idx(kr)
                s = torch.einsum('qhd,khd->hqk', Q[qi], K[ki]) * q.shape[-1] ** -0.5
                out[qi] = torch.einsum('hqk,khd->qhd', torch.softmax(s, -1), V[ki])
            return out[:L].to(q.dtype), out[L:].to(q.dtype)
        saved = proc.scene
        proc.scene = scene
        try:
            return HY.Processor.__call__(proc, *a, **k)
        finally:
            proc.scene = saved


def test_processor_call_in_standin_matches_fp32_attention():
    if not torch.cuda.is_available():
        pytest.skip('needs a B200')
    from onereel_b200 import attention as A, hunyuan15 as HY, standin
    from onereel_b200.layout import SceneLayout
    lay = SceneLayout([3, 2, 4], halo=1, extra={0: [5], 2: [0]})
    T, counts = 48, [7, 9, 5]
    ctx = HY.Context(lay, T=T, counts={True: counts, False: counts}, own=[(0, lay.n_frames * T)])
    model = standin.build(ctx, 'cuda', dim=256, heads=2, blocks=2, seed=3)
    g = torch.Generator().manual_seed(0)
    hs = torch.randn(1, lay.n_frames * T, 256, generator=g).cuda().bfloat16()
    ehs = torch.randn(1, sum(counts), 256, generator=g).cuda().bfloat16()
    temb = torch.randn(1, 256, generator=g).cuda().bfloat16()
    cos, sin = standin.rope_3d(lay.n_frames, 6, 8, 128)
    rot = (cos.cuda(), sin.cuda())
    with torch.no_grad():
        ctx.fwd = 1
        out, eout = model(hs, ehs, temb, rot)
        torch.cuda.synchronize()
        A.check()
        for blk in model.transformer_blocks:
            blk.attn.processor = _RefProcessor(blk.attn.processor)
        ref, eref = model(hs, ehs, temb, rot)
    rel = lambda x, y: ((x.float() - y.float()).norm() / y.float().norm()).item()
    assert rel(out, ref) < 2e-2 and rel(eout, eref) < 2e-2, (rel(out, ref), rel(eout, eref))


def test_shared_pos_adjacent_matches_reference_math():
    """shared_pos='adjacent': the shared-frame keys re-rotated to their adjacent temporal positions (the reference's
    _move_shared: apply_rotary_emb with (cos[a], -sin[a]) then (cos[b], sin[b])) before the fp32 attention"""
    if not torch.cuda.is_available():
        pytest.skip('needs a B200')
    from onereel_b200 import attention as A, hunyuan15 as HY, standin
    from onereel_b200.layout import SceneLayout
    lay = SceneLayout([3, 2, 4], halo=1, extra={0: [7], 2: [0]})
    T, H, Dh, counts = 48, 2, 128, [7, 9, 5]
    L = lay.n_frames * T
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(L, H, Dh, generator=g).cuda().bfloat16() for _ in range(3))
    eq, ek, ev = (torch.randn(sum(counts), H, Dh, generator=g).cuda().bfloat16() for _ in range(3))
    cos, sin = (t.cuda() for t in standin.rope_3d(lay.n_frames, 6, 8, Dh))
    ctx = HY.Context(lay, T=T, counts={True: counts}, fwd=1, own=[(0, L)], shared_pos='adjacent')
    ctx._rot_full = (cos, sin)
    ov, ot = HY.Processor(ctx, 0).scene(q, k, v, eq, ek, ev)
    torch.cuda.synchronize()
    A.check()

    def rot(x, c, s_):                               # diffusers apply_rotary_emb, interleaved pairs, fp32
        xr, xi = x.float().unflatten(-1, (-1, 2)).unbind(-1)
        return x.float() * c[:, None] + torch.stack([-xi, xr], -1).flatten(-2) * s_[:, None]
    olay = LO.Layout(lay.lengths, lay.halo, lay.sides, lay.extra)
    segs = LO.hunyuan_segments(olay, T, counts, LO.scene_pieces(olay, T, (0, L))[0], {0, 1, 2})
    Q, K, V = (torch.cat([x, e]).float() for x, e in ((q, eq), (k, ek), (v, ev)))
    idx = lambda rows: torch.tensor([L + r[1] if isinstance(r, tuple) else r for r in rows], device='cuda')
    ref = torch.zeros_like(Q)
    for kind, j, qr, kr in segs:
        qi, ki = idx(qr), idx(kr)
        kk = K[ki].clone()
        if kind == 'v':
            shared = lay.shared_frames(j)
            n = len(lay.frames[j]) * T
            if shared:
                a_rows, b_rows = [], []
                for f, dst in zip(shared, HY.shared_positions(ctx, j)):
                    d = dst - HY.frame_position(ctx, f)
                    a = 0 if d >= 0 else -d
                    a_rows.append(torch.arange(a * T, (a + 1) * T))
                    b_rows.append(torch.arange((a + d) * T, (a + d + 1) * T))
                ar, br = torch.cat(a_rows).cuda(), torch.cat(b_rows).cuda()
                x = rot(kk[n:n + len(shared) * T].bfloat16(), cos[ar], -sin[ar]).bfloat16()
                kk[n:n + len(shared) * T] = rot(x, cos[br], sin[br]).bfloat16().float()
        s = torch.einsum('qhd,khd->hqk', Q[qi], kk) * Dh ** -0.5
        ref[qi] = torch.einsum('hqk,khd->qhd', torch.softmax(s, -1), V[ki])
    rel = lambda x, y: ((x.float() - y.float()).norm() / y.float().norm()).item()
    assert rel(ov, ref[:L]) < 2e-2 and rel(ot, ref[L:]) < 2e-2, (rel(ov, ref[:L]), rel(ot, ref[L:]))
    # and it differs from the 'source' positions (the rotation did something)
    ctx2 = HY.Context(lay, T=T, counts={True: counts}, fwd=1, own=[(0, L)])
    ov2, _ = HY.Processor(ctx2, 0).scene(q, k, v, eq, ek, ev)
    assert rel(ov2, ov) > 1e-3
