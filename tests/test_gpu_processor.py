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
