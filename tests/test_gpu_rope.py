"""The fused q/k RMSNorm + RoPE kernel against the reference processors' torch math (B200 only)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _torch_hunyuan(x, w, cos, sin, heads, eps):
    """hunyuan15.py:187-190: per-head RMSNorm, then diffusers' apply_rotary_emb (interleaved pairs), fp32"""
    x = x.float().unflatten(-1, (heads, -1))
    x = torch.nn.functional.rms_norm(x, (x.shape[-1],), w.float(), eps)
    xr, xi = x.unflatten(-1, (-1, 2)).unbind(-1)
    rot = torch.stack([-xi, xr], -1).flatten(-2)
    return x * cos[:, None].float() + rot * sin[:, None].float()


def _torch_wan(x, w, cos, sin, heads, eps):
    """wan.py:64-74 `_qk`: hidden RMSNorm, then cos[..., 0::2] / sin[..., 1::2] on interleaved pairs, fp32"""
    x = torch.nn.functional.rms_norm(x.float(), (x.shape[-1],), w.float(), eps).unflatten(-1, (heads, -1))
    x1, x2 = x.unflatten(-1, (-1, 2)).unbind(-1)
    c, s_ = cos[:, None, 0::2].float(), sin[:, None, 1::2].float()
    return torch.stack([x1 * c - x2 * s_, x1 * s_ + x2 * c], -1).flatten(-2)


@pytest.mark.parametrize('heads,dh,per_head', [(16, 128, True), (24, 128, False), (4, 64, True), (3, 64, False)])
def test_fused_qk_norm_rope_matches_torch(heads, dh, per_head):
    if not torch.cuda.is_available():
        pytest.skip('needs a B200')
    from onereel_b200.csrc.build import build
    build()
    from onereel_b200.rope import qk_norm_rope
    g = torch.Generator().manual_seed(heads)
    rows = 1001
    x = (3 * torch.randn(rows, heads * dh, generator=g)).cuda().bfloat16()
    w = (1 + 0.1 * torch.randn(dh if per_head else heads * dh, generator=g)).cuda().bfloat16()
    ang = torch.randn(rows, dh // 2, generator=g) * 3
    if per_head:
        cos, sin = ang.cos().repeat_interleave(2, -1).cuda(), ang.sin().repeat_interleave(2, -1).cuda()
        want = _torch_hunyuan(x, w, cos, sin, heads, 1e-6)
        got = qk_norm_rope(x, w, cos, sin, heads, 1e-6, per_head=True, sin_shift=0)
    else:
        cos, sin = ang.cos().repeat_interleave(2, -1).cuda(), ang.sin().repeat_interleave(2, -1).cuda()
        want = _torch_wan(x, w, cos, sin, heads, 1e-6)
        got = qk_norm_rope(x, w, cos, sin, heads, 1e-6, per_head=False, sin_shift=1)
    d = (got.float() - want).abs()
    assert d.max().item() < 3e-2 and d.mean().item() < 3e-3, (d.max().item(), d.mean().item())
    perm = torch.randperm(rows, generator=g).to(torch.int32).cuda()      # written straight into another row order
    out = torch.empty_like(got)
    qk_norm_rope(x, w, cos, sin, heads, 1e-6, per_head=per_head, sin_shift=0 if per_head else 1, out=out, row_map=perm)
    assert torch.equal(out[perm.long()], got)
