"""Random-init HunyuanVideo-1.5-architecture DiT stand-in, for the end-to-end DiT-step measurement (BASELINE cfg4).

diffusers (and the HunyuanVideo-1.5 checkpoint) are not available here, so the step is measured on a documented
stand-in with the block structure the reference's attention processor plugs into (src/onereel/models/hunyuan15.py:
177-210 touches to_q/k/v, norm_q/k, add_q/k/v_proj, norm_added_q/k, to_out, to_add_out): per block, a dual-stream
(video | text) AdaLN-modulated joint-attention layer followed by per-stream GELU FFNs (mlp ratio 4). Hidden 2048,
16 heads x 128, 54 blocks, bf16 weights and activations, random init (seeded). Attention runs through
onereel_b200.hunyuan15.Processor (scene / Ulysses paths, the B200 kernels); the GEMMs are cuBLAS through torch.

FLOPs per token per block (2 per multiply-add): q/k/v 6 d^2 + output 2 d^2 + FFN 16 d^2 = 24 d^2 = 100.7 MFLOP at
d = 2048, for video and text tokens alike, plus the scene attention (4 lq lk H D per segment).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from onereel_b200 import dist as D
from onereel_b200 import hunyuan15 as HY


class RMSNorm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.weight, self.eps = nn.Parameter(torch.ones(dim)), eps

    def forward(self, x):
        return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)


class Attention(nn.Module):
    """the projections diffusers' Attention module carries for HunyuanVideo-1.5 joint attention"""

    def __init__(self, dim, heads):
        super().__init__()
        self.heads = heads
        hd = dim // heads
        self.to_q, self.to_k, self.to_v = (nn.Linear(dim, dim) for _ in range(3))
        self.add_q_proj, self.add_k_proj, self.add_v_proj = (nn.Linear(dim, dim) for _ in range(3))
        self.norm_q, self.norm_k = RMSNorm(hd), RMSNorm(hd)
        self.norm_added_q, self.norm_added_k = RMSNorm(hd), RMSNorm(hd)
        self.to_out = nn.ModuleList([nn.Linear(dim, dim), nn.Identity()])
        self.to_add_out = nn.Linear(dim, dim)
        self.processor = None

    def set_processor(self, p):
        self.processor = p


class Block(nn.Module):
    def __init__(self, dim, heads, mlp_ratio=4):
        super().__init__()
        self.attn = Attention(dim, heads)
        self.mod = nn.Linear(dim, 12 * dim)          # shift / scale / gate x (attention, FFN) x (video, text)
        self.ff = nn.Sequential(nn.Linear(dim, mlp_ratio * dim), nn.GELU(approximate='tanh'),
                                nn.Linear(mlp_ratio * dim, dim))
        self.ff_context = nn.Sequential(nn.Linear(dim, mlp_ratio * dim), nn.GELU(approximate='tanh'),
                                        nn.Linear(mlp_ratio * dim, dim))

    def forward(self, hs, ehs, temb, rot):
        m = self.mod(F.silu(temb))[:, None].chunk(12, -1)
        ln = lambda x: F.layer_norm(x, (x.shape[-1],))
        x = ln(hs) * (1 + m[1]) + m[0]
        c = ln(ehs) * (1 + m[7]) + m[6]
        a, ea = self.attn.processor(self.attn, x, c, None, rot)
        hs = hs + m[2] * a
        ehs = ehs + m[8] * ea
        hs = hs + m[5] * self.ff(ln(hs) * (1 + m[4]) + m[3])
        ehs = ehs + m[11] * self.ff_context(ln(ehs) * (1 + m[10]) + m[9])
        return hs, ehs


class Transformer(nn.Module):
    """54 blocks of the stand-in; forward(hidden [1, video tokens (local rows when sharded), C], text [1, Nt, C],
    temb [1, C], rotary (cos, sin) [all video tokens, head_dim])"""

    def __init__(self, dim=2048, heads=16, blocks=54):
        super().__init__()
        self.transformer_blocks = nn.ModuleList([Block(dim, heads) for _ in range(blocks)])

    def forward(self, hs, ehs, temb, rot):
        for blk in self.transformer_blocks:
            hs, ehs = blk(hs, ehs, temb, rot)
        return hs, ehs


def rope_3d(frames: int, h: int, w: int, head_dim: int = 128, axes=(16, 56, 56), theta: float = 256.0):
    """(cos, sin) [frames * h * w, head_dim] of a 3-D rotary embedding over (frame, row, column), each axis's
    frequencies repeated per interleaved pair (the layout HunyuanVideo's apply_rotary_emb consumes)"""
    assert sum(axes) == head_dim
    parts = []
    grids = torch.meshgrid(torch.arange(frames), torch.arange(h), torch.arange(w), indexing='ij')
    for pos, dim in zip(grids, axes):
        freqs = 1.0 / theta ** (torch.arange(0, dim, 2).float() / dim)
        ang = pos.reshape(-1, 1).float() * freqs[None]
        parts.append(ang.repeat_interleave(2, -1))
    ang = torch.cat(parts, -1)
    return ang.cos(), ang.sin()


def build(ctx: HY.Context, device, dim=2048, heads=16, blocks=54, seed=0) -> Transformer:
    """the stand-in with a B200 Processor on every block (hunyuan15.install's attention part)"""
    torch.manual_seed(seed)
    with torch.device(device):                   # parameters created and initialised on the GPU
        model = Transformer(dim, heads, blocks).to(torch.bfloat16)
    for p in model.parameters():
        nn.init.normal_(p, std=0.02) if p.dim() > 1 else nn.init.zeros_(p)
    for blk in model.transformer_blocks:
        blk.attn.norm_q.weight.data.fill_(1)
        blk.attn.norm_k.weight.data.fill_(1)
        blk.attn.norm_added_q.weight.data.fill_(1)
        blk.attn.norm_added_k.weight.data.fill_(1)
    for i, blk in enumerate(model.transformer_blocks):
        blk.attn.set_processor(HY.Processor(ctx, i))
    return model


@torch.no_grad()
def dit_step(model, ctx: HY.Context, hs_local, ehs_cond, ehs_uncond, temb, rot):
    """one denoising step with classifier-free guidance: a conditional and an unconditional forward (the reference's
    diffusers loop runs the two CFG branches as two sequential forwards), each: 54 blocks on this rank's video rows
    with the scene-parallel attention, then the last-block all-gather of the video tokens (hunyuan15.py:432-439)"""
    outs = []
    for ehs in (ehs_cond, ehs_uncond):
        ctx.fwd += 1
        hs, _ = model(hs_local, ehs, temb, rot)
        outs.append(HY.gather_rows(ctx, hs) if D.world() > 1 else hs)
    return outs
