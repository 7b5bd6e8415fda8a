"""Wan2.2 self-attention on B200 — the reference's `onereel.models.wan` processor (src/onereel/models/wan.py:33-58
Context, 64-74 _qk, 77-173 Processor, 248-271 _plan_parallel).

Self-attention has no joint text. One GPU / Ulysses: `ranges` — every scene's keys are one contiguous token range
(scene plus adjacent halo), read in place by the attention kernel (orl_attn_plan_ranges: no copy), or packed per
scene by the gather/pack kernel when the scene also reads frame-memory frames. K/V gathering: `scene`, as Hunyuan's
without text. Bounded cross-scene memory (`memory` = M): `memory`, on onereel_b200/memory.py (one GPU, Ulysses, K/V
gathering). Cross-attention (per scene on its sentence) stays the model's own processor, as in the reference.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from onereel_b200 import attention as A
from onereel_b200 import comm, dist as D, ring as R
from onereel_b200 import memory as MEM
from onereel_b200 import scene as S
from onereel_b200.hunyuan15 import _attend, _layout_key
from onereel_b200.layout import SceneLayout
from onereel_b200.rope import qk_norm_rope as fused_qk_norm_rope

TEXT_LEN = 512


@dataclass
class Context:
    """wan.py:33-58 (same fields and defaults)"""
    layout: SceneLayout
    mode: str = 'scene'
    theta: float = 1.0
    kv_chunks: int = 1
    memory: int = 0
    frame_memory: object = None
    T: int = 0
    fwd: int = 0
    own: list = field(default_factory=list)
    path: dict = field(default_factory=dict)
    run_mode: str = 'scene'
    ring: object = None
    height: int = 704
    width: int = 1280
    cfg: bool = False
    attn_override: object = None
    _mem: object = None
    _cache: dict = field(default_factory=dict)

    def cond(self) -> bool:
        return (self.fwd - 1) % 2 == 0 if self.cfg else True

    def step(self) -> int:
        return (self.fwd - 1) // 2 if self.cfg else self.fwd - 1


def qk_norm_rope(q, k, wq, wk, eps: float, cos, sin, heads: int):
    """wan.py:64-74 in torch ops: RMSNorm over the hidden dimension, then the interleaved RoPE of diffusers' Wan
    attention. The processor uses the fused orl_qk_norm_rope kernel; this is the same math for other callers."""
    def norm(x, w):
        return F.rms_norm(x, (x.shape[-1],), w, eps)

    def rope(x):
        x1, x2 = x.unflatten(-1, (-1, 2)).unbind(-1)
        c, s_ = cos[..., 0::2], sin[..., 1::2]
        return torch.stack([x1 * c - x2 * s_, x1 * s_ + x2 * c], -1).flatten(-2).type_as(x)
    return rope(norm(q, wq).unflatten(2, (heads, -1))), rope(norm(k, wk).unflatten(2, (heads, -1)))


class Processor:
    def __init__(self, ctx: Context, kind: str, orig, layer: int):
        self.ctx, self.kind, self.orig, self.layer = ctx, kind, orig, layer

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, rotary_emb=None):
        """wan.py:81-108"""
        ctx, T, lay = self.ctx, self.ctx.T, self.ctx.layout
        a, b = ctx.own[D.rank()]
        if self.kind == 'cross':
            pieces = ([(j, lo, hi) for j, lo, hi in ctx.ring.local[D.rank()] if hi > lo] if ctx.run_mode == 'ring' else
                      [(j, lo - a, hi - a) for j, (lo, hi) in [(j, (max(lo * T, a), min(hi * T, b)))
                                                               for j, (lo, hi) in enumerate(lay.ranges)
                                                               if lo * T < b and hi * T > a]])
            return torch.cat([self.orig(attn, hidden_states[:, lo:hi],
                                        encoder_hidden_states[:, j * TEXT_LEN:(j + 1) * TEXT_LEN], None, rotary_emb)
                              for j, lo, hi in pieces], 1)
        rows = ctx.ring.perm[a:b] if ctx.run_mode == 'ring' else slice(a, b)
        cos, sin = (x[:, rows].reshape(b - a, -1) for x in rotary_emb)
        H = attn.heads
        # hidden-dimension RMSNorm + Wan's interleaved RoPE in one fused kernel (replaces the compiled _qk)
        q = fused_qk_norm_rope(attn.to_q(hidden_states).to(torch.bfloat16), attn.norm_q.weight, cos, sin, H,
                               attn.norm_q.eps, per_head=False, sin_shift=1)
        k = fused_qk_norm_rope(attn.to_k(hidden_states).to(torch.bfloat16), attn.norm_k.weight, cos, sin, H,
                               attn.norm_k.eps, per_head=False, sin_shift=1)
        v = attn.to_v(hidden_states).unflatten(2, (H, -1))[0].to(torch.bfloat16).contiguous()
        if ctx.attn_override is not None:
            qa, ka, va = comm.a2a_heads(q), comm.a2a_heads(k), comm.a2a_heads(v)
            r = ctx.attn_override(self.layer, qa, ka, va)
            o = comm.a2a_tokens(self.ranges(qa, ka, va) if r is None else r)
        elif ctx.memory:
            o = self.memory(q, k, v)
        elif ctx.run_mode == 'ulysses' or D.world() == 1:
            o = comm.a2a_tokens(self.ranges(comm.a2a_heads(q), comm.a2a_heads(k), comm.a2a_heads(v)))
        elif ctx.run_mode == 'ring':
            o = R.attention(ctx.ring, q, k, v, tag=id(lay.extra))[0]
        else:
            o = self.scene(q, k, v)
        return attn.to_out[1](attn.to_out[0](o.flatten(1, 2)[None].type_as(hidden_states)))

    def ranges(self, q, k, v):
        """wan.py:110-124: all tokens; every scene's keys one contiguous range read in place, or packed per scene when
        it reads extra frames"""
        T, lay = self.ctx.T, self.ctx.layout
        if any(lay.extra.get(j) for j in range(lay.n_scenes)):
            H, Dh = q.shape[1:]
            L = lay.n_frames * T
            key = ('wan_ranges', _layout_key(lay), T, H, Dh, str(q.device))
            plan = self.ctx._cache.get(key)
            if plan is None:
                scenes = [(j, (lo * T, hi * T)) for j, (lo, hi) in enumerate(lay.ranges)]
                plan = self.ctx._cache[key] = S.ScenePlan(S.scene_segments(lay, T, None, scenes, set(), (0, L)),
                                                          H * Dh * 2, H, q.device)
            o = torch.empty_like(q)
            _attend(plan, q, None, k, v, None, None, o, None)
            return o
        q_ranges = [(lo * T, hi * T) for lo, hi in lay.ranges]
        k_ranges = [(a * T, b * T) for a, b in (lay.key_range(j) for j in range(lay.n_scenes))]
        for j, (a, b) in enumerate(lay.key_range(j) for j in range(lay.n_scenes)):
            assert b - a == len(lay.key_frames(j)), 'halo must be contiguous with its scene'
        return A.overlapping_ranges(q, k, v, q_ranges, k_ranges)

    def scene(self, q, k, v):
        """wan.py:126-152: K/V gathering; scenes whose keys are all local attend while the exchange is in flight"""
        ctx, T, lay = self.ctx, self.ctx.T, self.ctx.layout
        H, Dh = q.shape[1:]
        r = D.rank()
        own = ctx.own[r]
        key = ('wan_scene', _layout_key(lay), T, tuple(map(tuple, ctx.own)), r, H, Dh, str(q.device))
        plans = ctx._cache.get(key)
        if plans is None:
            rindex = S.remote_index_of(lay, T, ctx.own, r, comm.needed) if D.world() > 1 else []
            mine, _ = S.pieces(lay, T, own)
            near = [p for p in mine if S.is_local(lay, T, own, p[0])]
            far = [p for p in mine if not S.is_local(lay, T, own, p[0])]
            mk = lambda g: S.ScenePlan(S.scene_segments(lay, T, None, g, set(), own, rindex), H * Dh * 2, H,
                                       q.device) if g else None
            plans = ctx._cache[key] = (rindex, mk(near), mk(far))
        rindex, near, far = plans
        ex = comm.kv_exchange(getattr(ctx, 'exchange', 'peer'), lay, ctx.own, T, k, v) if D.world() > 1 else None
        if ex is not None and ex.remote_index != rindex:
            raise RuntimeError('exchange layout differs from the compiled plan')
        ov = torch.empty_like(q)
        _attend(near, q, None, k, v, None, None, ov, None)
        if ex is not None:
            ex.wait()
        _attend(far, q, None, k, v, None, None, ov, None, ex.remote_k if ex else None, ex.remote_v if ex else None)
        return ov



    def memory(self, q, k, v):
        """wan.py:154-173: bounded cross-scene memory (onereel_b200.memory). One GPU / Ulysses: all tokens of the
        local heads; K/V gathering: this rank's scene pieces, with the missing scene frames and every boundary
        candidate received from their owners."""
        ctx, T, lay = self.ctx, self.ctx.T, self.ctx.layout
        if ctx._mem is None:
            ctx._mem = MEM.MemoryAttention(MEM.BoundaryMemory(ctx.memory))
        ulysses = ctx.run_mode == 'ulysses' or D.world() == 1
        rk = rv = None
        if ulysses:
            q, k, v = comm.a2a_heads(q), comm.a2a_heads(k), comm.a2a_heads(v)
            own, remote_index = (0, lay.n_frames * T), []
            scenes = [(j, (lo * T, hi * T)) for j, (lo, hi) in enumerate(lay.ranges)]
        else:
            own = tuple(ctx.own[D.rank()])
            ex = comm.HaloExchange(lay, ctx.own, T, k, v, extra=MEM.candidate_frames(lay)[0])
            ex.wait()
            remote_index, rk, rv = ex.remote_index, ex.remote_k, ex.remote_v
            scenes = S.pieces(lay, T, own)[0]
        Hl, Dh = q.shape[1:]
        pk = ('wan', _layout_key(lay), T, own, tuple(map(tuple, remote_index)), Hl, Dh, str(q.device))
        plan = ctx._mem.plans.get(pk)
        if plan is None:
            plan = ctx._mem.plans[pk] = MEM.MemoryPlan.for_rank(lay, T, None, own, remote_index, scenes, set(),
                                                                q.device)
        o = torch.empty_like(q)
        ctx._mem.run((self.layer, ctx.cond()), plan, q, k, v, None, None, None, o, None, rk, rv)
        return comm.a2a_tokens(o) if ulysses else o


def plan_parallel(ctx: Context, heads: int):
    """wan.py:248-271"""
    n, lay = D.world(), ctx.layout
    ctx.ring = None
    if n == 1:
        ctx.run_mode, ctx.own, ctx.path = 'scene', [(0, lay.n_frames * ctx.T)], {}
        return
    if ctx.mode == 'ring':                       # baseline: USP's Ring with every scene split evenly over the ranks
        assert not ctx.memory, 'the ring path runs the halo / frame-memory scene attention'
        ctx.ring = R.RingPlan(lay, n, ctx.T)
        ctx.run_mode, ctx.own = 'ring', ctx.ring.own
        ctx.path = dict(path='ring', V_R=ctx.ring.volume(), V_U=4 * lay.n_frames * ctx.T * (n - 1) / n ** 2)
        return
    gather = comm.partition(lay, n, ctx.T, 'scene', None, ctx.memory)
    ctx.path = comm.choose_path(lay, gather, ctx.T, ctx.theta)
    ctx.path['ulysses_ok'] = lay.n_frames * ctx.T % n == 0 and heads % n == 0
    ctx.run_mode = ctx.mode if ctx.mode != 'auto' else ctx.path['path'] if ctx.path['ulysses_ok'] else 'scene'
    assert ctx.run_mode != 'ulysses' or ctx.path['ulysses_ok'], f'Ulysses needs video tokens and heads divisible by {n}'
    ctx.own = gather if ctx.run_mode == 'scene' else comm.partition(lay, n, ctx.T, 'ulysses')


_plan_parallel = plan_parallel
