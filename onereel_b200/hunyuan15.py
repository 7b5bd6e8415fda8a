"""HunyuanVideo-1.5 scene attention on B200 — the reference's `onereel.models.hunyuan15` attention processor
(src/onereel/models/hunyuan15.py:34-89 Context, 153-170 _segments, 173-303 Processor, 553-573 _plan_parallel).

Same Context fields, same Processor(ctx, layer) with __call__ / scene / ulysses / _far_lse, same outputs. The device
work per layer is: one gather/pack launch for the K/V of every local segment, one attention launch per query source
(video rows of q, text rows of eq) writing straight into the output rows, and on several ranks the K/V exchange
(grouped NCCL send/recv on the high-priority NCCL stream) overlapped with the attention of the scenes whose keys are
all local. The segment list, run tables and work lists are compiled once per (layout, pass, partition) and cached.

The Ring baseline (`mode='ring'`, src/onereel/parallel/ring.py) runs on the same kernels (onereel_b200/ring.py).
Frame memory (`frame_memory`, onereel_b200/frame_memory.py) plugs in through install_attention's hooks;
`shared_pos='adjacent'` re-rotates the shared-frame keys inside the packed K (orl_rope_rows) and `scene_rope`
restarts the temporal RoPE index per scene. The bounded cross-scene memory (`memory` = M, onereel_b200/memory.py)
runs on one GPU, on Ulysses and on the gathering path. `subject_links`, a variant the reference also carries, is not
on this path and raises NotImplementedError.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from onereel_b200 import attention as A
from onereel_b200 import comm, dist as D, ring as R
from onereel_b200 import memory as MEM
from onereel_b200 import scene as S
from onereel_b200.layout import SceneLayout
from onereel_b200.rope import qk_norm_rope, rotate_rows


@dataclass
class Context:
    """hunyuan15.py:34-89 (same fields and defaults)"""
    layout: SceneLayout
    mode: str = 'scene'
    partition: str = 'balanced'
    theta: float = 1.0
    cfg: bool = True
    shared_pos: str = 'source'
    shared_switch: int = 10
    scene_rope: bool = False
    rope_lengths: list = None
    kv_chunks: int = 1
    overlap: str = 'none'
    text_sync: str = 'rows'
    exchange: str = 'peer'      # B200: K/V exchange over peer memory ('peer') or NCCL send/recv ('nccl')
    split_keys: bool = False    # B200: Ulysses may split the keys of a coarse launch in two (LSE merge; not bit-exact)
    memory: int = 0
    frame_memory: object = None
    subject_links: int = 0
    subject_step: int = 3
    subject_layers: tuple = (18, 36)
    subject_top: float = 0.2
    T: int = 0
    fwd: int = 0
    counts: dict = field(default_factory=dict)
    subj_tokens: list = field(default_factory=list)
    subject: object = None
    own: list = field(default_factory=list)
    path: dict = field(default_factory=dict)
    run_mode: str = 'scene'
    ring: object = None
    height: int = 480
    width: int = 848
    attn_override: object = None
    forward_ms: list = field(default_factory=list)
    vae_ms: list = field(default_factory=list)
    _cache: dict = field(default_factory=dict)
    _rot_full: tuple = None
    _mem: object = None

    def step(self) -> int:
        return (self.fwd - 1) // 2 if self.cfg else self.fwd - 1

    def cond(self) -> bool:
        return (self.fwd - 1) % 2 == 0 if self.cfg else True

    def text_ranges(self) -> list[tuple[int, int]]:
        return S.text_ranges(self.counts[self.cond()])


# Optional phase timing for benchmarks: when PHASES is a list, Processor.scene / ulysses append (name, event) pairs,
# each event recorded on the current stream at the end of the named phase (the first one, 'start', at its beginning).
PHASES = None


def _mark(name: str) -> None:
    if PHASES is not None:
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        PHASES.append((name, e))


def _layout_key(lay: SceneLayout):
    return (tuple(lay.lengths), lay.halo, lay.sides, tuple((j, tuple(sorted(v))) for j, v in sorted(lay.extra.items())))


def _unsupported(ctx):
    if ctx.subject_links:
        raise NotImplementedError('subject links are not on the B200 path')


def _move_active(ctx) -> bool:
    """hunyuan15.py:162: shared keys re-rotated to adjacent positions in this forward"""
    return ctx.shared_pos == 'adjacent' or (ctx.shared_pos == 'switch' and ctx.step() >= ctx.shared_switch)


def adjacent_positions(lay, j: int) -> list[int]:
    """hunyuan15.py:92-100: per shared frame of scene j (shared_frames order) its temporal position — the shared
    frames before the scene just before its first frame, those after it just after its last"""
    lo, hi = lay.ranges[j]
    shared = lay.shared_frames(j)
    before = sorted(f for f in shared if f < lo)
    after = sorted(f for f in shared if f >= hi)
    pos = {f: lo - len(before) + i for i, f in enumerate(before)}
    pos.update({f: hi + i for i, f in enumerate(after)})
    return [pos[f] for f in shared]


def frame_position(ctx, f: int) -> int:
    """hunyuan15.py:103-113: temporal RoPE index of latent frame f (with scene_rope: index within its scene, + 1
    after scene 0)"""
    if not ctx.scene_rope:
        return f
    start = 0
    for n in list(ctx.rope_lengths or ctx.layout.lengths):
        if f < start + n:
            return f - start + (start > 0)
        start += n
    raise IndexError(f)


def shared_positions(ctx, j: int) -> list[int]:
    """hunyuan15.py:116-124: per shared frame of scene j, its temporal RoPE index under shared_pos = 'adjacent'"""
    lay = ctx.layout
    if not ctx.scene_rope:
        return adjacent_positions(lay, j)
    shared = lay.shared_frames(j)
    last = max(frame_position(ctx, f) for f in lay.frames[j])
    pos = {f: last + 1 + i for i, f in enumerate(sorted(shared))}
    return [pos[f] for f in shared]


def _shift_rows(ctx, j: int):
    """per shared frame of scene j (shared_frames order), the rotary-table rows a, a + d of two frames d apart in the
    same spatial order, d = its adjacent position minus its own (hunyuan15.py:136-144): R(a + d) R(a)^-1 moves a key
    rotated at its own frame to the adjacent one (the temporal angles compose, the spatial ones cancel)"""
    T = ctx.T
    a_rows, b_rows = [], []
    for f, dst in zip(ctx.layout.shared_frames(j), shared_positions(ctx, j)):
        d = dst - frame_position(ctx, f)
        a = 0 if d >= 0 else -d
        a_rows.append(torch.arange(a * T, (a + 1) * T))
        b_rows.append(torch.arange((a + d) * T, (a + d + 1) * T))
    return torch.cat(a_rows), torch.cat(b_rows)


def _move_shared(ctx, j: int, k: torch.Tensor) -> torch.Tensor:
    """hunyuan15.py:127-150 with the reference's arguments: k = scene j's keys (own frames, then shared frames) rotated
    at their own frame index -> the shared frames' keys re-rotated to their adjacent positions, as one rotation by the
    composed angle (cos(b - a), sin(b - a) from the table rows a, b). Torch ops, for callers holding one scene's keys;
    the processors do the same inside the packed K with the orl_rope_rows kernel."""
    lay, T = ctx.layout, ctx.T
    if not lay.shared_frames(j):
        return k
    n = len(lay.frames[j]) * T
    ar, br = _shift_rows(ctx, j)
    cos, sin = ctx._rot_full
    ca, sa, cb, sb = (t.float().to(k.device) for t in (cos[ar], sin[ar], cos[br], sin[br]))
    x = apply_rotary_emb(k[None, n:], (cb * ca + sb * sa, sb * ca - cb * sa))[0]
    return torch.cat([k[:n], x.to(k.dtype)])


def scene_rope_rows(ctx, device):
    """hunyuan15.py:443-454: per video token row, the rotary row of the same spatial position at its frame index
    within its scene (+ 1 after scene 0)"""
    lengths = list(ctx.rope_lengths or ctx.layout.lengths)
    key = ('scene_rope', tuple(lengths), ctx.T)
    if key not in ctx._cache:
        start = np.repeat(np.cumsum([0] + lengths[:-1]), lengths)
        local = np.arange(sum(lengths)) - start + (start > 0)
        rows = (local[:, None] * ctx.T + np.arange(ctx.T)[None]).reshape(-1)
        ctx._cache[key] = torch.as_tensor(rows, device=device)
    return ctx._cache[key]


def _shared_rotation(ctx, plan, device):
    """hunyuan15.py:127-150 `_move_shared` as one rotation per row: for every video segment of `plan`, the packed K
    rows of its shared frames and the tables of R(dst) R(src)^-1 (the two rotary rows a, a + d of the reference,
    composed: cos(b - a), sin(b - a)); None when no segment has shared frames"""
    cos, sin = ctx._rot_full
    key = ('move', id(plan), cos.data_ptr(), sin.data_ptr())
    if key in ctx._cache:
        return ctx._cache[key]
    lay, T = ctx.layout, ctx.T
    rows, a_rows, b_rows = [], [], []
    for i, sg in enumerate(plan.segs):
        if sg.kind != 'v':
            continue
        shared = lay.shared_frames(sg.scene)
        if not shared:
            continue
        base = plan.cu_k[i] + len(lay.frames[sg.scene]) * T
        rows.append(torch.arange(base, base + len(shared) * T))
        for f, dst in zip(shared, shared_positions(ctx, sg.scene)):
            d = dst - frame_position(ctx, f)
            a = 0 if d >= 0 else -d
            a_rows.append(torch.arange(a * T, (a + 1) * T))
            b_rows.append(torch.arange((a + d) * T, (a + d + 1) * T))
    if not rows:
        ctx._cache[key] = None
        return None
    ar, br = torch.cat(a_rows).to(cos.device), torch.cat(b_rows).to(cos.device)
    ca, sa, cb, sb = (t.float() for t in (cos[ar], sin[ar], cos[br], sin[br]))
    res = (torch.cat(rows).to(device=device, dtype=torch.int32),
           (cb * ca + sb * sa).contiguous(), (sb * ca - cb * sa).contiguous())
    ctx._cache[key] = res
    return res


class _RankPlan:
    """everything one rank needs for a scene-path layer: the pieces, the near / far segment plans (or the LSE
    overlap's local / remote plans), the receive-buffer layout"""

    def __init__(self, ctx, H, Dh, device, lse_overlap):
        lay, T, counts = ctx.layout, ctx.T, ctx.counts[ctx.cond()]
        r = D.rank()
        own = ctx.own[r]
        self.own = own
        self.remote_index = (S.remote_index_of(lay, T, ctx.own, r, comm.needed) if D.world() > 1 else [])
        mine, text_for = S.pieces(lay, T, own)
        near = [p for p in mine if S.is_local(lay, T, own, p[0])]
        far = [p for p in mine if not S.is_local(lay, T, own, p[0])]
        rb = H * Dh * 2
        mk = lambda g, side=None: (S.ScenePlan(S.scene_segments(lay, T, counts, g, text_for & {j for j, _ in g}, own,
                                                                self.remote_index, side), rb, H, device) if g else None)
        self.near = mk(near)
        self.lse = lse_overlap and bool(far)
        if self.lse:
            self.far = None
            self.far_local = mk(far, 'local')
            self.far_remote = mk(far, 'remote')
        else:
            self.far = mk(far)
            self.far_local = self.far_remote = None


def _attend(plan, q, eq, k, v, ek, ev, ov, ot, rk=None, rv=None, lse_v=None, lse_t=None, ctx=None, split_keys=False):
    if plan is None or not plan.segs:
        return
    kp, vp = plan.pack_kv(k, v, ek, ev, rk, rv)
    if ctx is not None and _move_active(ctx):
        rot = _shared_rotation(ctx, plan, kp.device)
        if rot is not None:
            rotate_rows(kp, *rot)
    S.attend_segments(plan, q, eq, kp, vp, ov, ot, lse_v, lse_t, split_keys=split_keys)


class Processor:
    def __init__(self, ctx: Context, layer: int):
        self.ctx, self.layer = ctx, layer

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None, image_rotary_emb=None):
        """hunyuan15.py:177-210: projections, RMSNorm, RoPE on the local rows, bf16, scene / Ulysses attention,
        output projections. `attn` is the diffusers Attention module (to_q/k/v, norm_q/k, add_*_proj, norm_added_*,
        to_out, to_add_out)."""
        ctx = self.ctx
        _unsupported(ctx)
        cos, sin = image_rotary_emb
        ctx._rot_full = image_rotary_emb
        rows = local_rows(ctx)
        if ctx.scene_rope:
            rows = scene_rope_rows(ctx, cos.device)[rows]
        H = attn.heads
        # per-head RMSNorm + rotary embedding of the local rows in one fused kernel (orl_qk_norm_rope)
        q = qk_norm_rope(attn.to_q(hidden_states).to(torch.bfloat16), attn.norm_q.weight, cos[rows], sin[rows], H,
                         attn.norm_q.eps, per_head=True, sin_shift=0)
        k = qk_norm_rope(attn.to_k(hidden_states).to(torch.bfloat16), attn.norm_k.weight, cos[rows], sin[rows], H,
                         attn.norm_k.eps, per_head=True, sin_shift=0)
        v = attn.to_v(hidden_states).unflatten(2, (H, -1))[0].to(torch.bfloat16).contiguous()
        eq, ek, ev = (f(encoder_hidden_states).unflatten(2, (attn.heads, -1))
                      for f in (attn.add_q_proj, attn.add_k_proj, attn.add_v_proj))
        if getattr(attn, 'norm_added_q', None) is not None:
            eq = attn.norm_added_q(eq)
        if getattr(attn, 'norm_added_k', None) is not None:
            ek = attn.norm_added_k(ek)
        eq, ek, ev = (x[0].to(torch.bfloat16).contiguous() for x in (eq, ek, ev))
        if ctx.memory:
            hs, ehs = self.memory(q, k, v, eq, ek, ev)
        elif ctx.run_mode == 'ulysses' or ctx.attn_override is not None:
            hs, ehs = self.ulysses(q, k, v, eq, ek, ev)
        elif ctx.run_mode == 'ring':
            hs, ehs = R.attention(ctx.ring, q, k, v, eq, ek, ev, ctx.text_ranges(), id(ctx.layout.extra))
        else:
            hs, ehs = self.scene(q, k, v, eq, ek, ev)
        hs = attn.to_out[1](attn.to_out[0](hs.flatten(1, 2)[None].to(hidden_states.dtype)))
        ehs = attn.to_add_out(ehs.flatten(1, 2)[None].to(hidden_states.dtype))
        return hs, ehs

    def memory(self, q, k, v, eq, ek, ev):
        """hunyuan15.py:305-333: bounded cross-scene memory (onereel_b200.memory). One GPU or Ulysses: all tokens of
        the local heads, each rank clusters its own heads. K/V gathering: the rank's scene pieces read their scenes
        (split scenes completed from the peers) and every boundary candidate (received from its owner); every rank
        clusters the same candidates, so all agree on the representatives without exchanging them."""
        ctx, T, lay = self.ctx, self.ctx.T, self.ctx.layout
        if ctx._mem is None:
            ctx._mem = MEM.MemoryAttention(MEM.BoundaryMemory(ctx.memory))
        key, counts = (self.layer, ctx.cond()), ctx.counts[ctx.cond()]
        n, r, H = D.world(), D.rank(), q.shape[1]
        eq_full = eq
        rk = rv = None
        if ctx.run_mode == 'ulysses' or n == 1:
            sl = slice(r * H // n, (r + 1) * H // n)
            if n > 1:
                q, k, v = comm.a2a_heads(q), comm.a2a_heads(k), comm.a2a_heads(v)
                eq, ek, ev = (x[:, sl].contiguous() for x in (eq, ek, ev))
            own, remote_index = (0, lay.n_frames * T), []
            scenes = [(j, (lo * T, hi * T)) for j, (lo, hi) in enumerate(lay.ranges)]
            text_for = set(range(lay.n_scenes))
        else:
            sl = slice(None)
            own = tuple(ctx.own[r])
            ex = comm.HaloExchange(lay, ctx.own, T, k, v, extra=MEM.candidate_frames(lay)[0])
            ex.wait()
            remote_index, rk, rv = ex.remote_index, ex.remote_k, ex.remote_v
            scenes, text_for = S.pieces(lay, T, own)
        Hl, Dh = q.shape[1:]
        pk = (_layout_key(lay), T, tuple(counts), own, tuple(map(tuple, remote_index)), Hl, Dh, str(q.device))
        plan = ctx._mem.plans.get(pk)
        if plan is None:
            plan = ctx._mem.plans[pk] = MEM.MemoryPlan.for_rank(lay, T, counts, own, remote_index, scenes, text_for,
                                                                q.device)
        ov = torch.empty_like(q)
        ot = torch.zeros_like(eq)
        ctx._mem.run(key, plan, q, k, v, eq, ek, ev, ov, ot, rk, rv)
        if n == 1:
            return ov, ot
        if sl != slice(None):
            full = torch.zeros_like(eq_full)
            full[:, sl] = ot
            D.all_reduce(full)
            return comm.a2a_tokens(ov), full
        D.all_reduce(ot)
        return ov, ot

    def _plan(self, H, Dh, device, lse_overlap):
        ctx = self.ctx
        key = ('scene', _layout_key(ctx.layout), ctx.T, tuple(ctx.counts[ctx.cond()]), tuple(map(tuple, ctx.own)),
               D.rank(), H, Dh, str(device), lse_overlap)
        plan = ctx._cache.get(key)
        if plan is None:
            plan = ctx._cache[key] = _RankPlan(ctx, H, Dh, device, lse_overlap)
        return plan

    def scene(self, q, k, v, eq, ek, ev):
        """hunyuan15.py:212-251: the scenes of this rank's token range. The exchange is posted first; scenes whose keys
        are all local attend while it is in flight; then the others (or, with overlap='lse', the others attend to
        their local keys during the exchange and to the received keys after it, merged by log-sum-exp). kv_chunks
        does not change the result (attention is per head) and a single exchange is posted on NVLink."""
        ctx = self.ctx
        _unsupported(ctx)
        H, Dh = q.shape[1:]
        lse_overlap = ctx.overlap == 'lse'
        plan = self._plan(H, Dh, q.device, lse_overlap)
        _mark('start')
        ex = comm.kv_exchange(ctx.exchange, ctx.layout, ctx.own, ctx.T, k, v) if D.world() > 1 else None
        if ex is not None and ex.remote_index != plan.remote_index:
            raise RuntimeError('exchange layout differs from the compiled plan')
        _mark('exchange')         # posted (NCCL) or done on this stream (peer memory: copy-in, barrier, pull)
        if _move_active(ctx) and plan.lse:
            raise NotImplementedError("overlap='lse' with shared_pos='adjacent' is not on the B200 path")
        ov, ot = torch.empty_like(q), torch.zeros_like(eq)
        _attend(plan.near, q, eq, k, v, ek, ev, ov, ot, ctx=ctx)
        _mark('near')
        if plan.lse:
            self._far_lse(plan, ex, q, eq, k, v, ek, ev, ov, ot)
        else:
            if ex is not None:
                ex.wait()
            _mark('exchange_wait')
            _attend(plan.far, q, eq, k, v, ek, ev, ov, ot, ex.remote_k if ex else None, ex.remote_v if ex else None,
                    ctx=ctx)
            _mark('far')
        if ctx.text_sync == 'all_reduce' or D.world() == 1:
            D.all_reduce(ot)
        else:
            comm.send_text_rows(ot, ctx.layout, ctx.own, ctx.T, ctx.text_ranges())
        _mark('text_sync')
        return ov, ot

    def _far_lse(self, plan, ex, q, eq, k, v, ek, ev, ov, ot):
        """hunyuan15.py:253-277: far pieces attend to their local keys (and text) while the exchange is in flight, then
        to the received keys; the two partial results are merged by log-sum-exp (orl_lse_merge)"""
        H = q.shape[1]
        lse_v = torch.empty(H, q.shape[0], dtype=torch.float32, device=q.device)
        lse_t = torch.empty(H, eq.shape[0], dtype=torch.float32, device=q.device)
        _attend(plan.far_local, q, eq, k, v, ek, ev, ov, ot, lse_v=lse_v, lse_t=lse_t)
        _mark('far_local')
        if ex is not None:
            ex.wait()
        _mark('exchange_wait')
        fr = plan.far_remote
        if fr is None or not fr.segs:
            return
        o2v, o2t = torch.empty_like(q), torch.empty_like(eq)
        l2v = torch.empty_like(lse_v)
        l2t = torch.empty_like(lse_t)
        _attend(fr, q, eq, k, v, ek, ev, o2v, o2t, ex.remote_k, ex.remote_v, l2v, l2t)
        for s in fr.segs:
            lo, hi = s.q[1], s.q[2]
            if s.kind == 'v':
                A.lse_merge(ov[lo:hi], lse_v[:, lo:hi], o2v[lo:hi], l2v[:, lo:hi])
            else:
                A.lse_merge(ot[lo:hi], lse_t[:, lo:hi], o2t[lo:hi], l2t[:, lo:hi])
        _mark('far_remote')

    def ulysses(self, q, k, v, eq, ek, ev):
        """hunyuan15.py:279-303: heads redistributed by all-to-all; every scene on the local heads; text outputs of the
        local heads all-reduced"""
        ctx = self.ctx
        n, r, H = D.world(), D.rank(), q.shape[1]
        sl = slice(r * H // n, (r + 1) * H // n)
        _mark('start')
        # over peer memory when every rank holds the same number of tokens (the Ulysses split), else NCCL
        sizes = {b - a for a, b in ctx.own} if ctx.own else {q.shape[0]}
        use_peer = (ctx.exchange == 'peer' and n > 1 and len(sizes) == 1 and H % n == 0 and
                    ctx.attn_override is None and comm.PEER_UNAVAILABLE is None)
        if use_peer:
            from onereel_b200 import peer
            try:
                qa, ka, va = peer.a2a_heads_qkv(q, k, v)
            except (RuntimeError, AttributeError, NotImplementedError) as e:
                if peer.initialised():
                    raise
                comm.PEER_UNAVAILABLE = f'{type(e).__name__}: {e}'
                use_peer = False
        if not use_peer:
            qa, ka, va = comm.a2a_heads(q), comm.a2a_heads(k), comm.a2a_heads(v)
        eqs, eks, evs = (x[:, sl].contiguous() for x in (eq, ek, ev))
        _mark('a2a_in')
        if ctx.attn_override is not None:
            res = ctx.attn_override(self.layer, qa, ka, va, eqs, eks, evs)
            if res is not None:
                ot = eq.new_zeros(eq.shape)
                ot[:, sl] = res[1]
                D.all_reduce(ot)
                return comm.a2a_tokens(res[0]), ot
        Hl, Dh = qa.shape[1:]
        lay, T = ctx.layout, ctx.T
        L = lay.n_frames * T
        key = ('ulysses', _layout_key(lay), T, tuple(ctx.counts[ctx.cond()]), Hl, Dh, str(q.device))
        plan = ctx._cache.get(key)
        if plan is None:
            scenes = [(j, (lo * T, hi * T)) for j, (lo, hi) in enumerate(lay.ranges)]
            plan = ctx._cache[key] = S.ScenePlan(
                S.scene_segments(lay, T, ctx.counts[ctx.cond()], scenes, set(range(lay.n_scenes)), (0, L)),
                Hl * Dh * 2, Hl, q.device)
        if use_peer:
            # video and text outputs of this rank's heads in symmetric memory; one barrier, then every rank pulls its
            # tokens of all heads and all heads of the text rows (no all-reduce)
            ov, otl, handle = peer.out_buffer(qa.shape[0], Hl, Dh, qa.dtype, qa.device, eqs.shape[0])
            if otl is not None:
                otl.zero_()
            else:
                otl = torch.zeros_like(eqs)
            _attend(plan, qa, eqs, ka, va, eks, evs, ov, otl, ctx=ctx, split_keys=ctx.split_keys)
            _mark('attention')
            if eqs.shape[0]:
                out, ot = peer.a2a_tokens_from(ov, handle, otl)
            else:
                out, ot = peer.a2a_tokens_from(ov, handle), eq.new_zeros(eq.shape)
            _mark('a2a_out')
            return out, ot
        ov = torch.empty_like(qa)
        otl = torch.zeros_like(eqs)
        _attend(plan, qa, eqs, ka, va, eks, evs, ov, otl, ctx=ctx, split_keys=ctx.split_keys)
        _mark('attention')
        ot = eq.new_zeros(eq.shape)
        ot[:, sl] = otl
        D.all_reduce(ot)
        _mark('text_sync')
        out = comm.a2a_tokens(ov)
        _mark('a2a_out')
        return out, ot


def apply_rotary_emb(x, freqs):
    """real-valued rotary embedding over interleaved pairs (diffusers' apply_rotary_emb with use_real=True,
    use_real_unbind_dim=-1, sequence_dim=1): x [B, S, H, D], cos / sin [S, D]. Torch ops; the processor uses the fused
    orl_qk_norm_rope kernel, this stays for callers that rotate other tensors."""
    cos, sin = (f[None, :, None, :].to(x.device) for f in freqs)
    xr, xi = x.float().unflatten(-1, (-1, 2)).unbind(-1)
    rot = torch.stack([-xi, xr], -1).flatten(-2)
    return (x.float() * cos + rot * sin).to(x.dtype)


def plan_parallel(ctx: Context, heads: int):
    """hunyuan15.py:553-573: the work-balanced partition (Algorithm 1) for K/V gathering, equal ranges for Ulysses;
    'auto' takes the gathering path when Eq. 2 says it moves less (and when Ulysses cannot split frames or heads)"""
    n, lay = D.world(), ctx.layout
    ctx.ring = None
    if n == 1:
        ctx.run_mode, ctx.own, ctx.path = 'scene', [(0, lay.n_frames * ctx.T)], {}
        return
    if ctx.mode == 'ring':                       # baseline: USP's Ring with every scene split evenly over the ranks
        assert not ctx.memory and not ctx.subject_links, 'the ring path runs the halo / frame-memory scene attention'
        ctx.ring = R.RingPlan(lay, n, ctx.T)
        ctx.run_mode, ctx.own = 'ring', ctx.ring.own
        ctx.path = dict(path='ring', V_R=ctx.ring.volume(), V_U=4 * lay.n_frames * ctx.T * (n - 1) / n ** 2)
        return
    _unsupported(ctx)
    gather = comm.partition(lay, n, ctx.T, 'scene', ctx.counts[True], ctx.memory, ctx.partition)
    ctx.path = comm.choose_path(lay, gather, ctx.T, ctx.theta)
    ctx.path['ulysses_ok'] = lay.n_frames * ctx.T % n == 0 and heads % n == 0
    ctx.run_mode = ctx.mode if ctx.mode != 'auto' else ctx.path['path'] if ctx.path['ulysses_ok'] else 'scene'
    assert ctx.run_mode != 'ulysses' or ctx.path['ulysses_ok'], f'Ulysses needs video tokens and heads divisible by {n}'
    ctx.own = gather if ctx.run_mode == 'scene' else comm.partition(lay, n, ctx.T, 'ulysses')
    # a rank planning from a different layout or text would post mismatched exchanges: fail on every rank instead
    D.check_consistent('hunyuan15 parallel plan', (_layout_key(lay), ctx.T, ctx.run_mode, [tuple(o) for o in ctx.own],
                                                   [tuple(ctx.counts.get(c, ())) for c in (True, False)]))


_plan_parallel = plan_parallel      # the reference's private name (hunyuan15.py:553)


def _segments(ctx, scenes, qf, kf, vf, eq, ek, ev, text_for):
    """hunyuan15.py:153-170 on tensors (API compatibility; the processors use the compiled plans instead): packed
    (q, k, v) per scene piece and its meta"""
    lay, tr = ctx.layout, ctx.text_ranges()
    segs, meta = [], []
    for j, (qlo, qhi) in scenes:
        t0, t1 = tr[j]
        keys = lay.key_frames(j)
        segs.append((qf(qlo, qhi), torch.cat([kf(keys), ek[t0:t1]]), torch.cat([vf(keys), ev[t0:t1]])))
        meta.append(('v', j, qlo, qhi))
        if j in text_for:
            fr = lay.frames[j]
            segs.append((eq[t0:t1], torch.cat([kf(fr), ek[t0:t1]]), torch.cat([vf(fr), ev[t0:t1]])))
            meta.append(('t', j, t0, t1))
    return segs, meta


def local_rows(ctx):
    """hunyuan15.py:457-460: this rank's video rows — a token slice, or the ring's permuted rows"""
    a, b = ctx.own[D.rank()]
    return ctx.ring.perm[a:b] if ctx.run_mode == 'ring' else slice(a, b)


def gather_rows(ctx, x):
    """hunyuan15.py:463-466: [B, local rows, C] -> [B, all tokens, C] in token order"""
    x = comm.gather_tokens(x, ctx.own)
    return x[:, ctx.ring.inv] if ctx.run_mode == 'ring' and D.world() > 1 else x


def install_attention(transformer, ctx: Context):
    """the attention part of hunyuan15.install (407-440, _observe 469-495): a Processor on every block; the forward
    counter and the frame-memory step / layer / pooling hooks; the token shard / gather hooks of the first / last block
    when parallel. `transformer` is the diffusers HunyuanVideo15Transformer3DModel (or any module with
    .transformer_blocks[i].attn.set_processor); blocks return (hidden states, text states)."""
    if ctx.memory:
        assert ctx.layout.halo == 0, 'the bounded memory replaces the halo frames: use halo = 0'
        assert not ctx.subject_links, 'the bounded memory and subject links are separate variants'
        ctx._mem = MEM.MemoryAttention(MEM.BoundaryMemory(ctx.memory))
    if ctx.frame_memory is not None:
        assert ctx.layout.halo == 0 and not ctx.memory, 'frame memory replaces the halo frames: use halo = 0'
    for i, blk in enumerate(transformer.transformer_blocks):
        blk.attn.set_processor(Processor(ctx, i))

    def pre(m, args, kw):
        ctx.fwd += 1
        if ctx.frame_memory is not None:
            ctx.frame_memory.begin_step(ctx.step())

    def post(m, args, kw, out):
        if ctx.frame_memory is not None and ctx.cond():
            ctx.frame_memory.finish()
    transformer.register_forward_pre_hook(pre, with_kwargs=True)
    transformer.register_forward_hook(post, with_kwargs=True)
    frame_of_row = {}

    def hooks(i):
        def block_pre(m, args):
            if ctx.frame_memory is not None:
                ctx.frame_memory.use_layer(i)

        def block_post(m, args, out):
            fm = ctx.frame_memory
            if fm is None or not fm.observes(i) or not ctx.cond():
                return
            hs = out[0][0]
            key = (tuple(ctx.own[D.rank()]), ctx.run_mode)
            if key not in frame_of_row:
                frame_of_row.clear()
                a, b = ctx.own[D.rank()]
                rows = ctx.ring.perm[a:b] if ctx.run_mode == 'ring' else torch.arange(a, b, device=hs.device)
                frame_of_row[key] = rows.to(hs.device) // ctx.T
            fm.collect(frame_of_row[key], hs, i)
        return block_pre, block_post
    for i, blk in enumerate(transformer.transformer_blocks):
        bp, bq = hooks(i)
        blk.register_forward_pre_hook(bp)
        blk.register_forward_hook(bq)
    if D.world() > 1:
        def shard(m, args):
            return (args[0][:, local_rows(ctx)],) + tuple(args[1:])

        def gather(m, args, out):
            return gather_rows(ctx, out[0]), out[1]
        transformer.transformer_blocks[0].register_forward_pre_hook(shard)
        transformer.transformer_blocks[-1].register_forward_hook(gather)
