"""shared_pos = 'adjacent' (HunyuanVideo-1.5) on the CPU — the checks of the reference's tests/test_shared_pos.py: a
shared frame's key rotated at its own frame and moved by _move_shared equals the same key rotated at its adjacent
position (3-D RoPE table with temporal, height and width frequencies on separate groups of interleaved pairs), with
frame-index RoPE and with scene-local RoPE; and the per-segment tables the processors hand to the orl_rope_rows kernel
are the same composed rotations."""
import torch

from onereel_b200 import hunyuan15 as HY
from onereel_b200.layout import SceneLayout


def _table(F, Hh, Ww):
    f, y, x = torch.meshgrid(torch.arange(F), torch.arange(Hh), torch.arange(Ww), indexing='ij')
    parts = []
    for pos, n in ((f, 16), (y, 24), (x, 24)):                      # pairs per axis: 16 + 24 + 24 = 64 = D / 2
        parts.append(pos.reshape(-1, 1).double() * (1e4 ** (-torch.arange(n).double() / n)))
    ang = torch.cat(parts, 1)
    return ang.cos().float().repeat_interleave(2, 1), ang.sin().float().repeat_interleave(2, 1)


F, Hh, Ww, D, H = 30, 4, 6, 128, 2
T = Hh * Ww
COS, SIN = _table(F, Hh, Ww)


def _layout():
    lay = SceneLayout([8, 7, 9, 6], halo=0)
    lay.extra = {0: [12, 20, 27], 1: [2, 20, 27], 2: [2, 12, 27], 3: [2, 12, 20]}
    return lay


def _rot(k, rows):
    return HY.apply_rotary_emb(k[None], (COS[rows], SIN[rows]))[0]


def _tokens(frames):
    return torch.cat([torch.arange(f * T, (f + 1) * T) for f in frames])


def test_move_shared_equals_rotation_at_adjacent_position():
    lay = _layout()
    ctx = HY.Context(lay, T=T, shared_pos='adjacent')
    ctx._rot_full = (COS, SIN)
    g = torch.Generator().manual_seed(0)
    for j in range(lay.n_scenes):
        frames = lay.key_frames(j)
        k0 = torch.randn(len(frames) * T, H, D, generator=g)
        dst = lay.frames[j] + HY.adjacent_positions(lay, j)
        moved = HY._move_shared(ctx, j, _rot(k0, _tokens(frames)))
        assert (moved - _rot(k0, _tokens(dst))).abs().max().item() < 1e-4, j


def test_move_shared_with_scene_local_rope():
    lay = _layout()
    ctx = HY.Context(lay, T=T, shared_pos='adjacent', scene_rope=True)
    ctx._rot_full = (COS, SIN)
    g = torch.Generator().manual_seed(1)
    for j in range(lay.n_scenes):
        frames = lay.key_frames(j)
        k0 = torch.randn(len(frames) * T, H, D, generator=g)
        src = [HY.frame_position(ctx, f) for f in frames]
        dst = [HY.frame_position(ctx, f) for f in lay.frames[j]] + HY.shared_positions(ctx, j)
        moved = HY._move_shared(ctx, j, _rot(k0, _tokens(src)))
        assert (moved - _rot(k0, _tokens(dst))).abs().max().item() < 1e-4, j


def test_processor_tables_are_the_composed_rotations():
    """_shared_rotation (the rows and tables orl_rope_rows applies inside the packed K) against _move_shared's"""
    lay = _layout()
    counts = [3, 3, 3, 3]
    ctx = HY.Context(lay, T=T, counts={True: counts}, fwd=1, own=[(0, lay.n_frames * T)], shared_pos='adjacent')
    ctx._rot_full = (COS, SIN)
    scenes = [(j, (lo * T, hi * T)) for j, (lo, hi) in enumerate(lay.ranges)]
    plan = HY.S.ScenePlan(HY.S.scene_segments(lay, T, counts, scenes, set(range(4)), (0, lay.n_frames * T)),
                          H * D * 2, H, 'cpu')
    rows, cos_d, sin_d = HY._shared_rotation(ctx, plan, 'cpu')
    at = 0
    for i, sg in enumerate(plan.segs):
        if sg.kind != 'v':
            continue
        n_sh = len(lay.shared_frames(sg.scene)) * T
        base = plan.cu_k[i] + len(lay.frames[sg.scene]) * T
        assert rows[at:at + n_sh].tolist() == list(range(base, base + n_sh))
        ar, br = HY._shift_rows(ctx, sg.scene)
        ca, sa, cb, sb = COS[ar], SIN[ar], COS[br], SIN[br]
        assert torch.equal(cos_d[at:at + n_sh], cb * ca + sb * sa)
        assert torch.equal(sin_d[at:at + n_sh], sb * ca - cb * sa)
        at += n_sh
    assert at == len(rows)
