"""The C-ABI library on the CPU: it loads, exports every symbol include/onereel_b200.h declares, and its host-only
entry points (work planning, pack preparation, error strings) behave; the product's segment builder against the
oracle and the reference's golden segment order. No kernel is launched."""
import json
import re
from pathlib import Path

import numpy as np
import pytest

from oracle import layout_oracle as LO

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope='module')
def lib():
    from onereel_b200.csrc.build import build
    build()
    from onereel_b200 import _lib
    return _lib


def declared_symbols():
    text = (ROOT / 'include' / 'onereel_b200.h').read_text()
    return set(re.findall(r'ORL_API[^;(]*?\b(orl_\w+)\s*\(', text))


def test_exports_every_declared_symbol(lib):
    import subprocess
    names = declared_symbols()
    assert {'orl_attn_fwd', 'orl_attn_plan', 'orl_pack', 'orl_lse_merge'} <= names
    nm = subprocess.run(['nm', '-D', '--defined-only', str(lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r'\bT (orl_\w+)', nm))
    assert names <= exported, names - exported
    assert set(lib.SIGNATURES) == names          # the ctypes binding covers exactly the header
    h = lib.lib()
    for n in names:
        getattr(h, n)
    assert b'sm_100a' in h.orl_version()
    assert h.orl_error_string(-2).decode().startswith('pointer')


def test_attn_plan_items(lib):
    h = lib.lib()
    cu_q = np.array([0, 300, 300, 557], np.int32)
    cu_k = np.array([0, 10, 5000, 5001], np.int32)
    need = h.orl_attn_plan(lib.i32p(cu_q), lib.i32p(cu_k), 3, 2, None, 0)
    assert need == -(2 * 2 + 2 * 2) - 1000           # segment 1 has no queries
    work = np.zeros(8, dtype=lib.WORK_DTYPE)
    n = h.orl_attn_plan(lib.i32p(cu_q), lib.i32p(cu_k), 3, 2, work.ctypes.data, 8)
    assert n == 8
    # largest key range first: segment 2 (1 key) before... no: segment 0 (10 keys) before segment 2 (1 key)
    assert work['seg'].tolist() == [0, 0, 0, 0, 2, 2, 2, 2]
    assert work['head'].tolist() == [0, 0, 1, 1, 0, 0, 1, 1]
    assert work['q_row0'].tolist() == [0, 256, 0, 256, 300, 556, 300, 556]
    assert work['q_len'].tolist() == [256, 44, 256, 44, 256, 1, 256, 1]
    assert work['k_row0'].tolist() == [0] * 4 + [5000] * 4 and work['k_len'].tolist() == [10] * 4 + [1] * 4
    bad = np.array([0, 5, 3], np.int32)
    assert h.orl_attn_plan(lib.i32p(bad), lib.i32p(cu_k[:3]), 2, 1, work.ctypes.data, 8) == -1


def test_pack_prepare(lib):
    h = lib.lib()
    runs = np.zeros(3, dtype=lib.RUN_DTYPE)
    runs['src_off'] = [0, 4096, 32]
    nb = np.array([256, 0, 48], np.int64)
    assert h.orl_pack_prepare(runs.ctypes.data, lib.i64p(nb), 3) == 19
    assert runs['vec0'].tolist() == [0, 16, 16]
    nb[2] = 40
    assert h.orl_pack_prepare(runs.ctypes.data, lib.i64p(nb), 3) == -2


def test_scene_plan_matches_golden_segment_order():
    """onereel_b200.scene (the product's layout builder) reproduces the reference's packed calls (world 1)"""
    from onereel_b200 import scene as S
    from onereel_b200.layout import SceneLayout
    cases = json.loads((ROOT / 'tests' / 'golden' / 'segments.json').read_text())
    checked = 0
    for c in cases:
        if c['model'] != 'hunyuan' or c['n'] != 1:
            continue
        lay = SceneLayout(c['lengths'], c['halo'], c['sides'], {int(j): v for j, v in c['extra'].items()})
        T, counts = c['T'], c['counts']
        L = lay.n_frames * T
        mine = [(j, (lo * T, hi * T)) for j, (lo, hi) in enumerate(lay.ranges)]
        segs = S.scene_segments(lay, T, counts, mine, set(range(lay.n_scenes)), (0, L))
        (call,) = c['calls']
        kind = {S.VIDEO: 'v', S.TEXT: 't'}
        assert [[[kind[s.q[0]], s.q[1], s.q[2]]] for s in segs] == call['q']
        assert [[[kind[x], lo, hi] for x, lo, hi in s.kv] for s in segs] == call['k']
        assert np.concatenate([[0], np.cumsum([s.lq for s in segs])]).tolist() == call['cu_q']
        assert np.concatenate([[0], np.cumsum([s.lk for s in segs])]).tolist() == call['cu_k']
        checked += 1
    assert checked >= 40


def test_layout_api_matches_golden():
    from onereel_b200.layout import SceneLayout
    data = json.loads((ROOT / 'tests' / 'golden' / 'layout.json').read_text())
    for c in data['cases']:
        lay = SceneLayout(c['lengths'], c['halo'], c['sides'], {int(j): v for j, v in c['extra'].items()})
        for j in range(lay.n_scenes):
            assert lay.halo_frames(j) == c['halo_frames'][j]
            assert lay.shared_frames(j) == c['shared_frames'][j]
            assert lay.key_frames(j) == c['key_frames'][j]
            assert list(lay.key_range(j)) == c['key_range'][j]
    for e in data['even']:
        assert SceneLayout.even(e['n_frames'], e['n_scenes']).lengths == e['lengths']


def test_comm_abi_rejects_bad_arguments_without_a_gpu():
    """the NCCL wrappers validate their arguments before touching NCCL or CUDA"""
    import ctypes
    from onereel_b200 import _lib as L
    lib = L.lib()
    assert lib.orl_comm_exchange(None, None, 0, None, 0, None) == -1
    assert lib.orl_comm_broadcast(None, None, 0, 0, None) == -1
    assert lib.orl_comm_all_to_all(None, None, None, 0, None) == -1
    assert lib.orl_comm_all_reduce_f32(None, None, 0, None) == -1
    assert lib.orl_comm_wait(None, None, 0) == -1
    assert lib.orl_comm_destroy(None) == -1
    h = ctypes.c_void_p()
    assert lib.orl_comm_init(ctypes.byref(h), None, 2, 0, 0) == -1          # no id
    assert lib.orl_comm_unique_id(None) == -1
    assert lib.orl_error_string(-8) == b'NCCL error (communicator aborted after a failed wait)'
    assert lib.orl_error_string(-9) == b'collective wait timed out (communicator aborted)'
