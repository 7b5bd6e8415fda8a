"""ctypes binding of libonereel_b200.so (the C ABI declared in include/onereel_b200.h).

The library is built in-tree (onereel_b200/csrc/build.py). Loading fails loudly when it is missing: the product has no
CPU or library fallback.
"""
from __future__ import annotations

import ctypes
from pathlib import Path as _FsPath

import numpy as np

LIB_PATH = _FsPath(__file__).resolve().parent / 'libonereel_b200.so'

c_int, c_ll, c_float, c_vp = ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_void_p
P_I32 = ctypes.POINTER(ctypes.c_int32)
P_I64 = ctypes.POINTER(ctypes.c_int64)


class AttnWork(ctypes.Structure):
    """orl_attn_work"""
    _fields_ = [(n, ctypes.c_int32) for n in ('q_row0', 'q_len', 'k_row0', 'k_len', 'head', 'seg', 'pad0', 'pad1')]


class CopyRun(ctypes.Structure):
    """orl_copy_run"""
    _fields_ = [('src_slot', ctypes.c_int32), ('dst_slot', ctypes.c_int32), ('src_off', ctypes.c_int64),
                ('dst_off', ctypes.c_int64), ('vec0', ctypes.c_int64)]


class Layout(ctypes.Structure):
    """orl_layout"""
    _fields_ = [('lengths', P_I32), ('n_scenes', ctypes.c_int32), ('halo', ctypes.c_int32), ('sides', ctypes.c_int32),
                ('extra_offsets', P_I32), ('extra_frames', P_I32)]


class P2P(ctypes.Structure):
    """orl_p2p: one send or receive of orl_comm_exchange"""
    _fields_ = [('peer', ctypes.c_int32), ('pad', ctypes.c_int32), ('ptr', ctypes.c_void_p), ('bytes', ctypes.c_longlong)]


class Path(ctypes.Structure):
    """orl_path"""
    _fields_ = [('remote_rows', ctypes.c_longlong), ('V_G', ctypes.c_double), ('V_U', ctypes.c_double),
                ('gather', ctypes.c_int32)]


# numpy views of the same layouts (for building tables without Python loops over ctypes objects)
WORK_DTYPE = np.dtype([(n, np.int32) for n, _ in AttnWork._fields_])
RUN_DTYPE = np.dtype([('src_slot', np.int32), ('dst_slot', np.int32), ('src_off', np.int64), ('dst_off', np.int64),
                      ('vec0', np.int64)])
assert WORK_DTYPE.itemsize == ctypes.sizeof(AttnWork) == 32 and RUN_DTYPE.itemsize == ctypes.sizeof(CopyRun) == 32

# name -> (restype, argtypes); every symbol include/onereel_b200.h declares
SIGNATURES = {
    'orl_version': (ctypes.c_char_p, []),
    'orl_error_string': (ctypes.c_char_p, [c_int]),
    'orl_error_bits_describe': (c_int, [c_int, ctypes.c_char_p, c_int]),
    'orl_selftest_timeout': (c_int, [c_vp, ctypes.c_ulonglong, c_vp]),
    'orl_attn_plan': (c_int, [P_I32, P_I32, c_int, c_int, c_vp, c_int]),
    'orl_attn_plan_ranges': (c_int, [P_I32, P_I32, P_I32, P_I32, c_int, c_int, c_vp, c_int]),
    'orl_attn_fwd': (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_ll, c_ll, c_int, c_int, c_float, c_vp, c_int, c_vp,
                             c_vp]),
    'orl_attn_fwd_cu': (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_ll, c_ll, c_int, c_int, c_float, c_vp, c_vp, c_int,
                                c_vp, c_ll, c_vp, c_vp]),
    'orl_attn_fwd_cu_capacity': (c_ll, [c_ll, c_int, c_int]),
    'orl_attn_fwd_noalloc': (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_ll, c_ll, c_int, c_int, c_float, P_I32, P_I32,
                                     c_int, c_vp, c_vp]),
    'orl_pack_prepare': (c_ll, [c_vp, P_I64, c_int]),
    'orl_pack': (c_int, [c_vp, c_int, c_ll, c_int, c_int, c_vp, c_vp, c_vp, c_int, c_vp, c_vp, c_vp]),
    'orl_peer_barrier': (c_int, [ctypes.POINTER(c_vp), c_int, c_int, c_int, ctypes.c_ulonglong, c_vp, c_vp]),
    'orl_peer_gather': (c_int, [ctypes.POINTER(c_vp), ctypes.POINTER(c_vp), c_int, c_int, c_ll, c_ll, c_ll, c_ll, c_ll,
                                c_ll, c_vp]),
    'orl_lse_merge': (c_int, [c_vp, c_vp, c_vp, c_vp, c_ll, c_ll, c_ll, c_int, c_int, c_vp]),
    'orl_lse_merge_acc': (c_int, [c_vp, c_vp, c_vp, c_vp, c_ll, c_ll, c_ll, c_int, c_int, c_vp]),
    'orl_qk_norm_rope': (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_ll, c_int, c_int, c_int, c_float, c_int, c_ll, c_vp,
                                 c_vp]),
    'orl_rope_rows': (c_int, [c_vp, c_vp, c_ll, c_int, c_int, c_vp, c_vp, c_ll, c_int, c_vp]),
    'orl_frame_pool': (c_int, [c_vp, c_int, c_ll, c_int, c_vp, c_vp, c_int, c_vp, c_ll, c_vp]),
    'orl_frame_select_scratch': (c_ll, [c_int, c_int, c_int]),
    'orl_frame_select': (c_int, [c_vp, c_ll, c_ll, c_int, c_int, c_int, c_vp, c_int, c_int, c_int, c_vp, c_ll, c_vp,
                                 c_vp]),
    'orl_key_frames': (c_int, [c_vp, c_int, P_I32, c_int]),
    'orl_query_cost': (c_int, [c_vp, c_ll, P_I32, c_ll, ctypes.POINTER(ctypes.c_double)]),
    'orl_balanced': (c_int, [P_I64, ctypes.POINTER(ctypes.c_double), c_int, c_int, P_I64]),
    'orl_partition': (c_int, [c_vp, c_ll, c_int, c_int, P_I32, c_ll, c_int, P_I64]),
    'orl_needed': (c_int, [c_vp, c_ll, c_ll, c_ll, P_I32, c_int, P_I64, c_int]),
    'orl_choose_path': (c_int, [c_vp, c_ll, P_I64, c_int, ctypes.c_double, P_I32, c_int, c_vp]),
    'orl_comm_available': (c_int, []),
    'orl_comm_unique_id': (c_int, [c_vp]),
    'orl_comm_init': (c_int, [ctypes.POINTER(c_vp), c_vp, c_int, c_int, c_int]),
    'orl_comm_destroy': (c_int, [c_vp]),
    'orl_comm_exchange': (c_int, [c_vp, c_vp, c_int, c_vp, c_int, c_vp]),
    'orl_comm_broadcast': (c_int, [c_vp, c_vp, c_ll, c_int, c_vp]),
    'orl_comm_all_to_all': (c_int, [c_vp, c_vp, c_vp, c_ll, c_vp]),
    'orl_comm_all_reduce_f32': (c_int, [c_vp, c_vp, c_ll, c_vp]),
    'orl_comm_wait': (c_int, [c_vp, c_vp, ctypes.c_ulonglong]),
}

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f'{LIB_PATH} is missing: build it with `python -m onereel_b200.csrc.build` '
                               '(the B200 path has no fallback)')
        h = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype, fn.argtypes = res, args
        _lib = h
    return _lib


class OrlError(RuntimeError):
    pass


def check(rc: int, what: str = '') -> int:
    if rc < 0:
        raise OrlError(f'{what}: {lib().orl_error_string(rc).decode()} ({rc})')
    return rc


def describe_error_bits(bits: int) -> str:
    buf = ctypes.create_string_buffer(512)
    lib().orl_error_bits_describe(bits, buf, 512)
    return buf.value.decode()


def i32p(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(P_I32)


def i64p(a: np.ndarray):
    assert a.dtype == np.int64 and a.flags.c_contiguous
    return a.ctypes.data_as(P_I64)
