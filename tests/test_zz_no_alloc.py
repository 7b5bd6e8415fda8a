"""The allocation-free entry point orl_attn_fwd_noalloc, called through the C ABI, against the regular entry point.

Some callers cannot call cudaMalloc — code running inside another framework's memory pool or allocator hook, or a
plugin host that owns all device memory — so they cannot hand orl_attn_fwd its scratch (work list and error word).
orl_attn_fwd_noalloc keeps that scratch in a fixed array inside the library instead. This test calls it twice in a row
with different shapes (the second call must not see the first call's work list or error word) and checks each output
against orl_attn_fwd on the same inputs, within the tolerance the other GPU tests use. It also checks that a call
larger than the array's capacity is rejected before any work. This file sorts last so that a stop-at-first-failure
run has already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.gpu_ref import MAX_ABS, MEAN_ABS

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def lib():
    if not torch.cuda.is_available():
        pytest.skip('needs a B200')
    from onereel_b200.csrc.build import build
    build()
    from onereel_b200 import _lib
    return _lib


def rand(*shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to('cuda', torch.bfloat16)


def call_noalloc(lib, q, k, v, cu_q, cu_k, with_lse):
    Nq, H, Dh = q.shape
    out = torch.empty_like(q)
    lse = torch.empty(H, Nq, dtype=torch.float32, device='cuda') if with_lse else None
    status = ctypes.c_int(-1)
    cq, ck = np.ascontiguousarray(cu_q, np.int32), np.ascontiguousarray(cu_k, np.int32)
    rc = lib.lib().orl_attn_fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        None if lse is None else lse.data_ptr(), Nq, k.shape[0], H, Dh, Dh ** -0.5,
                                        lib.i32p(cq), lib.i32p(ck), len(cq) - 1, ctypes.byref(status),
                                        torch.cuda.current_stream().cuda_stream)
    return rc, status.value, out, lse


def regular(q, k, v, cu_q, cu_k):
    from onereel_b200 import attention as A
    o, l = A.varlen_lse(q, k, v, list(cu_q), list(cu_k), None, None)
    torch.cuda.synchronize()
    A.check()
    return o, l


def test_noalloc_matches_regular_entry_point_twice(lib):
    cases = [
        # (segments (q rows, k rows), heads, head_dim, with_lse)
        ([(300, 1000), (16, 336), (129, 77), (1, 1)], 4, 128, True),
        ([(64, 64), (700, 130), (255, 2049)], 2, 64, False),
    ]
    for i, (segs, H, Dh, with_lse) in enumerate(cases):
        lq, lk = [a for a, _ in segs], [b for _, b in segs]
        cu_q, cu_k = np.concatenate([[0], np.cumsum(lq)]), np.concatenate([[0], np.cumsum(lk)])
        q, k, v = rand(sum(lq), H, Dh, seed=10 * i), rand(sum(lk), H, Dh, seed=10 * i + 1), rand(sum(lk), H, Dh, seed=10 * i + 2)
        rc, status, out, lse = call_noalloc(lib, q, k, v, cu_q, cu_k, with_lse)
        assert rc == 0, lib.lib().orl_error_string(rc)
        assert status == 0, lib.describe_error_bits(status)
        want, want_lse = regular(q, k, v, cu_q, cu_k)
        d = (out.float() - want.float()).abs()
        assert d.max().item() <= MAX_ABS and d.mean().item() <= MEAN_ABS, (i, d.max().item())
        if with_lse:
            assert (lse - want_lse).abs().max().item() < 1e-3


def test_noalloc_rejects_oversized_calls(lib):
    q = rand(16, 1, 64, seed=0)
    # one segment needing 16385 work items (heads x ceil(rows / 256)) exceeds the scratch array: rejected up front
    cu_q = np.array([0, 16385 * 256], np.int32)
    cu_k = np.array([0, 16], np.int32)
    out = torch.empty_like(q)
    st = ctypes.c_int(-1)
    rc = lib.lib().orl_attn_fwd_noalloc(q.data_ptr(), q.data_ptr(), q.data_ptr(), out.data_ptr(), None, 16385 * 256, 16,
                                        1, 64, 0.125, lib.i32p(cu_q), lib.i32p(cu_k), 1, ctypes.byref(st),
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == -7 and st.value == -1          # ORL_ERR_CAPACITY, nothing ran
    many = np.arange(4098, dtype=np.int32)      # 4097 segments > 4096
    rc = lib.lib().orl_attn_fwd_noalloc(q.data_ptr(), q.data_ptr(), q.data_ptr(), out.data_ptr(), None, 16, 16, 1, 64,
                                        0.125, lib.i32p(many), lib.i32p(many), 4097, None,
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == -7
