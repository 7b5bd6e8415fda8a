"""The allocation-free entry point orl_attn_fwd_noalloc, called through the C ABI, against the regular entry point.

Some callers cannot call cudaMalloc — code running inside another framework's memory pool or allocator hook, or a
plugin host that owns all device memory — so they cannot hand orl_attn_fwd its scratch (work list and error word).
orl_attn_fwd_noalloc keeps that scratch in a fixed array inside the library instead. This test calls it twice in a row
with different shapes (the second call must not see the first call's work list or error word) and checks each output
and LSE for bitwise equality with orl_attn_fwd on the same inputs (the same kernel over the same schedule), and the
output against an fp32 reference within the tolerance the other GPU tests use. The shapes include segments without
query rows and without keys; an empty call must still report status 0. Calls beyond the array's capacity are
rejected before any work; their tensors are allocated at the sizes the call states. This file sorts last so that a
stop-at-first-failure run has already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.gpu_ref import MAX_ABS, MEAN_ABS, compare, ref_attention

pytestmark = pytest.mark.gpu

ORL_ERR_CAPACITY = -7


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


def call_noalloc(lib, q, k, v, cu_q, cu_k, with_lse, out=None):
    Nq, H, Dh = q.shape
    out = torch.zeros_like(q) if out is None else out
    lse = torch.zeros(H, Nq, dtype=torch.float32, device='cuda') if with_lse else None
    status = ctypes.c_int(-1)
    cq, ck = np.ascontiguousarray(cu_q, np.int32), np.ascontiguousarray(cu_k, np.int32)
    rc = lib.lib().orl_attn_fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        None if lse is None else lse.data_ptr(), Nq, k.shape[0], H, Dh, Dh ** -0.5,
                                        lib.i32p(cq), lib.i32p(ck), len(cq) - 1, ctypes.byref(status),
                                        torch.cuda.current_stream().cuda_stream)
    return rc, status.value, out, lse


def regular(q, k, v, cu_q, cu_k):
    """orl_attn_fwd through the package's varlen_lse (zero-initialised output and LSE, as the no-alloc call gets)"""
    from onereel_b200 import attention as A
    cq, ck = [int(x) for x in cu_q], [int(x) for x in cu_k]
    ql = [b - a for a, b in zip(cq[:-1], cq[1:])]
    kl = [b - a for a, b in zip(ck[:-1], ck[1:])]
    out = torch.zeros_like(q)
    lse = torch.zeros(q.shape[1], q.shape[0], dtype=torch.float32, device='cuda')
    A.attend(q, k, v, cq[:-1], ql, ck[:-1], kl, out=out, lse=lse)
    torch.cuda.synchronize()
    A.check()
    return out, lse, cq[:-1], ql, ck[:-1], kl


CASES = [
    # (segments (q rows, k rows), heads, head_dim, with_lse): a segment without query rows (0, 64) and one without
    # keys (40, 0) among ordinary ones
    ([(300, 1000), (0, 64), (16, 336), (129, 77), (40, 0), (1, 1)], 4, 128, True),
    ([(64, 64), (700, 130), (255, 2049)], 2, 64, False),
]


def test_noalloc_matches_regular_entry_point_twice(lib):
    for i, (segs, H, Dh, with_lse) in enumerate(CASES):
        lq, lk = [a for a, _ in segs], [b for _, b in segs]
        cu_q, cu_k = np.concatenate([[0], np.cumsum(lq)]), np.concatenate([[0], np.cumsum(lk)])
        q, k, v = (rand(sum(lq), H, Dh, seed=10 * i), rand(sum(lk), H, Dh, seed=10 * i + 1),
                   rand(sum(lk), H, Dh, seed=10 * i + 2))
        rc, status, out, lse = call_noalloc(lib, q, k, v, cu_q, cu_k, with_lse)
        assert rc == 0, lib.lib().orl_error_string(rc)
        assert status == 0, lib.describe_error_bits(status)
        want, want_lse, qs, ql, ks, kl = regular(q, k, v, cu_q, cu_k)
        assert torch.equal(out, want), i
        if with_lse:
            assert torch.equal(lse, want_lse), i
        ref = ref_attention(q, k, v, qs, ql, ks, kl)
        mx, mean, lmx = compare(out, lse, ref, qs)
        assert mx < MAX_ABS and mean < MEAN_ABS, (i, mx, mean)
        if with_lse:
            assert lmx < 1e-3, (i, lmx)


def test_noalloc_empty_call_reports_ok(lib):
    q = rand(16, 1, 64, seed=3)
    cu = np.zeros(1, np.int32)
    rc, status, out, _ = call_noalloc(lib, q, q, q, cu, cu, False)
    assert rc == 0 and status == 0
    assert torch.count_nonzero(out).item() == 0


def test_noalloc_rejects_oversized_calls(lib):
    stream = torch.cuda.current_stream().cuda_stream
    # 1024 one-row segments x 17 heads = 17408 work items > 16384: rejected before any work (tensors sized truthfully)
    n, H = 1024, 17
    q = rand(n, H, 64, seed=0)
    out = torch.zeros_like(q)
    cu = np.arange(n + 1, dtype=np.int32)
    st = ctypes.c_int(-1)
    rc = lib.lib().orl_attn_fwd_noalloc(q.data_ptr(), q.data_ptr(), q.data_ptr(), out.data_ptr(), None, n, n, H, 64,
                                        0.125, lib.i32p(cu), lib.i32p(cu), n, ctypes.byref(st), stream)
    assert rc == ORL_ERR_CAPACITY and st.value == -1          # nothing ran, status untouched
    # 1025 segments > 1024
    n = 1025
    q = rand(n, 1, 64, seed=1)
    out = torch.zeros_like(q)
    cu = np.arange(n + 1, dtype=np.int32)
    rc = lib.lib().orl_attn_fwd_noalloc(q.data_ptr(), q.data_ptr(), q.data_ptr(), out.data_ptr(), None, n, n, 1, 64,
                                        0.125, lib.i32p(cu), lib.i32p(cu), n, None, stream)
    assert rc == ORL_ERR_CAPACITY
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0
