"""Failure detection on the GPU without a fault: a bounded wait that runs out ends its kernel with an error status the
host reads, and the context stays usable (B200 only). No trap, no bad address, no endless loop."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_with_status_and_context_survives():
    if not torch.cuda.is_available():
        pytest.skip('needs a B200')
    from onereel_b200.csrc.build import build
    build()
    from onereel_b200 import _lib, attention as A
    status = torch.full((1,), -1, dtype=torch.int32, device='cuda')
    rc = _lib.lib().orl_selftest_timeout(status.data_ptr(), 20_000_000, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert status.item() != 0 and 'softmax' in _lib.describe_error_bits(status.item())
    # the context is intact: a regular attention call afterwards runs and reports no error
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(300, 2, 64, generator=g).cuda().bfloat16() for _ in range(3))
    o = A.varlen(q, k, v, [0, 300], [0, 300], 300, 300)
    torch.cuda.synchronize()
    A.check()
    ref = torch.nn.functional.scaled_dot_product_attention(*(x.float().transpose(0, 1)[None] for x in (q, k, v)))
    assert (o.float() - ref[0].transpose(0, 1)).abs().max().item() < 2e-2
    assert _lib.lib().orl_selftest_timeout(status.data_ptr(), 0, None) == -1          # invalid limit rejected


def test_peer_barrier_times_out_when_a_peer_never_arrives():
    """the device barrier of the peer-memory exchange, with two signal pads on this one GPU standing for a rank and a
    peer that never signals: the wait runs out after its limit, sets its error bit, and the context stays usable; a
    barrier whose other slot is already signalled passes"""
    if not torch.cuda.is_available():
        pytest.skip('needs a B200')
    from onereel_b200.csrc.build import build
    build()
    from onereel_b200 import _lib
    pads = torch.zeros(2, 2, dtype=torch.int32, device='cuda')          # pads[p]: rank p's pad of world 2
    err = torch.zeros(1, dtype=torch.int32, device='cuda')
    ptrs = (ctypes.c_void_p * 2)(pads[0].data_ptr(), pads[1].data_ptr())
    s = torch.cuda.current_stream().cuda_stream
    assert _lib.lib().orl_peer_barrier(ptrs, 2, 0, 1, 20_000_000, err.data_ptr(), s) == 0
    torch.cuda.synchronize()
    assert err.item() != 0 and 'barrier' in _lib.describe_error_bits(err.item())
    assert pads[1, 0].item() == 1 and pads[0, 0].item() == 1            # rank 0 signalled every pad
    err.zero_()
    pads[0, 1] = 2                                                       # the peer's signal for epoch 2 is there
    assert _lib.lib().orl_peer_barrier(ptrs, 2, 0, 2, 20_000_000, err.data_ptr(), s) == 0
    torch.cuda.synchronize()
    assert err.item() == 0
    assert _lib.lib().orl_peer_barrier(ptrs, 2, 2, 3, 20_000_000, err.data_ptr(), s) == -1   # rank outside world
