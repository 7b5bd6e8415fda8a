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
