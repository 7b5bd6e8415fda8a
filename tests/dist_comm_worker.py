"""Multi-GPU worker for the C ABI's NCCL collectives (orl_comm_*, through onereel_b200.collectives.NcclComm), run by
tests/test_gpu_dist.py under torchrun: point-to-point exchange, broadcast, all-to-all and all-reduce against
torch.distributed on the same data, the timeout-aware wait on completed work, and the K/V exchange of a scene layout
(HaloExchange) through the C ABI equal to the torch.distributed one row for row. Prints PASS on rank 0."""
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from onereel_b200 import comm, dist as D                       # noqa: E402
from onereel_b200.collectives import NcclComm                 # noqa: E402
from onereel_b200.layout import SceneLayout                     # noqa: E402


def main():
    D.init('nccl', timeout_s=60)
    r, n = D.rank(), D.world()
    dev = torch.device('cuda', torch.cuda.current_device())
    nc = NcclComm(dev)
    # point to point: every rank sends (r, p)-stamped rows to every peer p
    sends = [(p, torch.full((5, 3), float(100 * r + p), device=dev)) for p in range(n) if p != r]
    recvs = [(p, torch.zeros(5, 3, device=dev)) for p in range(n) if p != r]
    nc.exchange(sends, recvs)
    nc.wait(timeout_s=30)
    for p, t in recvs:
        assert torch.all(t == float(100 * p + r)), (r, p)
    # broadcast from the last rank
    b = torch.arange(1000, dtype=torch.float32, device=dev) * (r + 1)
    nc.broadcast(b, n - 1)
    nc.wait()
    assert torch.equal(b, torch.arange(1000, dtype=torch.float32, device=dev) * n)
    # all-to-all against torch's
    x = torch.randn(4 * n, 6, generator=torch.Generator().manual_seed(r)).to(dev)
    y, y_ref = torch.empty_like(x), torch.empty_like(x)
    nc.all_to_all(y, x)
    nc.wait()
    dist.all_to_all_single(y_ref, x, group=D.group())
    assert torch.equal(y, y_ref)
    # all-reduce against torch's
    z = torch.randn(333, generator=torch.Generator().manual_seed(10 + r)).to(dev)
    z_ref = z.clone()
    nc.all_reduce(z)
    nc.wait()
    dist.all_reduce(z_ref, group=D.group())
    assert torch.allclose(z, z_ref, rtol=1e-6, atol=1e-6)
    # the K/V exchange of a layout with halo and shared extra frames through both backends
    T, H, Dh = 32, 4, 64
    lay = SceneLayout([3, 5, 2, 4, 6], halo=1)
    lay.extra = {j: [lay.n_frames - 1] for j in range(lay.n_scenes)}
    L = lay.n_frames * T
    g = torch.Generator().manual_seed(7)
    k = torch.randn(L, H, Dh, generator=g).to(dev, torch.bfloat16)
    v = torch.randn(L, H, Dh, generator=g).to(dev, torch.bfloat16)
    own = comm.partition(lay, n, T, 'scene', [4] * lay.n_scenes)
    a, b_ = own[r]
    ex_t = comm.HaloExchange(lay, own, T, k[a:b_].contiguous(), v[a:b_].contiguous())
    ex_t.wait()
    ex_c = comm.HaloExchange(lay, own, T, k[a:b_].contiguous(), v[a:b_].contiguous(), collectives=nc)
    ex_c.wait(timeout_s=30)
    assert ex_c.remote_index == ex_t.remote_index
    assert torch.equal(ex_c.remote_k, ex_t.remote_k) and torch.equal(ex_c.remote_v, ex_t.remote_v)
    for lo, hi, off in ex_c.remote_index:
        assert torch.equal(ex_c.remote_k[off:off + hi - lo], k[lo:hi])
    torch.cuda.synchronize()
    nc.close()
    if r == 0:
        print(f'PASS n={n} orl_comm exchange/broadcast/all_to_all/all_reduce/HaloExchange '
              f'(broadcast rows {ex_c.broadcast_rows})', flush=True)
    D.barrier()
    D.shutdown()


if __name__ == '__main__':
    main()
