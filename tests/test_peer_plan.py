"""Host logic of the peer-memory K/V exchange (onereel_b200.peer._Plan), no GPU: the run tables of stage 1 (pulls from
the owners) and stage 2 (stripes of rows every rank reads, pulled from the readers that fetched them), executed here
as plain array copies between simulated per-rank buffers, must fill every rank's receive buffer exactly as the
reference's HaloExchange lays it out (remote_index), and stage 2 may only read rows stage 1 already filled."""
import numpy as np
import pytest

from onereel_b200 import comm
from onereel_b200 import peer as P
from onereel_b200.layout import SceneLayout


class _Runs:
    def __init__(self, src_slot, dst_slot, src_off, dst_off, nbytes, device):
        self.runs = list(zip(src_slot, src_off, dst_off, nbytes))


CASES = [([8, 6, 10, 7] * 4, [0, 8, 14, 24], 8, 1), ([3, 5, 2, 4, 6], [1, 9], 3, 1), ([4] * 8, [], 4, 2),
         ([10, 1, 1, 2], [0], 4, 0), ([2, 2, 2, 2, 2, 2], [3], 6, 1)]


@pytest.mark.parametrize('lengths,memory,n,halo', CASES)
def test_two_stage_pull_fills_the_reference_layout(monkeypatch, lengths, memory, n, halo):
    monkeypatch.setattr(P, 'RunTable', _Runs)
    lay = SceneLayout(lengths, halo=halo)
    lay.extra = {j: [f for f in memory if not lo <= f < hi] for j, (lo, hi) in enumerate(lay.ranges)}
    T = 16
    own = comm.partition(lay, n, T, 'scene', [4] * len(lengths))
    plans = [P._Plan(lay, own, T, (), r, 'cpu', 1) for r in range(n)]
    recv = [np.full(max(pl.rows, 1), -1) for pl in plans]
    for r, pl in enumerate(plans):
        for p, so, do, nb in (pl.stage1.runs if pl.stage1 else []):
            recv[r][do:do + nb] = np.arange(own[p][0] + so, own[p][0] + so + nb)
    for r, pl in enumerate(plans):
        for q, so, do, nb in (pl.stage2.runs if pl.stage2 else []):
            assert (recv[q][so:so + nb] >= 0).all()
            recv[r][do:do + nb] = recv[q][so:so + nb]
    for r, pl in enumerate(plans):
        want = np.full(max(pl.rows, 1), -1)
        for lo, hi, off in pl.remote_index:
            want[off:off + hi - lo] = np.arange(lo, hi)
        assert (recv[r] == want).all()
        # the same receive layout as the NCCL exchange's
        need, _, _ = comm.exchange_plan(lay, own, T)
        ref = sorted((lo, hi) for p in range(n) if p != r for lo, hi in comm.clip(need[r], *own[p]))
        assert [(lo, hi) for lo, hi, _ in pl.remote_index] == ref
    if memory and n > 2:
        # the owner of the common rows sends each of them once in total
        owner_rows = sum(nb for pl in plans for p, _, _, nb in (pl.stage1.runs if pl.stage1 else []) if p == 0)
        need, common, p2p = comm.exchange_plan(lay, own, T)
        private = sum(hi - lo for q in range(n) if q != 0 for lo, hi in p2p[(0, q)])
        assert owner_rows == private + sum(hi - lo for lo, hi in common[0])


def test_plans_build_real_run_tables_on_the_host():
    """the bench's accounting builds every rank's plan with real run tables on the host (16-byte rows, the smallest
    the pack accepts): cfg2's scene set on 8 ranks"""
    lengths = [8, 6, 10, 7] * 8
    lay = SceneLayout(lengths, halo=0)
    lay.extra = {j: [f for f in (0, 8, 14, 24) if not lo <= f < hi] for j, (lo, hi) in enumerate(lay.ranges)}
    T, n = 1590, 8
    own = comm.partition(lay, n, T, 'scene', [128] * len(lengths))
    plans = [P._Plan(lay, own, T, (), q, 'cpu', 16) for q in range(n)]
    served = [sum(nb // 16 for pl in plans for tab in (pl.stage1, pl.stage2) if tab is not None
                  for src, nb in zip(tab.src_slot, tab.nbytes_list) if src == r) for r in range(n)]
    received = [pl.rows for pl in plans]
    assert sum(served) == sum(received) and all(x > 0 for x in received[1:])
