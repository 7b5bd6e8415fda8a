"""The collectives of the parallel paths on CPU gloo ranks (world size 2 and 3): the K/V exchange lands exactly the
rows each rank's compiled plan expects (at world 3 rows every peer reads arrive by broadcast), the text-row P2P and the Ulysses all-to-all round trip move the right rows,
gather_tokens reassembles unequal ranges — the reference's tests/dist_onereel_gather.py checks, without a GPU; the
peer-memory exchange falls back to NCCL-style send/recv where symmetric memory is unavailable."""
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                          LOCAL_RANK=str(rank))
        from onereel_b200 import comm, dist as D
        from onereel_b200 import scene as S
        from onereel_b200.layout import SceneLayout
        D.init('gloo', timeout_s=60)
        r, n = D.rank(), D.world()
        T, H, Dh = 16, 2, 8
        bcast = 0
        for lengths, halo, extra in (([3, 5, 2, 4, 6], 0, True), ([10, 1, 1, 2], 2, False), ([5, 2, 7], 1, True)):
            g = torch.Generator().manual_seed(len(lengths))
            lay = SceneLayout(lengths, halo=halo)
            if extra:
                lay.extra = {j: [(7 * j + 3) % lay.n_frames, lay.n_frames - 1] for j in range(lay.n_scenes)}
            L = lay.n_frames * T
            k, v = torch.randn(L, H, Dh, generator=g), torch.randn(L, H, Dh, generator=g)
            counts = [3 + j for j in range(lay.n_scenes)]
            own = comm.partition(lay, n, T, 'scene', counts)
            a, b = own[r]
            ex = comm.HaloExchange(lay, own, T, k[a:b].contiguous(), v[a:b].contiguous())
            ex.wait()
            bcast += ex.broadcast_rows
            assert ex.remote_index == S.remote_index_of(lay, T, own, r, comm.needed)
            for lo, hi, off in ex.remote_index:                    # every received row is the sender's row
                assert torch.equal(ex.remote_k[off:off + hi - lo], k[lo:hi])
                assert torch.equal(ex.remote_v[off:off + hi - lo], v[lo:hi])
            for j, (flo, fhi) in enumerate(lay.ranges):             # rows() as the reference's test checks it
                if flo * T < b and fhi * T > a:
                    want = torch.cat([k[f * T:(f + 1) * T] for f in lay.key_frames(j)])
                    assert torch.equal(ex.rows(0)(lay.key_frames(j)), want), (lengths, r, j)
            # the peer-memory exchange needs CUDA symmetric memory: on CPU ranks it falls back to this exchange, with
            # the reason kept, and delivers the same rows
            ex2 = comm.kv_exchange('peer', lay, own, T, k[a:b].contiguous(), v[a:b].contiguous())
            ex2.wait()
            assert comm.PEER_UNAVAILABLE is not None and isinstance(ex2, comm.HaloExchange)
            assert ex2.remote_index == ex.remote_index and torch.equal(ex2.remote_k, ex.remote_k)
            kb, vb, token_row = ex.buffer()
            held = token_row >= 0
            assert torch.equal(kb[token_row[held]], k[held])
            # text rows: scene j's text outputs travel from the rank holding its first frame to the others touching j
            tr = S.text_ranges(counts)
            x = torch.zeros(sum(counts), H, Dh)
            for j, (flo, _) in enumerate(lay.ranges):
                if a <= flo * T < b:
                    x[tr[j][0]:tr[j][1]] = float(j + 1)
            comm.send_text_rows(x, lay, own, T, tr)
            for j, (flo, fhi) in enumerate(lay.ranges):
                if flo * T < b and fhi * T > a:
                    assert torch.all(x[tr[j][0]:tr[j][1]] == float(j + 1)), (lengths, r, j)
            # gather_tokens over the unequal ranges
            full = torch.arange(L, dtype=torch.float32)[None, :, None].expand(1, L, 3).contiguous()
            assert torch.equal(comm.gather_tokens(full[:, a:b].contiguous(), own), full)
        # at world 3 the frame every scene reads (extra frame F - 1) travels as a broadcast from its owner
        assert n < 3 or bcast > 0, 'no broadcast exercised'
        # Ulysses all-to-all round trip on an equal split
        S_, H4 = 6 * n, 2 * n
        x = torch.randn(S_, H4, Dh, generator=torch.Generator().manual_seed(5))
        lo, hi = r * S_ // n, (r + 1) * S_ // n
        xa = comm.a2a_heads(x[lo:hi].contiguous())
        sl = slice(r * H4 // n, (r + 1) * H4 // n)
        assert torch.equal(xa, x[:, sl])
        assert torch.equal(comm.a2a_tokens(xa).contiguous(), x[lo:hi])
        D.barrier()
        D.shutdown()
        q.put((rank, None))
    except Exception:
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize('world', [2, 3])
def test_collectives_on_gloo(world):
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    errors = [f'rank {r}:\n{e}' for r, e in results if e]
    assert not errors, '\n'.join(errors)


def _mismatch_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                          LOCAL_RANK=str(rank))
        from onereel_b200 import dist as D, hunyuan15 as HY
        from onereel_b200.layout import SceneLayout
        D.init('gloo', timeout_s=30)
        lengths = [3, 5, 2] if rank == 0 else [3, 5, 3]          # rank 1 planned from another request
        ctx = HY.Context(SceneLayout(lengths, halo=1), mode='scene', T=16, counts={True: [4, 4, 4]})
        try:
            HY.plan_parallel(ctx, 4)
            q.put((rank, 'no error raised'))
        except RuntimeError as e:
            q.put((rank, None if 'differs across ranks' in str(e) else repr(e)))
        D.shutdown()
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_mismatched_plans_fail_on_every_rank():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mismatch_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(e is None for _, e in results), results


def _early_exit_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                          LOCAL_RANK=str(rank))
        import time
        from onereel_b200 import comm, dist as D
        D.init('gloo', timeout_s=10)
        D.barrier()
        if rank == 1:
            q.put((rank, None))
            q.close()
            q.join_thread()                                        # the result is delivered before the rank leaves
            os._exit(0)                                            # leaves between steps, nothing in flight
        t0 = time.time()
        try:
            comm.gather_tokens(torch.zeros(1, 4, 2), [(0, 4), (4, 8)])
            q.put((rank, 'collective with a departed rank returned'))
        except Exception:
            q.put((rank, None if time.time() - t0 < 120 else 'detected too late'))
        q.close()
        q.join_thread()
        os._exit(0)
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_departed_rank_is_detected_not_waited_for():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_early_exit_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(e is None for _, e in results), results
