"""Sequence-parallel process group — the reference's `onereel.parallel.dist` (src/onereel/parallel/dist.py:1-82).

One process per GPU, launched by torchrun; torch.distributed over NCCL (NVLink / NVSwitch on B200) for the GPU path,
gloo for CPU tests. World 1 needs no process group. The reference optionally takes xfuser's sequence-parallel group;
this build always uses one group over all ranks (xfuser is not part of the B200 path).
"""
from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist

_ON = False
_GROUP = None


def init(backend: str | None = None, timeout_s: float = 120.0) -> int:
    """initialise from torchrun's variables (WORLD_SIZE, RANK, LOCAL_RANK); returns the world size. backend:
    'nccl' (default when CUDA is available) or 'gloo'. NCCL collectives get a high-priority stream so that the
    exchange is scheduled ahead of attention blocks when both are pending."""
    global _ON, _GROUP
    n = int(os.environ.get('WORLD_SIZE', 1))
    backend = backend or ('nccl' if torch.cuda.is_available() else 'gloo')
    if backend == 'nccl':
        torch.cuda.set_device(int(os.environ.get('LOCAL_RANK', 0)))
    if n == 1 or _ON:
        return n
    if not dist.is_initialized():
        kw = dict(timeout=timedelta(seconds=timeout_s))
        if backend == 'nccl':
            opts = dist.ProcessGroupNCCL.Options()
            opts.is_high_priority_stream = True
            kw.update(pg_options=opts, device_id=torch.device('cuda', torch.cuda.current_device()))
        dist.init_process_group(backend, **kw)
    _GROUP = dist.group.WORLD
    _ON = True
    return n


def world() -> int:
    return dist.get_world_size() if _ON else 1


def rank() -> int:
    return dist.get_rank() if _ON else 0


def group():
    return _GROUP if _ON else None


def peer_rank(r: int) -> int:
    """global rank of sequence-parallel rank r (one group over all ranks: the identity)"""
    return r


def all_reduce(x: torch.Tensor):
    if world() > 1:
        dist.all_reduce(x, group=group())


def all_gather_object(obj):
    if world() == 1:
        return [obj]
    out = [None] * world()
    dist.all_gather_object(out, obj, group=group())
    return out


def barrier():
    if world() > 1:
        dist.barrier(group=group())


def shutdown():
    global _ON, _GROUP
    if _ON and dist.is_initialized():
        dist.destroy_process_group()
    _ON, _GROUP = False, None


def check_consistent(what: str, obj) -> None:
    """every rank must hold the same `obj` (a plan: layout, partition, chosen path); ranks that disagree would post
    mismatched exchanges and wait on each other. Compares a digest of obj across ranks (all_gather_object) and raises
    on every rank if any differs."""
    if not _ON or world() == 1:
        return
    import hashlib
    import pickle
    digest = hashlib.sha256(pickle.dumps(obj)).hexdigest()
    digests = all_gather_object(digest)
    if len(set(digests)) > 1:
        bad = [r for r, d in enumerate(digests) if d != digests[0]]
        raise RuntimeError(f'{what} differs across ranks (ranks {bad} disagree with rank 0)')
