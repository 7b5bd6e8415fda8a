"""Multi-GPU parity of the parallel paths (K/V gathering, LSE overlap, Ulysses, Eq. 2 chooser) on 2, 4 and 8 GPUs (peer
memory and NCCL; from 3 ranks up the peer exchange moves rows every rank reads in two stages),
run as child processes under torchrun (tests/dist_scene_worker.py). Skipped on a box with fewer than 2 GPUs; the
host-side logic of the same paths is covered on CPU by test_dist_gloo.py and test_planner_native.py."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


@pytest.mark.parametrize('n', [2, 4, 8])
def test_parallel_paths_match_single_gpu(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f'needs {n} GPUs')
    from onereel_b200.csrc.build import build
    build()
    env = dict(os.environ, NCCL_NVLS_ENABLE='0', PYTHONPATH=str(ROOT))
    cmd = ['timeout', '-k', '30', '600', sys.executable, '-m', 'torch.distributed.run', '--nnodes=1',
           f'--nproc-per-node={n}', '--master-addr', '127.0.0.1', '--master-port', str(_free_port()),
           str(ROOT / 'tests' / 'dist_scene_worker.py')]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert p.returncode == 0, p.stdout[-4000:] + p.stderr[-4000:]
    assert p.stdout.count('PASS') == 5, p.stdout


@pytest.mark.parametrize('n', [2])
def test_c_abi_collectives_match_torch_distributed(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f'needs {n} GPUs')
    env = dict(os.environ, NCCL_NVLS_ENABLE='0', PYTHONPATH=str(ROOT))
    cmd = ['timeout', '-k', '30', '300', sys.executable, '-m', 'torch.distributed.run', '--nnodes=1',
           f'--nproc-per-node={n}', '--master-addr', '127.0.0.1', '--master-port', str(_free_port()),
           str(ROOT / 'tests' / 'dist_comm_worker.py')]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert p.returncode == 0, p.stdout[-4000:] + p.stderr[-4000:]
    assert 'PASS' in p.stdout, p.stdout
