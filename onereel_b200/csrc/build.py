"""Build libonereel_b200.so in-tree with nvcc for sm_100a (no torch extension machinery: a plain C-ABI library).

    python -m onereel_b200.csrc.build            # or build() from __graft_entry__.py
Compiles every .cu and .cpp of this directory with -gencode arch=compute_100a,code=sm_100a and links them into
onereel_b200/libonereel_b200.so. Rebuilds only when a source or header is newer than the library.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
LIB = PKG / 'libonereel_b200.so'
SOURCES = sorted(HERE.glob('*.cu')) + sorted(HERE.glob('*.cpp'))
HEADERS = sorted(HERE.glob('*.cuh')) + sorted(HERE.glob('*.h')) + sorted((PKG.parent / 'include').glob('*.h'))
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
FLAGS = ['-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '-lineinfo', '-std=c++17', '--use_fast_math',
         '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden', '--expt-relaxed-constexpr']


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    out = HERE / '_build'
    out.mkdir(exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = out / (src.stem + '.o')
        cmd = [NVCC, *FLAGS, '-c', str(src), '-o', str(obj)]
        if verbose:
            cmd += ['-Xptxas', '-v']
            print(' '.join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix('.so.tmp')
    subprocess.run([NVCC, '-shared', '-gencode', 'arch=compute_100a,code=sm_100a', *objs, '-o', str(tmp),
                    '-lcudart', '-ldl'], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose='-v' in sys.argv))
