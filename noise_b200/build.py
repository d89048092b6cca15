"""Build the in-tree shared library ``noise_b200/libnoise_b200.so`` (sm_100a) with nvcc.

The library has no PyTorch dependency: it exports the C ABI of ``include/noise_b200.h`` and links the CUDA runtime
statically. ``python -m noise_b200.build`` (or ``__graft_entry__.build()``) rebuilds it when a source is newer.
"""
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / 'csrc'
LIB = PKG / 'libnoise_b200.so'
SOURCES = sorted(CSRC.glob('*.cu'))
HEADERS = sorted(CSRC.glob('*.cuh')) + sorted((ROOT / 'include').glob('*.h'))
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']


def nvcc():
    for cand in (os.environ.get('NVCC'), shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError('nvcc not found')


def stale():
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS + [Path(__file__)])


def build(force=False, verbose=False):
    if not force and not stale():
        return LIB
    tmp = LIB.with_suffix('.so.tmp')
    cmd = [nvcc(), *ARCH, '-O3', '-lineinfo', '-std=c++17', '-DNOISE_B200_BUILD',
           '-I', str(ROOT / 'include'), '-I', str(CSRC), '-Xcompiler', '-fPIC,-O3', '-shared', '-cudart', 'static',
           '-o', str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, '-Xptxas=-v')
        print(' '.join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    build(force='--force' in sys.argv, verbose='-v' in sys.argv)
    print(LIB)
