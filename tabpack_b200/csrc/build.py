"""Build `tabpack_b200/libtabpack_b200.so` (sm_100a) with nvcc, in-tree.

    python -m tabpack_b200.csrc.build [--verbose]

The library is a single translation unit (`tabpack_b200.cu`) linked against the
static CUDA runtime, so it only needs the NVIDIA driver at run time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, 'libtabpack_b200.so')
SOURCES = ['tabpack_b200.cu']
# every header beside the translation unit, so that an edit to any of them triggers a rebuild
HEADERS = sorted(f for f in os.listdir(HERE) if f.endswith('.cuh'))


def nvcc_path() -> str:
    for cand in (os.environ.get('NVCC'), shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError('nvcc not found')


def _inputs():
    files = [os.path.join(HERE, f) for f in SOURCES + HEADERS]
    files.append(os.path.join(ROOT, 'include', 'tabpack_b200.h'))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [
        nvcc_path(), '-O3', '-std=c++17', '-lineinfo',
        '-gencode', 'arch=compute_100a,code=sm_100a',
        '-Xcompiler', '-fPIC', '-shared', '-cudart', 'static',
        '--expt-relaxed-constexpr',
        '-I', os.path.join(ROOT, 'include'), '-I', HERE,
        '-o', LIB + '.tmp',
    ] + [os.path.join(HERE, s) for s in SOURCES]
    if verbose:
        cmd.insert(1, '-Xptxas=-v')
        print(' '.join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(LIB + '.tmp', LIB)
    return LIB


if __name__ == '__main__':
    build(force=True, verbose='--verbose' in sys.argv)
    print(LIB)
