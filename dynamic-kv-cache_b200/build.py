"""Builds libdkv.so (the sm_100a CUDA library) in-tree with nvcc.

The library is compiled for sm_100a only, without fast-math (the pack kernel
relies on IEEE fp32 division and subtraction for bit-exact codes), and is placed
next to this file so it travels with the source tree.
"""
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / 'csrc'
INCLUDE = HERE.parent / 'include'
LIB = HERE / 'libdkv.so'
SOURCES = ['api.cu', 'pack.cu', 'attention_combine.cu', 'attention_tc.cu', 'attention_split.cu',
           'attention_noalloc.cu', 'decoder_ops.cu', 'pool.cu']
NVCC_FLAGS = ['-O3', '-std=c++17', '-gencode', 'arch=compute_100a,code=sm_100a', '-lineinfo',
              '-Xcompiler', '-fPIC', '-shared', '-Xptxas', '-warn-spills']


def _nvcc():
    home = os.environ.get('CUDA_HOME', '/usr/local/cuda')
    path = Path(home) / 'bin' / 'nvcc'
    return str(path) if path.exists() else 'nvcc'


def stale():
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    inputs = [CSRC / s for s in SOURCES] + list(CSRC.glob('*.cuh')) + list(INCLUDE.glob('*.h'))
    return any(p.stat().st_mtime > built for p in inputs)


def build(force=False, verbose=False):
    """Compiles libdkv.so if any source is newer than it; returns its path."""
    if not force and not stale():
        return LIB
    tmp = LIB.with_suffix('.so.tmp')
    cmd = [_nvcc(), *NVCC_FLAGS, '-I', str(INCLUDE), '-o', str(tmp), *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        print(' '.join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose=True))
