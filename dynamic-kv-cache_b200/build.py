"""Builds libdkv.so (the sm_100a CUDA library) in-tree with nvcc, and the C++
host binding of GPUCache's per-layer calls (_dkv_torch, csrc/torch_ops.cpp) with
g++ against PyTorch's headers.

The library is compiled for sm_100a only, without fast-math (the pack kernel
relies on IEEE fp32 division and subtraction for bit-exact codes); both files are
placed next to this file so they travel with the source tree.
"""
import os
import subprocess
import sys
import sysconfig
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


BINDING = HERE / ('_dkv_torch' + sysconfig.get_config_var('EXT_SUFFIX'))
BINDING_SOURCE = CSRC / 'torch_ops.cpp'


def build_binding(verbose=False):
    """Compiles the C++ host binding (a CPython extension over libdkv.so's C ABI,
    using PyTorch's tensor and stream types) next to libdkv.so."""
    import torch
    from torch.utils import cpp_extension as ce
    tmp = BINDING.with_name(BINDING.name + '.tmp')
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ['g++', '-O2', '-std=c++17', '-shared', '-fPIC', '-DTORCH_EXTENSION_NAME=_dkv_torch',
           '-DTORCH_API_INCLUDE_EXTENSION_H', f'-D_GLIBCXX_USE_CXX11_ABI={abi}',
           '-I', str(INCLUDE), '-I', sysconfig.get_paths()['include'],
           *[f'-I{p}' for p in ce.include_paths(device_type='cuda')],
           str(BINDING_SOURCE), '-o', str(tmp), '-L', str(HERE), '-ldkv', "-Wl,-rpath,$ORIGIN",
           *[f'-L{p}' for p in ce.library_paths(device_type='cuda')],
           '-lc10', '-lc10_cuda', '-ltorch', '-ltorch_cpu', '-ltorch_python', '-lcudart']
    if verbose:
        print(' '.join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, BINDING)
    return BINDING


def build(force=False, verbose=False):
    """Compiles libdkv.so if any source is newer than it, and the host binding if
    it or libdkv.so is newer than the binding; returns libdkv.so's path."""
    if force or stale():
        tmp = LIB.with_suffix('.so.tmp')
        cmd = [_nvcc(), *NVCC_FLAGS, '-I', str(INCLUDE), '-o', str(tmp), *[str(CSRC / s) for s in SOURCES]]
        if verbose:
            print(' '.join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    if force or not BINDING.exists() or any(p.stat().st_mtime > BINDING.stat().st_mtime
                                            for p in [LIB, BINDING_SOURCE, *INCLUDE.glob('*.h')]):
        build_binding(verbose)
    return LIB


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose=True))
