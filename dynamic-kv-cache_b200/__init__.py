"""B200 (sm_100a) packed mixed-precision KV cache: drop-in for the reference's
packed-KV hot path (zoaibs/Dynamic-KV-Cache src/gpu_cache.py, src/gpu_kernels.py,
src/gpu_ops.py, src/inference.py).

The Python modules live in the `src` subpackage under the reference's own module
names, so a user puts this directory on sys.path and keeps
`from src.gpu_cache import GPUCache`. The CUDA kernels are in csrc/ and are
reached through the C ABI of libdkv.so (include/dkv.h).
"""
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
LIBRARY = PACKAGE_DIR / 'libdkv.so'
