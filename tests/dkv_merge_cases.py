"""Seeded attention calls shared by the split-merge tests; run as a script it
writes the outputs to the .npz named on the command line (used to run the same
calls in a child process with another DKV_ATTENTION_MERGE setting)."""
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / 'dynamic-kv-cache_b200')]

# (past, nq, kv heads, group): tensor-core shapes with 2..37 splits and 1..2 row blocks
CASES = [(8128, 64, 5, 3), (2000, 128, 5, 3), (16000, 16, 8, 4), (700, 64, 2, 7), (130, 64, 1, 1)]


def run_case(past, nq, heads, group, seed=0, fused=False):
    """append + attend of nq new rows over `past` packed rows (fused: one
    append_attend call, which merges its splits inside the attention kernel by
    default); returns the output and the launches dkv_packed_attention makes."""
    from src.gpu_cache import GPUCache
    from src import gpu_kernels as K
    gen = torch.Generator(device='cuda').manual_seed(seed + past)
    cache = GPUCache(None, layers=1, heads=heads, device='cuda', max_tokens=past + nq + 64)
    start, f = 0, 0
    while start < past:
        n = min(64, past - start)
        cache.select((4, 8, 16)[f % 3], f)
        k = torch.randn(1, heads, n, 64, generator=gen, device='cuda').bfloat16()
        v = torch.randn(1, heads, n, 64, generator=gen, device='cuda').bfloat16()
        cache.append(k, v, 0)
        start += n
        f += 1
    q = torch.randn(1, heads * group, nq, 64, generator=gen, device='cuda').bfloat16()
    kn = torch.randn(1, heads, nq, 64, generator=gen, device='cuda').bfloat16()
    vn = torch.randn(1, heads, nq, 64, generator=gen, device='cuda').bfloat16()
    cache.select(16)
    if fused:
        p = past
        out = cache.append_attend(q, kn, vn, 0)
    else:
        p = cache.append(kn, vn, 0)
        out = cache.attend(q, kn, vn, 0, p)
    cache.check()
    return out, K.attention_launches(p, nq, heads, group)


def main(path):
    outs, launches = {}, {}
    for i, case in enumerate(CASES):
        out, n = run_case(*case)
        outs[f'out{i}'] = out.view(torch.int16).cpu().numpy()
        outs[f'launches{i}'] = np.int32(n)
    np.savez(path, **outs)


if __name__ == '__main__':
    main(sys.argv[1])
