"""Split attention calls running next to other work on the same GPU.

A call whose history splits merge inside the attention kernel waits, in every
block, for the other blocks of its group. That is only safe when all blocks are
on the GPU together, which the library guarantees with a cooperative launch
rather than assumes. Here two caches attend on two streams at once while a long
GEMM keeps a third stream busy; both outputs must be bit-identical to the same
calls run alone, and no status word may report an error (a pipeline wait that
gave up would show up as DKV_ETIMEOUT through check()). Attend-only calls merge
in the combine kernel by default, so the same calls also run in a child process
with DKV_ATTENTION_MERGE=kernel, where they merge inside the attention kernel.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from dkv_testlib import frame_mix, outlier_kv

pytestmark = pytest.mark.gpu


def _cache(seed, past=8128, nq=64):
    from src.gpu_cache import GPUCache
    gen = torch.Generator().manual_seed(seed)
    outliers = torch.randperm(64, generator=gen)[:4]
    cache = GPUCache(None, layers=1, heads=5, max_tokens=past + nq + 64)
    hist_k, hist_v = outlier_kv(gen, 5, past, outliers)
    start = 0
    for f, bits in enumerate(frame_mix(seed, (past + 63) // 64)):
        n = min(64, past - start)
        cache.select(bits, f)
        cache.append(hist_k[:, :, start:start + n].cuda(), hist_v[:, :, start:start + n].cuda(), 0)
        start += n
    q = torch.randn(1, 15, nq, 64, generator=gen).bfloat16().cuda()
    kn, vn = (x.cuda() for x in outlier_kv(gen, 5, nq, outliers))
    return cache, q, kn, vn, past


def two_streams_next_to_a_long_kernel(launches):
    from src import gpu_kernels as K
    calls = [_cache(31), _cache(32)]
    assert K.attention_launches(8128, 64, 5, 3) == launches  # 1: splits merged inside the attention kernel
    alone = [c.attend(q, kn, vn, 0, p) for c, q, kn, vn, p in calls]
    torch.cuda.synchronize()

    a = torch.randn(8192, 8192, device='cuda', dtype=torch.bfloat16)
    streams = [torch.cuda.Stream() for _ in range(3)]
    for s in streams:
        s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(streams[2]):  # several milliseconds of GEMMs holding SMs
        busy = a
        for _ in range(4):
            busy = busy @ a
    together = [None, None]
    for rounds in range(3):  # every call overlaps the GEMMs or the other stream's calls
        for i, (c, q, kn, vn, p) in enumerate(calls):
            with torch.cuda.stream(streams[i]):
                together[i] = c.attend(q, kn, vn, 0, p)
    torch.cuda.synchronize()
    for (c, _, _, _, _), x, y in zip(calls, alone, together):
        c.check()
        assert torch.equal(x, y), float((x.float() - y.float()).abs().max())
    del busy  # the GEMMs only occupy the GPU; their result is not checked


def test_two_streams_next_to_a_long_kernel_match_the_calls_run_alone(cuda):
    two_streams_next_to_a_long_kernel(2)


def test_in_kernel_merge_next_to_a_long_kernel(cuda):
    root = Path(__file__).resolve().parents[1]
    code = ("import sys; sys.path[:0] = ['tests', 'dynamic-kv-cache_b200'];"
            "import test_gpu_concurrency as t; t.two_streams_next_to_a_long_kernel(1); print('ok')")
    env = dict(os.environ, DKV_ATTENTION_MERGE='kernel')
    r = subprocess.run([sys.executable, '-c', code], cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith('ok'), r.stderr[-2000:]
