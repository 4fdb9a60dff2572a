"""Append + attend in one call (dkv_append_attention): the output, the pools and
the token maps must be bit-identical to pack_rows (+ map_fill) followed by
packed_attention (one launch: the attention blocks pack the frame), from decode-
shaped calls (1 query) to two row blocks per KV head."""
import os
import subprocess
import sys

import pytest
import torch

from conftest import ROOT
from dkv_testlib import frame_mix, outlier_kv
from src.gpu_cache import GPUCache

pytestmark = pytest.mark.gpu


def _twins(past, seed, layers=2):
    gen = torch.Generator().manual_seed(seed)
    outliers = torch.randperm(64, generator=gen)[:4]
    hist_k, hist_v = outlier_kv(gen, 5, max(past, 1), outliers)
    out = []
    for _ in range(2):
        c = GPUCache(None, layers=layers, heads=5, device='cuda', max_tokens=past + 256)
        start, f = 0, 0
        for bits in frame_mix(seed, (past + 63) // 64):
            m = min(64, past - start)
            c.select(bits, f)
            for layer in range(layers):
                c.append(hist_k[:, :, start:start + m].cuda(), hist_v[:, :, start:start + m].cuda(), layer)
            start, f = start + m, f + 1
        out.append(c)
    return out, gen, outliers


@pytest.mark.parametrize('past,n,bits', [(0, 64, 4), (300, 64, 8), (8128, 64, 16), (4000, 96, 4), (2500, 5, 8),
                                         (1000, 1, 16)])
def test_append_attend_equals_append_then_attend(cuda, past, n, bits):
    (a, b), gen, outliers = _twins(past, past + n)
    for layer in range(2):
        q = torch.randn(1, 15, n, 64, generator=gen).bfloat16().cuda()
        k = outlier_kv(gen, 5, n, outliers)[0].cuda()
        v = torch.randn(1, 5, n, 64, generator=gen).bfloat16().cuda()
        a.select(bits, 500), b.select(bits, 500)
        p = a.append(k, v, layer)
        want = a.attend(q, k, v, layer, p)
        got = b.append_attend(q, k, v, layer)
        a.check(), b.check()
        assert torch.equal(got, want), float((got.float() - want.float()).abs().max())
        assert a.seen == b.seen and a.plan == b.plan
    total = a.seen[0]
    assert torch.equal(a.rows[:total], b.rows[:total]) and torch.equal(a.codes[:total], b.codes[:total])
    for layer in range(2):
        for x, y in zip(a.materialize(layer), b.materialize(layer)):
            assert torch.equal(x, y)


def test_append_attend_with_the_separate_merge_kernel(cuda):
    """DKV_ATTENTION_MERGE=combine: the attention kernel packs after its epilogue
    and a combine launch merges; still bit-identical to the two calls."""
    code = (
        "import sys, torch; sys.path.insert(0, 'tests'); sys.path.insert(0, 'dynamic-kv-cache_b200');"
        "from test_gpu_fused_append import _twins; from dkv_testlib import outlier_kv;"
        "(a, b), gen, o = _twins(6000, 9);"
        "q = torch.randn(1, 15, 64, 64, generator=gen).bfloat16().cuda();"
        "k = outlier_kv(gen, 5, 64, o)[0].cuda(); v = torch.randn(1, 5, 64, 64, generator=gen).bfloat16().cuda();"
        "a.select(4, 9); b.select(4, 9); p = a.append(k, v, 0); w = a.attend(q, k, v, 0, p);"
        "g = b.append_attend(q, k, v, 0); a.check(); b.check();"
        "assert torch.equal(g, w);"
        "assert all(torch.equal(x, y) for x, y in zip(a.materialize(0), b.materialize(0)));"
        "print('ok')")
    env = dict(os.environ, DKV_ATTENTION_MERGE='combine')
    r = subprocess.run([sys.executable, '-c', code], cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith('ok'), r.stderr[-2000:]
