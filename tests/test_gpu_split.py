"""The split-K attention kernel for short query chunks (at most 16 stacked rows
per KV head: decode steps and small candidate chunks) against the CPU oracle.

Covers history lengths around the 32-key tile and the split boundaries, 1 to
16 stacked rows (group 3, 8 and 1), histories split across whole 16-block
clusters, the current chunk's native rows, the causal cut inside the last tile,
bit-identical reruns, and the single-launch, no-workspace plan.
"""
import pytest
import torch

from dkv_testlib import assert_attention_close, frame_mix, oracle_attention, oracle_frames, outlier_kv

pytestmark = pytest.mark.gpu


def _run(past, nq, heads, group, seed, bits=None):
    from src.gpu_cache import GPUCache
    gen = torch.Generator().manual_seed(seed)
    outliers = torch.randperm(64, generator=gen)[:4]
    frames = (past + 63) // 64
    mix = frame_mix(seed, frames) if bits is None else [bits] * frames
    plan = [(b, min(64, past - 64 * f)) for f, b in enumerate(mix)]
    cache = GPUCache(None, layers=1, heads=heads, max_tokens=past + nq + 64)
    hist_k, hist_v = outlier_kv(gen, heads, past, outliers)
    start = 0
    for f, (b, n) in enumerate(plan):
        cache.select(b, f)
        cache.append(hist_k[:, :, start:start + n].cuda(), hist_v[:, :, start:start + n].cuda(), 0)
        start += n
    q = torch.randn(1, heads * group, nq, 64, generator=gen).bfloat16()
    kn, vn = outlier_kv(gen, heads, nq, outliers)
    out = cache.attend(q.cuda(), kn.cuda(), vn.cuda(), 0, past)
    again = cache.attend(q.cuda(), kn.cuda(), vn.cuda(), 0, past)
    cache.check()
    expected = oracle_attention(oracle_frames(hist_k, hist_v, plan), q, kn, vn)
    return out, again, expected


@pytest.mark.parametrize('past', [0, 1, 31, 32, 33, 63, 127, 128, 129, 511, 999, 2047, 4096, 8128])
@pytest.mark.parametrize('nq', [1, 5])
def test_short_chunks_vs_oracle(cuda, past, nq):
    out, again, expected = _run(past, nq, 5, 3, seed=past * 7 + nq)
    assert_attention_close(out, expected, atol=0.01, rtol=0.01)
    assert torch.equal(out, again)  # deterministic: fixed split plan and merge order


@pytest.mark.parametrize('heads,group,nq', [(2, 8, 2), (1, 1, 16), (4, 4, 3), (8, 2, 8)])
def test_row_counts_up_to_sixteen(cuda, heads, group, nq):
    out, _, expected = _run(3000, nq, heads, group, seed=heads * 100 + group * 10 + nq)
    assert_attention_close(out, expected, atol=0.01, rtol=0.01)


@pytest.mark.parametrize('bits', [4, 8, 16])
def test_uniform_precision_histories(cuda, bits):
    out, _, expected = _run(1500, 1, 5, 3, seed=bits, bits=bits)
    assert_attention_close(out, expected, atol=0.01, rtol=0.01)


def test_plan_is_one_launch_without_workspace(cuda):
    from src import gpu_kernels as K
    for past, nq in ((8128, 1), (8128, 5), (0, 1), (100000, 3)):
        assert K.attention_launches(past, nq, 5, 3) == 1
        assert K.attention_workspace_bytes(past, nq, 5, 3) == 0
