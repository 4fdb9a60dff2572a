"""Shared seeded input generators and comparison helpers for the tests."""
import random

import numpy as np
import torch

from oracle import cpu_path, kvq, pools

MIX_BITS = [4, 8, 16]
MIX_WEIGHTS = [0.5, 0.3, 0.2]


def outlier_kv(gen, heads, n, outliers):
    """K ~ N(0,1) with the seeded outlier channels x8, V ~ N(0,1); bf16 (CPU)."""
    k = torch.randn(1, heads, n, 64, generator=gen)
    k[..., outliers] *= 8
    v = torch.randn(1, heads, n, 64, generator=gen)
    return k.bfloat16(), v.bfloat16()


def frame_mix(seed, frames):
    return random.Random(seed).choices(MIX_BITS, weights=MIX_WEIGHTS, k=frames)


def bits_np(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def oracle_frames(hist_k, hist_v, plan):
    """Oracle-packs each (bits, n) segment of bf16 history [1, H, P, 64]."""
    out, start = [], 0
    for bits, n in plan:
        out.append(pools.pack_frame(bits_np(hist_k[:, :, start:start + n]),
                                    bits_np(hist_v[:, :, start:start + n]), bits))
        start += n
    return out


def oracle_attention(frames, q, knew, vnew, round_history_bf16=True):
    return cpu_path.cpu_cache_attention(frames, q.float().cpu(), knew.float().cpu(), vnew.float().cpu(),
                                        round_history_bf16=round_history_bf16)


def assert_attention_close(actual, expected, atol=0.035, rtol=0.015, max_rel=2e-2):
    """The reference's tolerance (tests/test_gpu_backend.py:101: atol .035, rtol .015)
    and a global relative error bound max|diff| / max|expected| <= 2e-2."""
    a, e = actual.float().cpu(), expected.float().cpu()
    assert a.shape == e.shape, (a.shape, e.shape)
    assert torch.isfinite(a).all()
    diff = (a - e).abs()
    assert torch.allclose(a, e, atol=atol, rtol=rtol), float(diff.max())
    rel = float(diff.max() / e.abs().max().clamp_min(1e-6))
    assert rel <= max_rel, rel
    return float(diff.max()), rel
