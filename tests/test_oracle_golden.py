"""Pins the CPU oracle against golden vectors produced by the reference itself
(its quantiser and its Triton kernels in the interpreter; tests/golden/make_golden.py)."""
import math

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import cpu_path, kvq, pools

PACK = np.load(GOLDEN / 'pack_golden.npz')
PACK_CASES = sorted({k.split('__')[0] for k in PACK.files})
ATTN_CASES = sorted(p.stem[len('attn_'):] for p in GOLDEN.glob('attn_*.npz'))


def f32_bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize('case', PACK_CASES)
@pytest.mark.parametrize('bits', [4, 8, 16])
def test_oracle_pack_is_bit_exact_with_reference(case, bits):
    x = PACK[f'{case}__x']
    dtype = str(PACK[f'{case}__dtype'])
    p = kvq.pack(x, bits, 64, dtype=dtype)
    assert np.array_equal(p.payload, PACK[f'{case}__{bits}__payload'])
    assert np.array_equal(p.header, PACK[f'{case}__{bits}__header'])
    # scales / offsets compared as values (-0.0 == +0.0) and as bit patterns
    assert np.array_equal(p.scales, PACK[f'{case}__{bits}__scales'])
    assert np.array_equal(p.offsets, PACK[f'{case}__{bits}__offsets'])
    assert np.array_equal(f32_bits(p.scales), f32_bits(PACK[f'{case}__{bits}__scales']))


def test_golden_has_the_reference_test_shapes():
    assert PACK['odd65_f32__x'].shape == (1, 3, 7, 65)
    assert PACK['c2_k__x'].shape == (1, 5, 64, 64)


@pytest.mark.parametrize('bits', [4, 8, 16])
def test_oracle_payload_bytes_and_roundtrip_bound(bits):
    # tests/test_quantization.py:6-23 restated on the oracle
    x = PACK['odd65_f32__x']
    p = kvq.pack(x, bits, 64, dtype='float32')
    assert p.payload.size == math.ceil(x.size * bits / 8)
    meta = p.scales.nbytes + p.offsets.nbytes + p.header.nbytes
    assert meta == 64 + (0 if bits == 16 else 8 * math.ceil(x.size / 64))
    out = kvq.unpack(p)
    if bits == 16:
        assert np.array_equal(out, x.astype(np.float16).astype(np.float32))
    else:
        scale = np.repeat(p.scales, 64)[:x.size]
        assert np.all(np.abs(out - x).reshape(-1) <= scale / 2 + 1e-5)


def test_oracle_constant_group_exact_and_nonfinite_rejected():
    x = np.full((1, 1, 3, 17), -2.5, np.float32)
    for bits in (4, 8, 16):
        assert np.array_equal(kvq.unpack(kvq.pack(x, bits, dtype='float32')), x)
    with pytest.raises(ValueError):
        kvq.pack(np.full((1, 1, 1, 1), np.nan, np.float32), 4, dtype='float32')
    with pytest.raises(ValueError):
        kvq.pack(np.zeros((1, 1, 1, 1), np.float32), 5, dtype='float32')


def test_oracle_half_step_ties_round_to_even():
    x = PACK['ties__x']
    p = kvq.pack(x, 4, dtype='bfloat16')
    codes = kvq.codes_of(p)[:64]
    values = kvq.bf16_bits_to_f32(x).reshape(-1)[:64]
    # (x - 0) / 1 lands exactly on k + 0.5: even k stays, odd k rounds up
    assert values[2] == 2.5 and codes[2] == 2
    assert values[3] == 3.5 and codes[3] == 4
    assert values[4] == 4.5 and codes[4] == 4
    assert values[14] == 0.5 and codes[14] == 0


@pytest.mark.parametrize('case', ATTN_CASES)
def test_oracle_attention_matches_reference_triton_kernel(case):
    g = np.load(GOLDEN / f'attn_{case}.npz')
    heads, group, nq = int(g['heads']), int(g['group']), int(g['nq'])
    frames = []
    start = 0
    for bits, n in zip(g['frame_bits'].tolist(), g['frame_tokens'].tolist()):
        k = g['hist_k'][:, :, start:start + n]
        v = g['hist_v'][:, :, start:start + n]
        frames.append(pools.pack_frame(k, v, bits))
        start += n
    q = torch.from_numpy(kvq.bf16_bits_to_f32(g['q']))
    kn = torch.from_numpy(kvq.bf16_bits_to_f32(g['knew']))
    vn = torch.from_numpy(kvq.bf16_bits_to_f32(g['vnew']))
    out = cpu_path.cpu_cache_attention(frames, q, kn, vn)
    assert out.shape == (1, nq, heads * group, 64)
    # both sides are fp32 end to end: agreement to rounding noise
    assert torch.allclose(out, torch.from_numpy(g['out']), atol=2e-5, rtol=1e-5)


@pytest.mark.parametrize('case', [c for c in ATTN_CASES if 'recon' in np.load(GOLDEN / f'attn_{c}.npz').files])
def test_oracle_unpack_matches_reference_reconstruct(case):
    g = np.load(GOLDEN / f'attn_{case}.npz')
    ks, vs, start = [], [], 0
    for bits, n in zip(g['frame_bits'].tolist(), g['frame_tokens'].tolist()):
        pk, pv = pools.pack_frame(g['hist_k'][:, :, start:start + n], g['hist_v'][:, :, start:start + n], bits)
        ks.append(kvq.unpack(pk)[0])
        vs.append(kvq.unpack(pv)[0])
        start += n
    mine = np.stack([np.concatenate(ks, 1), np.concatenate(vs, 1)])
    ref = g['recon']
    # the interpreter may fuse q*s+a; allow one fp32 ulp-scale difference
    assert np.allclose(mine, ref, atol=1e-6, rtol=1e-6)
    torch_path = torch.stack([torch.cat([cpu_path.unpack_torch(pools.pack_frame(
        g['hist_k'][:, :, s:s + n], g['hist_v'][:, :, s:s + n], b)[kv])[0] for b, n, s in zip(
        g['frame_bits'].tolist(), g['frame_tokens'].tolist(),
        np.concatenate([[0], np.cumsum(g['frame_tokens'])[:-1]]).tolist())], 1) for kv in (0, 1)])
    assert np.array_equal(torch_path.numpy(), mine)
