"""GPU parity of the pack / reconstruct kernels: bit-exact against the reference
quantiser (golden vectors) and the oracle, plus the reference's own GPU tests."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from dkv_testlib import bits_np, outlier_kv
from oracle import kvq, pools

pytestmark = pytest.mark.gpu
PACK = np.load(GOLDEN / 'pack_golden.npz')
BF16_CASES = ['c2_k', 'c2_v', 'ref19', 'ties', 'tiny']


def gpu_tensor(bits16):
    return torch.from_numpy(bits16.astype(np.int16)).view(torch.bfloat16).cuda()


def pool_rows(cache, layer, kv, bits, row0, n):
    """Pool bytes of rows [row0, row0+n) as (payload [H, n, rowbytes] uint8, meta [H, n, 2] f32 | None)."""
    if bits == 16:
        payload = cache.pool_rows('p16', layer, kv, row0, n).contiguous().view(torch.uint8)
        return payload.cpu().numpy(), None
    p = cache.pool_rows('p4' if bits == 4 else 'p8', layer, kv, row0, n)
    m = cache.pool_rows('m4' if bits == 4 else 'm8', layer, kv, row0, n)
    return p.cpu().numpy(), m.cpu().numpy()


@pytest.mark.parametrize('case', BF16_CASES)
@pytest.mark.parametrize('bits', [4, 8, 16])
def test_pack_bit_exact_vs_reference_golden(cuda, case, bits):
    from src.gpu_cache import GPUCache
    x = PACK[f'{case}__x']
    _, heads, n, _ = x.shape
    k = gpu_tensor(x)
    c = GPUCache([(bits, n)], layers=3, heads=heads)
    c.select(bits)
    c.append(k, k, 2)
    c.check()
    payload, meta = pool_rows(c, 2, 0, bits, 0, n)
    golden = PACK[f'{case}__{bits}__payload'].reshape(payload.shape)
    assert np.array_equal(payload, golden)
    if bits != 16:
        assert np.array_equal(meta[..., 0].reshape(-1), PACK[f'{case}__{bits}__offsets'])
        assert np.array_equal(meta[..., 1].reshape(-1), PACK[f'{case}__{bits}__scales'])
        assert np.array_equal(meta[..., 1].reshape(-1).view(np.uint32),
                              PACK[f'{case}__{bits}__scales'].view(np.uint32))


@pytest.mark.parametrize('bits', [4, 8, 16])
def test_reference_gpu_pack_independent_error_bound(cuda, bits):
    # tests/test_gpu_backend.py:13-27 of the reference, same seed and layouts
    from src.gpu_cache import GPUCache
    torch.manual_seed(71)
    k = torch.randn((1, 3, 19, 64), device='cuda', dtype=torch.bfloat16)
    v = torch.randn((1, 19, 3, 64), device='cuda', dtype=torch.bfloat16).transpose(1, 2)
    c = GPUCache([(bits, 19)], layers=1)
    c.select(bits)
    c.append(k, v, 0)
    rk, rv = c.materialize(0)
    for x, y in [(k, rk), (v, rv)]:
        if bits == 16:
            assert torch.equal(x, y)
        else:
            xf = x.float()
            scale = (xf.amax(-1, keepdim=True) - xf.amin(-1, keepdim=True)) / ((1 << bits) - 1)
            assert torch.all((xf - y.float()).abs() <= scale * .501 + .032)


def test_c2_sweep_bit_exact_and_materialize_exact(cuda):
    """Pack-microbench shape (32 layers x 5 KV heads, 64-token frames, outlier K):
    the online cache grows through several reallocations; every sampled frame's
    pool rows are bit-identical to the oracle and materialize() equals the oracle's
    unpack rounded to bf16."""
    from src.gpu_cache import GPUCache
    gen = torch.Generator().manual_seed(2)
    outliers = torch.randperm(64, generator=gen)[:4]
    layers, heads, frames = 32, 5, 24
    bits_seq = [4, 8, 16] * (frames // 3)
    c = GPUCache(None, layers=layers, heads=heads)
    data = []
    for f, bits in enumerate(bits_seq):
        c.select(bits, f)
        per_layer = []
        for layer in range(layers):
            k, v = outlier_kv(gen, heads, 64, outliers)
            c.append(k.cuda(), v.cuda(), layer)
            per_layer.append((k, v))
        data.append(per_layer)
    c.check()
    assert c.caps[4] >= 512 and c.caps[8] >= 512 and c.caps[16] >= 512
    for f in range(0, frames, 5):
        start, end, bits, row0 = c.plan[f]
        for layer in (0, 13, 31):
            k, v = data[f][layer]
            for kv, x in enumerate((k, v)):
                ref = kvq.pack(bits_np(x), bits)
                payload, meta = pool_rows(c, layer, kv, bits, row0, 64)
                exp_payload, exp_meta = pools.frame_rows(ref, heads, 64)
                assert np.array_equal(payload, exp_payload), (f, layer, kv, bits)
                if meta is not None:
                    assert np.array_equal(meta, exp_meta)
    for layer in (0, 31):
        mk, mv = c.materialize(layer)
        for kv, got in enumerate((mk, mv)):
            expect = np.concatenate([kvq.unpack(kvq.pack(bits_np(data[f][layer][kv]), bits_seq[f]))
                                     for f in range(frames)], axis=2)
            expect_bf16 = kvq.f32_to_bf16_bits(expect)
            assert np.array_equal(bits_np(got), expect_bf16)


def test_nonfinite_pack_input_sets_status(cuda):
    from src.gpu_cache import GPUCache
    c = GPUCache(None, layers=1, heads=2)
    x = torch.randn(1, 2, 8, 64, device='cuda').bfloat16()
    x[0, 1, 3, 7] = float('nan')
    c.select(4)
    c.append(x, x, 0)
    with pytest.raises(ValueError, match='Nonfinite'):
        c.check()
    c.check()  # status was cleared


def test_corrupt_token_map_is_reported_not_trapped(cuda):
    from src.gpu_cache import GPUCache
    c = GPUCache(None, layers=1, heads=2)
    x = torch.randn(1, 2, 8, 64, device='cuda').bfloat16()
    c.select(8)
    c.append(x, x, 0)
    c.codes[3] = 7  # not a precision code: the readers skip the row and flag it
    k, v = c.materialize(0)
    with pytest.raises(ValueError, match='precision code'):
        c.check()
    assert torch.equal(k[0, :, 3], torch.zeros_like(k[0, :, 3]))
    c.codes[3] = 8
    c.rows[5] = 10_000  # outside the 8-bit pool
    c.materialize(0)
    with pytest.raises(ValueError, match='capacity'):
        c.check()
