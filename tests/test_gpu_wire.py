"""Wire format on the GPU: frames exported from a GPUCache are byte-for-byte the
reference quantiser's pack() of the same bf16 K/V (payload, scales, offsets,
header); frames packed on the CPU and imported give the same cache (materialize
and attention bit-identical to appending them on the device)."""
import numpy as np
import pytest
import torch

from oracle import kvq
from src import wire
from src.gpu_cache import GPUCache

pytestmark = pytest.mark.gpu
PLAN = [4, 8, 16, 4, 16, 8]


def frames(seed, heads=5, n=64, layers=2):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in PLAN:
        k = torch.randn(layers, 1, heads, n, 64, generator=g)
        k[..., :4] *= 8
        out.append((k.bfloat16(), torch.randn(layers, 1, heads, n, 64, generator=g).bfloat16()))
    return out


def bits_np(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_export_matches_reference_pack(cuda):
    data = frames(3)
    cache = GPUCache(None, layers=2, heads=5, device='cuda')
    for f, (bits, (k, v)) in enumerate(zip(PLAN, data)):
        cache.select(bits, f)
        for layer in range(2):
            cache.append(k[layer].cuda(), v[layer].cuda(), layer)
    cache.check()
    for layer in range(2):
        for index, (bits, (k, v)) in enumerate(zip(PLAN, data)):
            got = wire.export_segment(cache, layer, index)
            for packed, x in zip(got, (k[layer], v[layer])):
                ref = kvq.pack(bits_np(x), bits)
                assert packed.header.numpy().tobytes() == ref.header.tobytes()
                assert np.array_equal(packed.payload.numpy(), ref.payload)
                assert np.array_equal(packed.scales.numpy().view(np.uint32), ref.scales.view(np.uint32))
                assert np.array_equal(packed.offsets.numpy().view(np.uint32), ref.offsets.view(np.uint32))


def test_import_of_cpu_packed_frames_equals_device_append(cuda):
    data = frames(5)
    device = GPUCache(None, layers=2, heads=5, device='cuda')
    imported = GPUCache(None, layers=2, heads=5, device='cuda')
    for f, (bits, (k, v)) in enumerate(zip(PLAN, data)):
        device.select(bits, f)
        imported.select(bits, f)
        for layer in range(2):
            device.append(k[layer].cuda(), v[layer].cuda(), layer)
            kp, vp = (wire.from_bytes(wire.to_bytes(wire.PackedTensor(
                torch.from_numpy(p.payload.copy()), torch.from_numpy(p.scales.copy()),
                torch.from_numpy(p.offsets.copy()), torch.from_numpy(p.header.copy()))))
                for p in (kvq.pack(bits_np(k[layer]), bits), kvq.pack(bits_np(v[layer]), bits)))
            assert wire.import_frame(imported, kp, vp, layer) == device.seen[layer] - 64
    assert imported.plan == device.plan and imported.seen == device.seen
    g = torch.Generator(device='cuda').manual_seed(1)
    q = torch.randn(1, 15, 64, 64, generator=g, device='cuda').bfloat16()
    kn = torch.randn(1, 5, 64, 64, generator=g, device='cuda').bfloat16()
    vn = torch.randn(1, 5, 64, 64, generator=g, device='cuda').bfloat16()
    for layer in range(2):
        for a, b in zip(device.materialize(layer), imported.materialize(layer)):
            assert torch.equal(a, b)
        past = device.seen[layer]
        assert torch.equal(device.attend(q, kn, vn, layer, past), imported.attend(q, kn, vn, layer, past))
    device.check()
    imported.check()


def test_import_rejects_mismatched_precision(cuda):
    cache = GPUCache(None, layers=1, heads=5, device='cuda')
    x = bits_np(torch.zeros(1, 5, 64, 64).bfloat16())
    p = kvq.pack(x, 8)
    packed = wire.PackedTensor(torch.from_numpy(p.payload.copy()), torch.from_numpy(p.scales.copy()),
                               torch.from_numpy(p.offsets.copy()), torch.from_numpy(p.header.copy()))
    cache.select(4)
    with pytest.raises(ValueError, match='8 bits'):
        wire.import_frame(cache, packed, packed, 0)
