"""CPU checks of the packed-tensor wire format (src/wire.py): headers match the
reference quantiser's, byte round trips, and the header validation."""
import numpy as np
import pytest
import torch

from oracle import kvq
from src import wire


def as_wire(p):
    return wire.PackedTensor(torch.from_numpy(p.payload.copy()), torch.from_numpy(p.scales.copy()),
                             torch.from_numpy(p.offsets.copy()), torch.from_numpy(p.header.copy()))


@pytest.mark.parametrize('bits', [4, 8, 16])
def test_header_and_bytes_round_trip(bits):
    rng = np.random.default_rng(bits)
    x = kvq.f32_to_bf16_bits(rng.standard_normal((1, 5, 64, 64)).astype(np.float32))
    ref = kvq.pack(x, bits)
    assert bytes(wire._header(bits, 5, 64, 64).tolist()) == ref.header.tobytes()
    packed = as_wire(ref)
    assert packed.fields() == ref.fields()
    back = wire.from_bytes(wire.to_bytes(packed))
    assert torch.equal(back.payload, packed.payload) and torch.equal(back.header, packed.header)
    assert torch.equal(back.scales, packed.scales) and torch.equal(back.offsets, packed.offsets)
    assert back.storage_bytes == packed.storage_bytes


def test_corrupt_bytes_are_rejected():
    x = kvq.f32_to_bf16_bits(np.ones((1, 2, 3, 64), np.float32))
    buf = wire.to_bytes(as_wire(kvq.pack(x, 8)))
    with pytest.raises(ValueError, match='do not match the header'):
        wire.from_bytes(buf[:-4])
    with pytest.raises(ValueError, match='Invalid packed tensor header'):
        wire.from_bytes(b'XXXX' + buf[4:])
