"""The reference's packed-tensor wire format for frames held in a GPUCache.

PackedTensor mirrors src/kv_quantization.py:15-39 (zoaibs/Dynamic-KV-Cache): a
64-byte header '<4sBBBB4qQQQ' (magic 'DKVC', version 1, bits, dtype code, ndim,
shape[4], group size, numel, groups; :12-13), the payload (4-bit codes two per
byte with the even element in the low nibble, 8-bit codes, or raw bf16 bytes) and
per-group float32 scales and offsets (:41-77). One layer's K (or V) of a frame is
[1, heads, n, 64] with group size 64 = head_dim, so each group is one pool row and
one (offset, scale) pair of the device pools: export and import are gathers and
scatters of pool rows, no requantisation. Export returns byte for byte what the
reference's pack() returns for the same bf16 tensor (the device quantiser is
bit-exact with it); import lets a cache adopt frames packed on the CPU.

to_bytes / from_bytes concatenate header, payload, scales and offsets (float32
little-endian): the reference keeps the four tensors separately, this is their
flat on-disk form.
"""
from dataclasses import dataclass
import struct

import torch

HEADER = struct.Struct('<4sBBBB4qQQQ')  # src/kv_quantization.py:12
DTYPES = {torch.float16: 1, torch.bfloat16: 2, torch.float32: 3}  # :13
GROUP = 64


@dataclass
class PackedTensor:
    payload: torch.Tensor  # uint8
    scales: torch.Tensor   # float32 [groups]
    offsets: torch.Tensor  # float32 [groups]
    header: torch.Tensor   # uint8 [64]

    def fields(self):
        magic, version, bits, dtype, ndim, *other = HEADER.unpack(bytes(self.header.tolist()))
        if magic != b'DKVC' or version != 1:
            raise ValueError('Invalid packed tensor header')
        shape, group, numel, groups = tuple(other[:ndim]), other[4], other[5], other[6]
        return bits, dtype, shape, group, numel, groups

    @property
    def payload_bytes(self):
        return self.payload.numel() * self.payload.element_size()

    @property
    def metadata_bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.scales, self.offsets, self.header))

    @property
    def storage_bytes(self):
        return self.payload_bytes + self.metadata_bytes


def to_bytes(packed):
    return b''.join((bytes(packed.header.tolist()), packed.payload.numpy().tobytes(),
                     packed.scales.to(torch.float32).numpy().astype('<f4').tobytes(),
                     packed.offsets.to(torch.float32).numpy().astype('<f4').tobytes()))


def from_bytes(buf):
    header = torch.tensor(list(buf[:HEADER.size]), dtype=torch.uint8)
    probe = PackedTensor(torch.empty(0, dtype=torch.uint8), torch.empty(0), torch.empty(0), header)
    bits, dtype, shape, group, numel, groups = probe.fields()
    if bits == 16:
        size = numel * 2
    else:
        size = (numel + 1) // 2 if bits == 4 else numel
    end = HEADER.size + size
    if len(buf) != end + 8 * groups:
        raise ValueError('Packed tensor bytes do not match the header')
    payload = torch.frombuffer(bytearray(buf[HEADER.size:end]), dtype=torch.uint8)
    meta = torch.frombuffer(bytearray(buf[end:]), dtype=torch.float32) if groups else torch.empty(0)
    return PackedTensor(payload, meta[:groups].clone(), meta[groups:].clone(), header)


def _header(bits, heads, n, dim):
    numel = heads * n * dim
    groups = 0 if bits == 16 else numel // GROUP
    raw = HEADER.pack(b'DKVC', 1, bits, DTYPES[torch.bfloat16], 4, 1, heads, n, dim, GROUP, numel, groups)
    return torch.tensor(list(raw), dtype=torch.uint8)


def export_segment(cache, layer, index):
    """K and V of plan segment `index` (one frame) of `layer` as PackedTensors on the
    CPU: what the reference's pack(k_frame, bits) / pack(v_frame, bits) return."""
    start, end, bits, row = cache.plan[index]
    n = min(end, cache.seen[layer]) - start
    if n <= 0:
        raise ValueError(f'layer {layer} holds no tokens of segment {index}')
    out = []
    for kv in (0, 1):
        if bits == 16:
            payload = cache.pool_rows('p16', layer, kv, row, n).contiguous().view(torch.uint8).flatten().cpu()
            scales = offsets = torch.empty(0, dtype=torch.float32)
        else:
            pool, meta = ('p4', 'm4') if bits == 4 else ('p8', 'm8')
            payload = cache.pool_rows(pool, layer, kv, row, n).contiguous().flatten().cpu()
            pairs = cache.pool_rows(meta, layer, kv, row, n).reshape(-1, 2).cpu()
            offsets, scales = pairs[:, 0].contiguous(), pairs[:, 1].contiguous()
        out.append(PackedTensor(payload, scales, offsets, _header(bits, cache.heads, n, cache.dim)))
    return tuple(out)


def import_frame(cache, k_packed, v_packed, layer):
    """Appends a frame given as the reference's PackedTensors (K and V of one layer,
    [1, heads, n, 64], packed at the cache's selected precision) without
    requantising: the same bookkeeping as GPUCache.append, then the pool rows are
    copied in. Returns the history length before the frame."""
    fields = []
    for packed in (k_packed, v_packed):
        bits, dtype, shape, group, numel, groups = packed.fields()
        if shape != (1, cache.heads, shape[2], cache.dim) or group != GROUP or numel != cache.heads * shape[2] * cache.dim:
            raise ValueError('Packed frame does not match the cache geometry')
        if bits != cache.pending_bits:
            raise ValueError(f'Packed frame has {bits} bits, the cache selected {cache.pending_bits}')
        if bits == 16 and dtype != DTYPES[torch.bfloat16]:
            raise ValueError('GPU kernel stores 16-bit rows as bfloat16')
        if bits != 16 and groups != numel // GROUP:
            raise ValueError('Packed frame has the wrong group count')
        fields.append((bits, shape[2]))
    if fields[0] != fields[1]:
        raise ValueError('K and V frames differ in precision or length')
    bits, n = fields[0]
    past, n, row = cache._claim(layer, n)
    dev = cache.device
    for kv, packed in enumerate((k_packed, v_packed)):
        if bits == 16:
            rows = packed.payload.view(torch.bfloat16).reshape(cache.heads, n, cache.dim)
            cache.write_pool_rows('p16', layer, kv, row, rows.to(dev))
        else:
            pool, meta = ('p4', 'm4') if bits == 4 else ('p8', 'm8')
            cache.write_pool_rows(pool, layer, kv, row, packed.payload.reshape(cache.heads, n, -1).to(dev))
            pairs = torch.stack((packed.offsets, packed.scales), dim=-1).reshape(cache.heads, n, 2)
            cache.write_pool_rows(meta, layer, kv, row, pairs.to(dev))
    cache.seen[layer] = past + n
    return past
