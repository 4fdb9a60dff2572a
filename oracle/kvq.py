"""TEST INFRASTRUCTURE ONLY — numpy restatement of the reference quantiser.

Follows src/kv_quantization.py (zoaibs/Dynamic-KV-Cache):
  HEADER '<4sBBBB4qQQQ' (64 bytes, magic 'DKVC', version 1)      :12-13
  pack(tensor, bits, group_size=64)                             :41-77
  unpack(packed)                                                 :79-92

Every step is float32 with IEEE round-to-nearest, in the reference's order:
offsets = group min, spans = max - offsets, scales = spans / (2^bits - 1) (1 for a
zero span), q = round_half_even((x - offset) / scale) clamped to [0, 2^bits - 1];
4-bit codes are packed two per byte, even element in the low nibble. bf16 data is
carried as raw uint16 bit patterns (numpy has no bfloat16).
"""
from dataclasses import dataclass
import math
import struct

import numpy as np

HEADER = struct.Struct('<4sBBBB4qQQQ')
DTYPE_CODES = {'float16': 1, 'bfloat16': 2, 'float32': 3}
CODE_DTYPES = {v: k for k, v in DTYPE_CODES.items()}


def bf16_bits_to_f32(bits):
    """Exact widening of bf16 bit patterns (uint16) to float32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x):
    """float32 -> bf16 bit patterns with round-to-nearest-even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + rounding) >> 16).astype(np.uint16)


def as_float32(x, dtype):
    if dtype == 'bfloat16':
        return bf16_bits_to_f32(x)
    return np.asarray(x).astype(np.float32)


@dataclass
class Packed:
    payload: np.ndarray   # uint8
    scales: np.ndarray    # float32 [groups]
    offsets: np.ndarray   # float32 [groups]
    header: np.ndarray    # uint8 [64]

    def fields(self):
        magic, version, bits, dtype, ndim, *other = HEADER.unpack(self.header.tobytes())
        if magic != b'DKVC' or version != 1:
            raise ValueError('Invalid packed tensor header')
        shape, group, numel, groups = tuple(other[:ndim]), other[4], other[5], other[6]
        return bits, dtype, shape, group, numel, groups


def pack(x, bits, group_size=64, dtype='bfloat16'):
    """Quantises a [batch, heads, tokens, head_dim] array. `x` holds bf16 bit
    patterns (uint16) when dtype == 'bfloat16', else float16/float32 values."""
    if bits not in (4, 8, 16) or group_size <= 0:
        raise ValueError('Supported bit widths: 4, 8, 16; positive group size required')
    x = np.ascontiguousarray(x)
    if x.ndim != 4 or x.size == 0 or dtype not in DTYPE_CODES:
        raise ValueError('Expected nonempty [batch, heads, tokens, head_dim] float tensor')
    values = as_float32(x, dtype)
    if not np.isfinite(values).all():
        raise ValueError('Nonfinite KV tensor')
    if bits == 16:
        if dtype == 'float32':  # the reference keeps 16-bit payloads as fp16 (:51-52)
            x, dtype = values.astype(np.float16), 'float16'
        payload = np.frombuffer(x.astype(x.dtype.newbyteorder('<')).tobytes(), dtype=np.uint8).copy()
        scales = offsets = np.empty(0, dtype=np.float32)
        groups = 0
    else:
        flat = values.reshape(-1)
        numel = flat.size
        groups = math.ceil(numel / group_size)
        if numel % group_size:  # replicate the last value into the padding (:59-61)
            flat = np.concatenate([flat, np.repeat(flat[-1:], groups * group_size - numel)])
        grouped = flat.reshape(groups, group_size)
        offsets = grouped.min(axis=1)
        spans = (grouped.max(axis=1) - offsets).astype(np.float32)
        levels = np.float32((1 << bits) - 1)
        with np.errstate(divide='ignore', invalid='ignore', over='ignore'):
            scales = np.where(spans > 0, spans / levels, np.float32(1)).astype(np.float32)
            q = np.rint((grouped - offsets[:, None]) / scales[:, None])
        q = np.clip(q, 0, (1 << bits) - 1)
        q = np.nan_to_num(q, nan=0.0).astype(np.uint8).reshape(-1)[:numel]
        if bits == 4:
            if q.size % 2:
                q = np.concatenate([q, np.zeros(1, np.uint8)])
            payload = (q[0::2] | (q[1::2] << 4)).astype(np.uint8)
        else:
            payload = q
    raw = HEADER.pack(b'DKVC', 1, bits, DTYPE_CODES[dtype], x.ndim, *x.shape, group_size, x.size, groups)
    return Packed(payload, scales.astype(np.float32), offsets.astype(np.float32),
                  np.frombuffer(raw, dtype=np.uint8).copy())


def codes_of(packed):
    """Unpacked integer codes (uint8, one per element) of a 4/8-bit Packed."""
    bits, _, _, _, numel, _ = packed.fields()
    if bits == 4:
        return np.stack([packed.payload & 15, packed.payload >> 4], axis=-1).reshape(-1)[:numel]
    return packed.payload[:numel]


def unpack(packed):
    """Dequantised float32 values with the stored shape (:79-92): 16-bit payloads
    are widened exactly; 4/8-bit use fp32 q*scale then + offset (two roundings)."""
    bits, dtype, shape, group_size, numel, groups = packed.fields()
    name = CODE_DTYPES[dtype]
    if bits == 16:
        if name == 'bfloat16':
            return bf16_bits_to_f32(packed.payload.view('<u2')).reshape(shape)
        return packed.payload.view('<f2').astype(np.float32).reshape(shape)
    q = codes_of(packed).astype(np.float32)
    q = np.concatenate([q, np.zeros(groups * group_size - numel, np.float32)]).reshape(groups, group_size)
    x = (q * packed.scales[:, None]).astype(np.float32) + packed.offsets[:, None]
    return x.astype(np.float32).reshape(-1)[:numel].reshape(shape)
