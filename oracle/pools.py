"""TEST INFRASTRUCTURE ONLY — host model of the GPU pool layout.

Maps oracle pack output (kvq.Packed, groups over the flattened [1, H, n, 64]
tensor) onto the reference's per-row GPU pools (src/gpu_cache.py:36-41):
group g = head * n + token is exactly one 64-wide (head, token) row, stored at
pool row `row_start + token` of block (layer, K|V, head); metadata is the
(offset, scale) fp32 pair per row (src/gpu_kernels.py:40-41,45-46).
"""
import numpy as np

from . import kvq

ROW_BYTES = {4: 32, 8: 64, 16: 128}


def frame_rows(packed, heads, n):
    """(payload rows uint8 [heads, n, row_bytes], meta float32 [heads, n, 2] or None)."""
    bits = packed.fields()[0]
    payload = packed.payload.reshape(heads, n, ROW_BYTES[bits])
    if bits == 16:
        return payload, None
    meta = np.stack([packed.offsets, packed.scales], axis=-1).reshape(heads, n, 2).astype(np.float32)
    return payload, meta


class HostPools:
    """Byte-level pools for one layer-set; layout [layers, 2, heads, cap, ...]."""

    def __init__(self, layers, heads, caps):
        self.layers, self.heads, self.caps = layers, heads, dict(caps)
        self.payload = {b: np.zeros((layers, 2, heads, caps[b], ROW_BYTES[b]), np.uint8) for b in (4, 8, 16)}
        self.meta = {b: np.zeros((layers, 2, heads, caps[b], 2), np.float32) for b in (4, 8)}

    def write(self, layer, kv, bits, row_start, packed, n):
        payload, meta = frame_rows(packed, self.heads, n)
        self.payload[bits][layer, kv, :, row_start:row_start + n] = payload
        if meta is not None:
            self.meta[bits][layer, kv, :, row_start:row_start + n] = meta


def plan_rows(plan):
    """Offline plan [(bits, n), ...] -> (segments, rows, codes) as src/gpu_cache.py:23-29."""
    counts = {4: 0, 8: 0, 16: 0}
    segments, rows, codes = [], [], []
    for bits, n in plan:
        segments.append((len(rows), len(rows) + n, bits, counts[bits]))
        rows.extend(range(counts[bits], counts[bits] + n))
        codes.extend([bits] * n)
        counts[bits] += n
    return segments, np.array(rows, np.int32), np.array(codes, np.uint8), counts


def pack_frame(k_bits, v_bits, bits):
    """Oracle-packs one frame's K and V ([1, H, n, 64] bf16 bit patterns)."""
    return kvq.pack(k_bits, bits), kvq.pack(v_bits, bits)
