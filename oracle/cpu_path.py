"""TEST INFRASTRUCTURE ONLY — the reference's CPU cache path, restated in torch.

MixedPrecisionCache.update (src/cache_manager.py:43-63) dequantises every stored
frame with unpack (src/kv_quantization.py:79-92), keeps the current frame's K/V
native, concatenates, and the decoder's attention runs torch SDPA over it. The
mask and GQA expansion follow the reference's own checks
(tests/test_gpu_backend.py:97-100, scripts/test_gpu_backend.py:8-10): key t is
visible to query m iff t <= past + m, KV heads repeated `group` times.

Used as (1) the attention oracle of the parity tests and (2) the timed CPU
baseline of bench.py (kind "port": the reference's path on the host cores;
cpu_cache_update is the whole per-call update, the current frame's pack included).
"""
import numpy as np
import torch
import torch.nn.functional as F

from . import kvq


def unpack_torch(packed, dtype=torch.float32, memo=False):
    """torch restatement of unpack: 16-bit payloads are reinterpreted; 4/8-bit codes
    are dequantised as q * scale + offset in fp32, then cast to `dtype`. memo=True
    (the oracle decoder, never the timed baseline, which must pay every unpack as
    the reference does) keeps the fp32 result on the Packed object, so a stored
    segment is unpacked once however many later calls read it."""
    if not memo:
        return _unpack_torch(packed).to(dtype)
    cached = getattr(packed, '_unpacked', None)
    if cached is None:
        cached = _unpack_torch(packed)
        packed._unpacked = cached
    return cached.to(dtype)


def _unpack_torch(packed):
    dtype = torch.float32
    bits, code, shape, group, numel, groups = packed.fields()
    payload = torch.from_numpy(packed.payload)
    if bits == 16:
        source = torch.bfloat16 if kvq.CODE_DTYPES[code] == 'bfloat16' else torch.float16
        return payload.view(source).reshape(shape).to(dtype)
    if bits == 4:
        q = torch.stack((payload & 15, payload >> 4), dim=-1).flatten()[:numel]
    else:
        q = payload
    q = F.pad(q, (0, groups * group - numel)).float().reshape(groups, group)
    x = q * torch.from_numpy(packed.scales)[:, None] + torch.from_numpy(packed.offsets)[:, None]
    return x.flatten()[:numel].reshape(shape).to(dtype)


def reference_attention(q, hist_k, hist_v, knew, vnew):
    """q [1, HQ, n, D]; hist_* [1, H, past, D]; knew/vnew [1, H, n, D] (float tensors).
    Returns [1, n, HQ, D] in fp32."""
    past, n = hist_k.shape[2], q.shape[2]
    group = q.shape[1] // hist_k.shape[1]
    k = torch.cat((hist_k, knew), dim=2).float().repeat_interleave(group, 1)
    v = torch.cat((hist_v, vnew), dim=2).float().repeat_interleave(group, 1)
    mask = torch.arange(past + n)[None, :] <= past + torch.arange(n)[:, None]
    out = F.scaled_dot_product_attention(q.float(), k, v, attn_mask=mask)
    return out.transpose(1, 2)


def cpu_cache_attention(frames, q, knew, vnew, round_history_bf16=False, memo=False):
    """The reference CPU path for one layer: `frames` is a list of (K Packed,
    V Packed) per stored frame; dequantise all, append the native current frame
    and attend. round_history_bf16 mimics dequantised history held in bf16, as
    the GPU kernel's tiles are (src/gpu_kernels.py:93-94); memo as unpack_torch."""
    ks = [unpack_torch(k, memo=memo) for k, _ in frames]
    vs = [unpack_torch(v, memo=memo) for _, v in frames]
    if not ks:
        empty = torch.zeros(1, knew.shape[1], 0, knew.shape[3])
        ks, vs = [empty], [empty]
    hist_k, hist_v = torch.cat(ks, dim=2), torch.cat(vs, dim=2)
    if round_history_bf16:
        hist_k, hist_v = hist_k.bfloat16().float(), hist_v.bfloat16().float()
    return reference_attention(q, hist_k, hist_v, knew, vnew)


def cpu_cache_update(frames, q, knew, vnew, bits):
    """One layer's call of the reference CPU cache path in full, as
    MixedPrecisionCache.update (src/cache_manager.py:43-63) and the attention
    after it run it: dequantise every stored frame, pack the current frame's K and
    V at `bits` (the compressed copy the next call reads; its result does not enter
    this call's output), concatenate with the native current frame and attend.
    knew / vnew are float32 tensors, packed as the reference packs float32 inputs.
    Returns (attention output [1, n, HQ, D], (K Packed, V Packed) of the frame)."""
    out = cpu_cache_attention(frames, q, knew, vnew)
    packed = (kvq.pack(knew.contiguous().numpy().astype(np.float32), bits, dtype='float32'),
              kvq.pack(vnew.contiguous().numpy().astype(np.float32), bits, dtype='float32'))
    return out, packed
