"""Host bindings of the sm_100a kernels (libdkv.so, C ABI in include/dkv.h).

Replaces the reference's Triton module src/gpu_kernels.py. The four launch
functions keep the Triton kernels' names and argument meaning:

  pack_rows         <- src/gpu_kernels.py:11-46
  packed_attention  <- src/gpu_kernels.py:71-105 (load_history :48-69 is fused in)
  reconstruct       <- src/gpu_kernels.py:107-119
  map_fill          <- the two map writes at src/gpu_cache.py:79-80

Each takes torch tensors, passes raw device pointers, element strides and the
current CUDA stream through ctypes, and raises ValueError (argument errors, the
reference's exception type) or RuntimeError (CUDA errors) on a non-zero status.
There is no fallback: importing this module without the built library raises.
"""
import ctypes
import functools
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent.parent / 'libdkv.so'

DKV_OK, DKV_EINVAL, DKV_ECAPACITY, DKV_EPLAN, DKV_ECUDA, DKV_ENONFINITE, DKV_EWORKSPACE, DKV_ETIMEOUT = range(8)
STATUS_NAMES = {DKV_EINVAL: 'invalid argument', DKV_ECAPACITY: 'capacity exceeded',
                DKV_EPLAN: 'bad precision code in token map', DKV_ECUDA: 'CUDA error',
                DKV_ENONFINITE: 'Nonfinite KV tensor', DKV_EWORKSPACE: 'workspace too small',
                DKV_ETIMEOUT: 'kernel pipeline wait timed out'}


_P, _I32, _I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
MAX_REQUESTS = 32  # DKV_MAX_REQUESTS


class History(ctypes.Structure):
    """dkv_history: one request's packed history for packed_attention_many."""
    _fields_ = [('p4', _P), ('m4', _P), ('p8', _P), ('m8', _P), ('p16', _P), ('rows', _P), ('codes', _P),
                ('cap4', _I64), ('cap8', _I64), ('cap16', _I64), ('past', _I32), ('capacity', _I32),
                ('status', _P)]


class PackTarget(ctypes.Structure):
    """dkv_pack_target: one request's destination for pack_rows_many."""
    _fields_ = [('p4', _P), ('m4', _P), ('p8', _P), ('m8', _P), ('p16', _P), ('cap4', _I64), ('cap8', _I64),
                ('cap16', _I64), ('row_start', _I64), ('bits', _I32), ('reserved', _I32), ('map_rows', _P),
                ('map_codes', _P), ('map_start', _I64), ('map_capacity', _I64), ('status', _P)]


def _load():
    if not _LIB_PATH.exists():
        raise ImportError(f'{_LIB_PATH} is not built; run `python __graft_entry__.py build` '
                          '(or dynamic-kv-cache_b200/build.py) first. There is no CPU fallback.')
    lib = ctypes.CDLL(str(_LIB_PATH))
    P, I32, I64, SZ, U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_uint64
    sigs = {
        'dkv_version': ([], I32),
        'dkv_last_error': ([], ctypes.c_char_p),
        'dkv_pack_rows': ([P, P, P, P, P, P, P, I64, I64, I64, I64, I32, I64, I32, I64, I64, I64,
                           I32, I32, I32, I32, P, P], ctypes.c_int),
        'dkv_packed_attention': ([P, P, P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64,
                                  I32, I32, I32, I64, I64, I64, I32, I32, I32, I32, I32, I32,
                                  P, SZ, P, P], ctypes.c_int),
        'dkv_packed_attention_workspace': ([I32, I32, I32, I32, I32], SZ),
        'dkv_packed_attention_batched': ([P, P, P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64,
                                          I32, I64, I64, I64, I64, I32, I32, I32, I64, I64, I64, I32, I32, I32,
                                          I32, I32, I32, P, SZ, P, P], ctypes.c_int),
        'dkv_packed_attention_batched_workspace': ([I32, I32, I32, I32, I32, I32], SZ),
        'dkv_packed_attention_launches': ([I32, I32, I32, I32, I32], I32),
        'dkv_reconstruct': ([P, P, P, P, P, P, P, P, I32, I32, I64, I64, I64, I32, I32, I32, P, P],
                            ctypes.c_int),
        'dkv_map_fill': ([P, P, I64, I32, I64, I32, I64, P], ctypes.c_int),
        'dkv_pack_rows_many': ([P, P, P, I32, I64, I64, I64, I64, I64, I64, I32, I32, I32, I32, I32, P],
                               ctypes.c_int),
        'dkv_packed_attention_many': ([P, P, P, P, I32, P, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64,
                                       I32, I32, I32, I32, I32, I32, P, SZ, P], ctypes.c_int),
        'dkv_packed_attention_many_workspace': ([I32, I32, I32, I32, I32, I32], SZ),
        'dkv_pack_rows_many_device': ([P, P, P, I32, I64, I64, I64, I64, I64, I64, I32, I32, I32, I32, I32, P],
                                      ctypes.c_int),
        'dkv_packed_attention_many_device': ([P, P, P, P, I32, I32, P, I64, I64, I64, I64, I64, I64, I64, I64, I64,
                                              I64, I32, I32, I32, I32, I32, I32, P, SZ, P], ctypes.c_int),
        'dkv_append_attention': ([P, P, P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I32, I32, I32, I64,
                                  I32, I32, I64, I64, I64, I64, I32, I32, I32, I32, I32, I32, P, SZ, P, P],
                                 ctypes.c_int),
        'dkv_rotary': ([P, P, P, P, I64, I64, I64, I32, I32, I32, I32, P], ctypes.c_int),
        'dkv_silu_mul': ([P, P, P, I64, I64, I64, I32, P], ctypes.c_int),
        'dkv_append_attention_many_device': ([P, P, P, P, P, I32, I32, P, I64, I64, I64, I64, I64, I64, I64, I64, I64,
                                              I64, I32, I32, I32, I32, I32, I32, P, SZ, P], ctypes.c_int),
        'dkv_pool_granularity': ([I32], U64),
        'dkv_pool_create': ([I32, U64, ctypes.POINTER(P)], ctypes.c_int),
        'dkv_pool_map': ([P, U64], ctypes.c_int),
        'dkv_pool_base': ([P], P),
        'dkv_pool_mapped_bytes': ([P], U64),
        'dkv_pool_reserved_bytes': ([P], U64),
        'dkv_pool_destroy': ([P], ctypes.c_int),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes, fn.restype = args, res
    return lib


LIB = _load()

try:  # the C++ host binding of the per-layer calls (csrc/torch_ops.cpp), built with libdkv.so
    import _dkv_torch as FAST
except ImportError as e:
    raise ImportError(f'{_LIB_PATH.with_name("_dkv_torch")}*.so is not built or does not load ({e}); run '
                      '`python __graft_entry__.py build` first. There is no CPU fallback.') from e
EXPORTS = ('dkv_version', 'dkv_last_error', 'dkv_pack_rows', 'dkv_packed_attention',
           'dkv_packed_attention_workspace', 'dkv_packed_attention_launches', 'dkv_packed_attention_batched',
           'dkv_packed_attention_batched_workspace', 'dkv_reconstruct', 'dkv_map_fill', 'dkv_pack_rows_many',
           'dkv_packed_attention_many', 'dkv_packed_attention_many_workspace', 'dkv_pack_rows_many_device',
           'dkv_packed_attention_many_device', 'dkv_append_attention', 'dkv_append_attention_many_device',
           'dkv_rotary', 'dkv_silu_mul', 'dkv_pool_granularity', 'dkv_pool_create', 'dkv_pool_map',
           'dkv_pool_base', 'dkv_pool_mapped_bytes', 'dkv_pool_reserved_bytes', 'dkv_pool_destroy')


def _check(rc):
    if rc == DKV_OK:
        return
    message = LIB.dkv_last_error().decode() or STATUS_NAMES.get(rc, f'status {rc}')
    if rc == DKV_ECUDA:
        raise RuntimeError(message)
    raise ValueError(message)


def _ptr(t):
    return None if t is None else t.data_ptr()


_RAW_STREAM = getattr(torch._C, '_cuda_getCurrentRawStream', None)


def _stream(t):
    """Handle of the current CUDA stream of t's device (the raw query when torch has
    it: a few hundred nanoseconds instead of a few microseconds per call)."""
    if _RAW_STREAM is not None:
        return _RAW_STREAM(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


def _rows_ready(x):
    """bf16 [1, heads, n, 64] view whose rows the kernels can load 16 bytes at a time."""
    if x.dtype != torch.bfloat16:
        raise ValueError('GPU kernels take bfloat16 queries, keys and values')
    ok = (x.stride(-1) == 1 and x.stride(1) % 8 == 0 and x.stride(2) % 8 == 0
          and x.data_ptr() % 16 == 0)
    return x if ok else x.contiguous()


def pack_rows(k, v, p4, m4, p8, m8, p16, layer, row_start, n, cap4, cap8, cap16, heads, dim, bits,
              layers, status=None):
    k, v = _rows_ready(k), _rows_ready(v)
    _check(LIB.dkv_pack_rows(_ptr(k), _ptr(v), _ptr(p4), _ptr(m4), _ptr(p8), _ptr(m8), _ptr(p16),
                             k.stride(1), k.stride(2), v.stride(1), v.stride(2), layer, row_start, n,
                             cap4, cap8, cap16, heads, dim, bits, layers, _ptr(status), _stream(k)))


@functools.lru_cache(maxsize=4096)
def attention_workspace_bytes(past, nq, heads, group, dim=64):
    """Workspace bytes of one packed_attention call of this shape (a pure function of
    the shape: memoised, so the per-call path makes a single library call)."""
    return LIB.dkv_packed_attention_workspace(past, nq, heads, group, dim)


def attention_launches(past, nq, heads, group, dim=64):
    """Kernel launches of one packed_attention call of this shape on the current device."""
    n = LIB.dkv_packed_attention_launches(past, nq, heads, group, dim)
    if n < 0:
        raise RuntimeError(LIB.dkv_last_error().decode() or 'CUDA error')
    return n


def _workspace(device, stream, size):
    """The attention workspace of (device, stream) with at least `size` bytes. One
    registry (in the C++ binding) serves both host paths: the library leaves the
    merge counters at a workspace's head zero after every call, so a workspace is
    zero-filled once and reused; calls on one stream never overlap, calls on other
    streams get other workspaces; outgrown ones stay referenced, so CUDA graphs
    captured with them keep valid addresses. `stream` is the current stream."""
    return FAST.workspace(torch.empty(0, device=device), size)


def packed_attention(q, knew, vnew, p4, m4, p8, m8, p16, rows, codes, out, layer, past, nq, cap4, cap8,
                     cap16, heads, group, dim, block_m, block_n, layers, status=None):
    q, knew, vnew = _rows_ready(q), _rows_ready(knew), _rows_ready(vnew)
    size = attention_workspace_bytes(past, nq, heads, group, dim)
    stream = _stream(q)
    workspace = _workspace(q.device, stream, size) if size else None
    _check(LIB.dkv_packed_attention(
        _ptr(q), _ptr(knew), _ptr(vnew), _ptr(p4), _ptr(m4), _ptr(p8), _ptr(m8), _ptr(p16), _ptr(rows),
        _ptr(codes), _ptr(out), q.stride(1), q.stride(2), knew.stride(1), knew.stride(2),
        vnew.stride(1), vnew.stride(2), layer, past, nq, cap4, cap8, cap16, heads, group, dim,
        block_m, block_n, layers, _ptr(workspace), size, _ptr(status), stream))
    return out


def packed_attention_batched(q, knew, vnew, p4, m4, p8, m8, p16, rows, codes, out, layer, past, nq, cap4, cap8,
                             cap16, heads, group, dim, block_m, block_n, layers, status=None):
    """B query chunks over one packed history: q [B, heads*group, nq, dim], knew / vnew
    [B, heads, nq, dim] (each chunk's own new rows, read natively, not appended), out
    [B, nq, heads*group, dim]. No reference counterpart (batched candidate scoring)."""
    q, knew, vnew = (_rows_ready(x) for x in (q, knew, vnew))
    chunks = q.shape[0]
    for x in (q, knew, vnew, out):
        if x.shape[0] != chunks or x.stride(0) % 8:
            raise ValueError('batched attention operands need one leading chunk dimension of 16-byte steps')
    size = LIB.dkv_packed_attention_batched_workspace(past, nq, heads, group, dim, chunks)
    stream = _stream(q)
    workspace = _workspace(q.device, stream, size) if size else None
    _check(LIB.dkv_packed_attention_batched(
        _ptr(q), _ptr(knew), _ptr(vnew), _ptr(p4), _ptr(m4), _ptr(p8), _ptr(m8), _ptr(p16), _ptr(rows),
        _ptr(codes), _ptr(out), q.stride(1), q.stride(2), knew.stride(1), knew.stride(2), vnew.stride(1),
        vnew.stride(2), chunks, q.stride(0), knew.stride(0), vnew.stride(0), out.stride(0), layer, past, nq,
        cap4, cap8, cap16, heads, group, dim, block_m, block_n, layers, _ptr(workspace), size, _ptr(status),
        stream))
    return out


def _chunked(x, name):
    if x.shape[0] and x.stride(0) % 8:
        raise ValueError(f'{name}: the request dimension must step in multiples of 8 elements')


def pack_rows_many(k, v, targets, layer, n, heads, dim, layers):
    """Frames of len(targets) requests in one launch: k / v [B, heads, n, dim] (request r
    packed into targets[r], a PackTarget). No reference counterpart (request batching)."""
    k, v = _rows_ready(k), _rows_ready(v)
    _chunked(k, 'k'), _chunked(v, 'v')
    if len(targets) != k.shape[0] or len(targets) != v.shape[0]:
        raise ValueError('one pack target per request')
    table = (PackTarget * len(targets))(*targets)
    _check(LIB.dkv_pack_rows_many(_ptr(k), _ptr(v), ctypes.addressof(table), len(targets), k.stride(1),
                                  k.stride(2), v.stride(1), v.stride(2), k.stride(0), v.stride(0), layer, n,
                                  heads, dim, layers, _stream(k)))


def packed_attention_many(q, knew, vnew, histories, out, layer, nq, heads, group, dim, layers):
    """len(histories) requests in one launch: q [B, heads*group, nq, dim] and knew / vnew
    [B, heads, nq, dim] of request r attend over histories[r] (a History); out
    [B, nq, heads*group, dim]. No reference counterpart (request batching)."""
    q, knew, vnew = (_rows_ready(x) for x in (q, knew, vnew))
    for x, name in ((q, 'q'), (knew, 'k'), (vnew, 'v'), (out, 'out')):
        if x.shape[0] != len(histories):
            raise ValueError('one history per request')
        _chunked(x, name)
    count = len(histories)
    table = (History * count)(*histories)
    size = LIB.dkv_packed_attention_many_workspace(max(h.past for h in histories), nq, heads, group, dim, count)
    stream = _stream(q)
    workspace = _workspace(q.device, stream, size) if size else None
    _check(LIB.dkv_packed_attention_many(
        _ptr(q), _ptr(knew), _ptr(vnew), ctypes.addressof(table), count, _ptr(out), q.stride(1), q.stride(2),
        knew.stride(1), knew.stride(2), vnew.stride(1), vnew.stride(2), q.stride(0), knew.stride(0),
        vnew.stride(0), out.stride(0), layer, nq, heads, group, dim, layers, _ptr(workspace), size, stream))
    return out


def pack_rows_many_device(k, v, targets_ptr, count, layer, n, heads, dim, layers):
    """pack_rows_many with the `count` PackTargets in device memory at targets_ptr
    (CUDA-graph replay reads whatever was written there before each replay)."""
    k, v = _rows_ready(k), _rows_ready(v)
    _chunked(k, 'k'), _chunked(v, 'v')
    if k.shape[0] != count or v.shape[0] != count:
        raise ValueError('one frame per request')
    _check(LIB.dkv_pack_rows_many_device(_ptr(k), _ptr(v), targets_ptr, count, k.stride(1), k.stride(2),
                                         v.stride(1), v.stride(2), k.stride(0), v.stride(0), layer, n, heads, dim,
                                         layers, _stream(k)))


def packed_attention_many_device(q, knew, vnew, histories_ptr, count, max_past, out, layer, nq, heads, group, dim,
                                 layers):
    """packed_attention_many with the `count` Histories in device memory at
    histories_ptr, planned for histories of at most max_past tokens."""
    q, knew, vnew = (_rows_ready(x) for x in (q, knew, vnew))
    for x, name in ((q, 'q'), (knew, 'k'), (vnew, 'v'), (out, 'out')):
        if x.shape[0] != count:
            raise ValueError('one history per request')
        _chunked(x, name)
    size = LIB.dkv_packed_attention_many_workspace(max_past, nq, heads, group, dim, count)
    stream = _stream(q)
    workspace = _workspace(q.device, stream, size) if size else None
    _check(LIB.dkv_packed_attention_many_device(
        _ptr(q), _ptr(knew), _ptr(vnew), histories_ptr, count, max_past, _ptr(out), q.stride(1), q.stride(2),
        knew.stride(1), knew.stride(2), vnew.stride(1), vnew.stride(2), q.stride(0), knew.stride(0),
        vnew.stride(0), out.stride(0), layer, nq, heads, group, dim, layers, _ptr(workspace), size, stream))
    return out


def append_attention(q, knew, vnew, p4, m4, p8, m8, p16, rows, codes, out, layer, past, nq, row_start, bits,
                     fill_map, map_capacity, cap4, cap8, cap16, heads, group, dim, block_m, block_n, layers,
                     status=None):
    """pack_rows (+ map_fill) and packed_attention of one frame in one launch."""
    q, knew, vnew = _rows_ready(q), _rows_ready(knew), _rows_ready(vnew)
    size = attention_workspace_bytes(past, nq, heads, group, dim)
    stream = _stream(q)
    workspace = _workspace(q.device, stream, size) if size else None
    _check(LIB.dkv_append_attention(
        _ptr(q), _ptr(knew), _ptr(vnew), _ptr(p4), _ptr(m4), _ptr(p8), _ptr(m8), _ptr(p16), _ptr(rows),
        _ptr(codes), _ptr(out), q.stride(1), q.stride(2), knew.stride(1), knew.stride(2), vnew.stride(1),
        vnew.stride(2), layer, past, nq, row_start, bits, int(fill_map), map_capacity, cap4, cap8, cap16, heads,
        group, dim, block_m, block_n, layers, _ptr(workspace), size, _ptr(status), stream))
    return out


def append_attention_many_device(q, knew, vnew, targets_ptr, histories_ptr, count, max_past, out, layer, nq, heads,
                                 group, dim, layers):
    """pack_rows_many_device + packed_attention_many_device in one launch."""
    q, knew, vnew = (_rows_ready(x) for x in (q, knew, vnew))
    for x, name in ((q, 'q'), (knew, 'k'), (vnew, 'v'), (out, 'out')):
        if x.shape[0] != count:
            raise ValueError('one history per request')
        _chunked(x, name)
    size = LIB.dkv_packed_attention_many_workspace(max_past, nq, heads, group, dim, count)
    stream = _stream(q)
    workspace = _workspace(q.device, stream, size) if size else None
    _check(LIB.dkv_append_attention_many_device(
        _ptr(q), _ptr(knew), _ptr(vnew), targets_ptr, histories_ptr, count, max_past, _ptr(out), q.stride(1),
        q.stride(2), knew.stride(1), knew.stride(2), vnew.stride(1), vnew.stride(2), q.stride(0), knew.stride(0),
        vnew.stride(0), out.stride(0), layer, nq, heads, group, dim, layers, _ptr(workspace), size, stream))
    return out


def reconstruct(p4, m4, p8, m8, p16, rows, codes, out, layer, n, cap4, cap8, cap16, heads, dim, layers,
                status=None):
    _check(LIB.dkv_reconstruct(_ptr(p4), _ptr(m4), _ptr(p8), _ptr(m8), _ptr(p16), _ptr(rows), _ptr(codes),
                               _ptr(out), layer, n, cap4, cap8, cap16, heads, dim, layers, _ptr(status),
                               _stream(out)))
    return out


def map_fill(rows, codes, start, n, row, bits, capacity):
    _check(LIB.dkv_map_fill(_ptr(rows), _ptr(codes), start, n, row, bits, capacity, _stream(rows)))


def rotary(x, cos, sin, heads):
    """Rotate-half rotary embedding of the first `heads` heads of x (bf16 [b, n, >= heads,
    64], heads contiguous) with fp32 tables cos / sin [b or 1, n, 1 or absent, 64]: one
    launch, bit-identical to the fp32 PyTorch form (x.float() * cos + rotate_half(x) * sin,
    rounded to bf16). Returns bf16 [b, n, heads, 64], contiguous."""
    if x.dtype != torch.bfloat16 or cos.dtype != torch.float32 or sin.dtype != torch.float32:
        raise ValueError('rotary takes bf16 activations and fp32 cos / sin tables')
    b, n, dim = x.shape[0], x.shape[1], x.shape[-1]
    if x.stride(-1) != 1 or x.stride(-2) != dim or x.stride(1) % 8 or x.stride(0) % 8 or x.data_ptr() % 16:
        x = x.contiguous()
    cos, sin = cos.reshape(cos.shape[0], n, dim), sin.reshape(sin.shape[0], n, dim)
    if cos.shape[0] not in (1, b) or sin.shape != cos.shape:
        raise ValueError('rotary tables must have 1 or b rows of n positions')
    cos, sin = cos.contiguous(), sin.contiguous()
    out = torch.empty((b, n, heads, dim), dtype=torch.bfloat16, device=x.device)
    cb = n * dim if cos.shape[0] > 1 else 0
    _check(LIB.dkv_rotary(_ptr(x), _ptr(cos), _ptr(sin), _ptr(out), x.stride(0), x.stride(1), cb, b, n, heads, dim,
                          _stream(x)))
    return out


def silu_mul(gate, up):
    """silu(gate) * up for bf16 gate / up of one shape [..., width] (rows with a common
    stride, e.g. the two halves of a joined gate/up projection): one launch,
    bit-identical to torch.nn.functional.silu(gate) * up. Returns a contiguous bf16
    tensor of that shape."""
    if gate.dtype != torch.bfloat16 or up.dtype != torch.bfloat16 or gate.shape != up.shape:
        raise ValueError('silu_mul takes bf16 gate and up of one shape')
    width = gate.shape[-1]
    g, u = gate.reshape(-1, width), up.reshape(-1, width)
    if g.stride(-1) != 1 or g.stride(0) % 8 or g.data_ptr() % 16:
        g = g.contiguous()
    if u.stride(-1) != 1 or u.stride(0) % 8 or u.data_ptr() % 16:
        u = u.contiguous()
    out = torch.empty(gate.shape, dtype=torch.bfloat16, device=gate.device)
    _check(LIB.dkv_silu_mul(_ptr(g), _ptr(u), _ptr(out), g.stride(0), u.stride(0), g.shape[0], width,
                            _stream(gate)))
    return out


def raise_for_status(status):
    """Reads a device status word (synchronises) and raises if a kernel reported an error."""
    code, detail = (int(x) for x in status[:2].tolist())
    if code == DKV_OK:
        return
    status.zero_()
    if code == DKV_ENONFINITE:
        raise ValueError('Nonfinite KV tensor')
    raise ValueError(f'{STATUS_NAMES.get(code, f"status {code}")} (index {detail})')


# -- growable device pools (dkv_pool_*; no reference counterpart) -----------------
# The reference grows a pool by allocating a larger tensor and copying every old
# row (src/gpu_cache.py:44-59). A region here reserves the largest size a pool can
# reach as device address space and maps memory onto its front as the pool grows
# (the pools are paged, so growth only appends pages): the base address never
# moves and nothing is copied. A region whose last user (cache, fork or tensor
# view) is gone goes to a per-device free list, memory still mapped, and the next
# reservation that fits reuses it; work the old owner queued is ordered before the
# new owner's through the stream current at release (a cache's kernels run on one
# stream, as in the reference). release_pool_memory() returns the free list's
# memory to the device.

class Region:
    """One reservation: `reserved` bytes of address space from `base`, the first
    `mapped` of them backed by device memory."""

    def __init__(self, device, handle):
        self.device, self.handle = device, handle
        self.base = LIB.dkv_pool_base(handle)
        self.reserved = LIB.dkv_pool_reserved_bytes(handle)

    @property
    def mapped(self):
        return LIB.dkv_pool_mapped_bytes(self.handle)

    def map(self, nbytes):
        """Makes the first `nbytes` usable. Mapping is a driver call that can take
        milliseconds, so a region that must grow maps at least twice what it has
        (up to its reservation) and grows rarely."""
        mapped = self.mapped
        if nbytes <= mapped:
            return
        _check(LIB.dkv_pool_map(self.handle, max(nbytes, min(self.reserved, 2 * mapped))))


class RegionLease:
    """A region in use. Dropping the last reference returns the region to the free
    list together with the stream that was current then."""

    def __init__(self, region):
        self.region = region

    def __del__(self):
        try:
            stream = torch.cuda.current_stream(self.region.device)
        except Exception:  # interpreter shutdown: the driver releases everything at exit
            return
        with _FREE_LOCK:
            _FREE.setdefault(self.region.device, []).append((self.region, stream))


_FREE = {}
_FREE_LOCK = threading.Lock()


def lease_region(device, nbytes):
    """A region of at least `nbytes` of address space on `device` (torch.device):
    from the free list the smallest fitting reservation, among equal ones the one
    with the most memory mapped already (so it rarely has to map more); else a
    new reservation."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    taken = None
    with _FREE_LOCK:
        free = _FREE.get(index, [])
        fits = [i for i, (r, _) in enumerate(free) if r.reserved >= nbytes]
        if fits:
            taken = free.pop(min(fits, key=lambda i: (free[i][0].reserved, -free[i][0].mapped)))
    if taken is not None:
        region, stream = taken
        current = torch.cuda.current_stream(index)
        if stream != current:  # the old owner's queued work first
            current.wait_stream(stream)
        return RegionLease(region)
    handle = ctypes.c_void_p()
    _check(LIB.dkv_pool_create(index, nbytes, ctypes.byref(handle)))
    return RegionLease(Region(index, handle))


def release_pool_memory():
    """Unmaps and frees every region on the free list (each release synchronises its
    device first). Regions still in use are untouched."""
    with _FREE_LOCK:
        regions = [r for free in _FREE.values() for r, _ in free]
        _FREE.clear()
    for r in regions:
        _check(LIB.dkv_pool_destroy(r.handle))


class _DeviceBytes:
    """The first `nbytes` of a leased region as a CUDA array (keeps the lease alive
    for as long as a tensor made from it)."""

    def __init__(self, lease, nbytes):
        self.lease = lease
        self.__cuda_array_interface__ = {'shape': (nbytes,), 'typestr': '|u1',
                                         'data': (lease.region.base, False), 'version': 2, 'strides': None}


def region_tensor(lease, shape, dtype):
    """A tensor of `shape` and `dtype` over the front of a leased region (no copy);
    the region must have that many bytes mapped."""
    nbytes = dtype.itemsize
    for d in shape:
        nbytes *= d
    if nbytes > lease.region.mapped:
        raise ValueError('region view beyond its mapped bytes')
    raw = torch.as_tensor(_DeviceBytes(lease, nbytes), device=torch.device('cuda', lease.region.device))
    return raw.view(dtype).view(shape)
