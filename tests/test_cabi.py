"""CPU checks of the C ABI: the library loads, exports every symbol include/dkv.h
declares, and rejects bad arguments on the host before any launch."""
import ctypes
import re

import pytest

from conftest import ROOT

HEADER = (ROOT / 'include' / 'dkv.h').read_text()
DECLARED = sorted(set(re.findall(r'^\s*(?:[\w\s\*]+?)\b(dkv_\w+)\s*\(', HEADER, re.M)))


def test_header_declares_the_hot_path_entry_points():
    for name in ('dkv_pack_rows', 'dkv_packed_attention', 'dkv_reconstruct', 'dkv_map_fill',
                 'dkv_packed_attention_workspace', 'dkv_last_error', 'dkv_version'):
        assert name in DECLARED


def test_library_exports_every_declared_symbol():
    from src import gpu_kernels as K
    raw = ctypes.CDLL(str(K._LIB_PATH))
    missing = [name for name in DECLARED if not hasattr(raw, name)]
    assert not missing, missing
    assert set(K.EXPORTS) <= set(DECLARED)
    assert K.LIB.dkv_version() == int(re.search(r'#define DKV_VERSION (\d+)', HEADER).group(1))


def _pack_args(**over):
    # Fake but 16-byte aligned "device" addresses: every call below fails in host
    # validation, before anything is dereferenced or launched.
    a = dict(k=0x1000, v=0x2000, p4=0x3000, m4=0x4000, p8=0x5000, m8=0x6000, p16=0x7000, kh=64 * 19,
             kt=64, vh=64 * 19, vt=64, layer=0, row_start=0, n=19, cap4=64, cap8=64, cap16=64, heads=3,
             dim=64, bits=4, layers=1, status=None, stream=None)
    a.update(over)
    return list(a.values())


@pytest.mark.parametrize('over,code,text', [
    (dict(dim=32), 1, 'head_dim=64'),
    (dict(bits=5), 1, 'bit widths'),
    (dict(layer=1), 1, 'layer'),
    (dict(row_start=50), 2, 'capacity'),
    (dict(kt=63), 1, 'aligned'),
    (dict(p8=None), 1, 'null pool'),
])
def test_pack_rejects_bad_arguments_on_host(over, code, text):
    from src import gpu_kernels as K
    rc = K.LIB.dkv_pack_rows(*_pack_args(**over))
    assert rc == code
    assert text in K.LIB.dkv_last_error().decode()


def test_attention_argument_checks_and_workspace_size():
    from src import gpu_kernels as K
    base = [0x1000] * 11 + [64 * 16, 64, 64 * 16, 64, 64 * 16, 64, 0, 128, 16, 64, 64, 64, 5, 3, 64]
    rc = K.LIB.dkv_packed_attention(*base, 16, 48, 1, None, 0, None, None)  # block_m=16, block_n=48
    assert rc == K.DKV_EINVAL and 'power' in K.LIB.dkv_last_error().decode()
    rc = K.LIB.dkv_packed_attention(*base, 16, 64, 1, None, 0, None, None)
    need = K.attention_workspace_bytes(128, 16, 5, 3)
    assert need > 0 and rc == K.DKV_EWORKSPACE
    assert K.attention_workspace_bytes(0, 1, 5, 3) == 0  # a single split needs no workspace
    assert K.attention_workspace_bytes(8128, 64, 5, 3) < 64 << 20


def test_map_fill_capacity_is_the_reference_context_limit_message():
    from src import gpu_kernels as K
    rc = K.LIB.dkv_map_fill(0x1000, 0x2000, 8190, 64, 0, 16, 8192, None)
    assert rc == K.DKV_ECAPACITY and K.LIB.dkv_last_error().decode() == 'GPU context limit exceeded'


def test_request_descriptor_layouts_match_the_header():
    """The C side static_asserts the same sizes and offsets (csrc/api.cu)."""
    from src import gpu_kernels as K
    assert ctypes.sizeof(K.History) == 96 and K.History.past.offset == 80 and K.History.status.offset == 88
    assert K.History.capacity.offset == 84
    assert ctypes.sizeof(K.PackTarget) == 120 and K.PackTarget.bits.offset == 72
    assert K.PackTarget.map_rows.offset == 80 and K.PackTarget.status.offset == 112
    assert K.MAX_REQUESTS == int(re.search(r'#define DKV_MAX_REQUESTS (\d+)', HEADER).group(1))


def _target(**over):
    from src import gpu_kernels as K
    a = dict(p4=0x3000, m4=0x4000, p8=0x5000, m8=0x6000, p16=0x7000, cap4=64, cap8=64, cap16=64, row_start=0,
             bits=4, reserved=0, map_rows=None, map_codes=None, map_start=0, map_capacity=0, status=None)
    a.update(over)
    return K.PackTarget(**a)


@pytest.mark.parametrize('count,over,code,text', [
    (0, {}, 1, 'request count'),
    (33, {}, 1, 'request count'),
    (2, dict(bits=5), 1, 'bit widths'),
    (2, dict(row_start=10), 2, 'capacity'),
    (1, dict(map_rows=0x8000), 1, 'half a token map'),
    (1, dict(map_rows=0x8000, map_codes=0x9000, map_start=30, map_capacity=64), 2, 'context limit'),
])
def test_pack_many_rejects_bad_arguments_on_host(count, over, code, text):
    from src import gpu_kernels as K
    table = (K.PackTarget * 33)(*[_target(**over) for _ in range(33)])
    rc = K.LIB.dkv_pack_rows_many(0x1000, 0x2000, ctypes.addressof(table), count, 64 * 64, 64, 64 * 64, 64,
                                  5 * 64 * 64, 5 * 64 * 64, 0, 64, 5, 64, 1, None)
    assert rc == code
    assert text in K.LIB.dkv_last_error().decode()


def test_attention_many_rejects_bad_arguments_on_host():
    from src import gpu_kernels as K
    h = K.History(0x3000, 0x4000, 0x5000, 0x6000, 0x7000, 0x8000, 0x9000, 64, 64, 64, 100, 128, None)
    table = (K.History * 2)(h, h)
    args = [0x1000, 0x2000, 0x3000, ctypes.addressof(table)]
    rest = [0xA000, 64 * 64, 64, 64 * 64, 64, 64 * 64, 64, 15 * 64 * 64, 5 * 64 * 64, 5 * 64 * 64, 15 * 64 * 64,
            0, 64, 5, 3, 64, 1, None, 0, None]
    rc = K.LIB.dkv_packed_attention_many(*args, 0, *rest)
    assert rc == K.DKV_EINVAL and 'request count' in K.LIB.dkv_last_error().decode()
    # this shape splits its history, so the missing workspace stops the call before any launch
    assert K.LIB.dkv_packed_attention_many_workspace(100, 64, 5, 3, 64, 2) > 0
    rc = K.LIB.dkv_packed_attention_many(*args, 2, *rest)
    assert rc == K.DKV_EWORKSPACE
    table[1].past = 129
    rc = K.LIB.dkv_packed_attention_many(*args, 2, *rest)
    assert rc == K.DKV_EINVAL and 'exceeds its token map' in K.LIB.dkv_last_error().decode()
    table[1].past = -1
    rc = K.LIB.dkv_packed_attention_many(*args, 2, *rest)
    assert rc == K.DKV_EINVAL and 'negative' in K.LIB.dkv_last_error().decode()
    # device-resident tables: only what the host can see is checked before the launch
    dev = [0x1000, 0x2000, 0x3000, 0x10008, 2, 100]  # table address not 16-byte aligned
    rc = K.LIB.dkv_packed_attention_many_device(*dev, *rest)
    assert rc == K.DKV_EINVAL and 'aligned' in K.LIB.dkv_last_error().decode()
    rc = K.LIB.dkv_pack_rows_many_device(0x1000, 0x2000, 0x10008, 2, 64 * 64, 64, 64 * 64, 64, 5 * 64 * 64,
                                         5 * 64 * 64, 0, 64, 5, 64, 1, None)
    assert rc == K.DKV_EINVAL and 'aligned' in K.LIB.dkv_last_error().decode()


def _append_args(**over):
    # Fake, 16-byte aligned addresses: every case below fails host validation first.
    a = dict(q=0x1000, knew=0x2000, vnew=0x3000, p4=0x4000, m4=0x5000, p8=0x6000, m8=0x7000, p16=0x8000,
             rows=0x9000, codes=0xA000, out=0xB000, qh=64 * 64, qt=64, kh=64 * 64, kt=64, vh=64 * 64, vt=64,
             layer=0, past=128, nq=64, row_start=0, bits=4, fill_map=1, map_capacity=4096, cap4=256, cap8=256,
             cap16=256, heads=5, group=3, dim=64, block_m=16, block_n=64, layers=1, workspace=None, ws=0,
             status=None, stream=None)
    a.update(over)
    return list(a.values())


@pytest.mark.parametrize('over,code,text', [
    (dict(bits=5), 1, 'bit widths'),
    (dict(row_start=200), 2, 'capacity'),
    (dict(rows=None), 1, 'null token map'),
    (dict(map_capacity=150), 2, 'context limit'),
    (dict(dim=128), 1, 'head_dim=64'),
    (dict(p16=None), 1, 'null pool'),
])
def test_append_attention_rejects_bad_arguments_on_host(over, code, text):
    from src import gpu_kernels as K
    rc = K.LIB.dkv_append_attention(*_append_args(**over))
    assert rc == code
    assert text in K.LIB.dkv_last_error().decode()


def test_append_attention_many_device_rejects_unaligned_tables():
    from src import gpu_kernels as K
    rest = [0xB000, 64 * 64, 64, 64 * 64, 64, 64 * 64, 64, 15 * 64 * 64, 5 * 64 * 64, 5 * 64 * 64, 15 * 64 * 64,
            0, 64, 5, 3, 64, 1, None, 0, None]
    rc = K.LIB.dkv_append_attention_many_device(0x1000, 0x2000, 0x3000, 0x10008, 0x20000, 2, 100, *rest)
    assert rc == K.DKV_EINVAL and 'aligned' in K.LIB.dkv_last_error().decode()
    rc = K.LIB.dkv_append_attention_many_device(0x1000, 0x2000, 0x3000, 0x10000, 0x20000, 0, 100, *rest)
    assert rc == K.DKV_EINVAL and 'request count' in K.LIB.dkv_last_error().decode()


@pytest.mark.parametrize('over,text', [
    (dict(dim=32), 'head_dim=64'),
    (dict(heads=0), 'no heads'),
    (dict(x=0x1008), 'aligned'),
    (dict(xt=20 * 64 - 8), 'token strides'),
    (dict(xb=12), 'token strides'),
    (dict(cb=6), 'batch stride'),
    (dict(cos=None), 'null pointer'),
])
def test_rotary_rejects_bad_arguments_on_host(over, text):
    from src import gpu_kernels as K
    a = dict(x=0x1000, cos=0x2000, sin=0x3000, out=0x4000, xb=64 * 25 * 8, xt=25 * 64, cb=8 * 64, b=2, n=8,
             heads=20, dim=64, stream=None)
    a.update(over)
    assert K.LIB.dkv_rotary(*a.values()) == K.DKV_EINVAL
    assert text in K.LIB.dkv_last_error().decode()
    a.update(b=0)  # an empty call is a no-op once the shape checks pass
    if 'dim' not in over and 'heads' not in over:
        assert K.LIB.dkv_rotary(*a.values()) == K.DKV_OK


@pytest.mark.parametrize('over,text', [
    (dict(width=12), 'multiple of 8'),
    (dict(width=0), 'multiple of 8'),
    (dict(up=0x2004), 'aligned'),
    (dict(gs=2552), 'row strides'),
    (dict(us=5124), 'row strides'),
    (dict(out=None), 'null pointer'),
])
def test_silu_mul_rejects_bad_arguments_on_host(over, text):
    from src import gpu_kernels as K
    a = dict(gate=0x1000, up=0x2000, out=0x3000, gs=5120, us=5120, rows=7, width=2560, stream=None)
    a.update(over)
    assert K.LIB.dkv_silu_mul(*a.values()) == K.DKV_EINVAL
    assert text in K.LIB.dkv_last_error().decode()
