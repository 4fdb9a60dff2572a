"""Device-resident pool growth: each pool reserves the address space of the largest
capacity its cache can reach and maps memory as it grows (dkv_pool_*), so growth
keeps the pool's address and copies no row. The capacities follow the reference's
policy (src/gpu_cache.py:44-59) exactly; the rows written before a growth read
back bit-identical after it, and attention over a history that grew many times
matches the oracle."""
import ctypes

import pytest
import torch

from dkv_testlib import assert_attention_close, oracle_attention, oracle_frames, outlier_kv

pytestmark = pytest.mark.gpu


def test_pool_c_abi_reserve_map_destroy(cuda):
    from src import gpu_kernels as K
    lib = K.LIB
    g = lib.dkv_pool_granularity(0)
    assert g > 0 and g % 4096 == 0
    h = ctypes.c_void_p()
    assert lib.dkv_pool_create(0, 3 * g + 1, ctypes.byref(h)) == K.DKV_OK
    assert lib.dkv_pool_reserved_bytes(h) == 4 * g and lib.dkv_pool_mapped_bytes(h) == 0
    base = lib.dkv_pool_base(h)
    assert lib.dkv_pool_map(h, 1) == K.DKV_OK and lib.dkv_pool_mapped_bytes(h) == g
    assert lib.dkv_pool_map(h, 2 * g + 5) == K.DKV_OK and lib.dkv_pool_mapped_bytes(h) == 3 * g
    assert lib.dkv_pool_map(h, g) == K.DKV_OK and lib.dkv_pool_mapped_bytes(h) == 3 * g  # never shrinks
    assert lib.dkv_pool_base(h) == base
    assert lib.dkv_pool_map(h, 5 * g) == K.DKV_ECAPACITY  # beyond the reservation: refused, nothing mapped
    assert lib.dkv_pool_mapped_bytes(h) == 3 * g
    lease = K.RegionLease(K.Region(0, h))
    t = K.region_tensor(lease, (3 * g // 4,), torch.float32)
    t.fill_(1.5)
    assert t.data_ptr() == base and float(t.sum()) == 1.5 * t.numel()
    del t, lease  # back to the free list (not destroyed)
    K.release_pool_memory()


def test_growth_keeps_addresses_and_rows(cuda):
    from src.gpu_cache import GPUCache
    gen = torch.Generator().manual_seed(5)
    c = GPUCache(None, layers=2, heads=3, max_tokens=4096)
    ptrs = {n: getattr(c, n).data_ptr() for n in ('p4', 'm4', 'p8', 'm8', 'p16')}
    caps_seen, snapshots = [], []
    for f in range(40):  # 40 frames of 64 tokens: every pool grows several times
        bits = (4, 8, 16, 4, 8)[f % 5]
        k = torch.randn(1, 3, 64, 64, generator=gen).bfloat16().cuda()
        v = torch.randn(1, 3, 64, 64, generator=gen).bfloat16().cuda()
        c.select(bits, f)
        for layer in range(2):
            c.append(k, v, layer)
        caps_seen.append(dict(c.caps))
        if f == 3:  # rows of the first frames, before any growth beyond the first page
            snapshots = [(n, c.pool_rows(n, 1, kv, 0, 64).clone()) for n in ('p4', 'm4', 'p16') for kv in (0, 1)]
    c.check()
    assert {n: getattr(c, n).data_ptr() for n in ptrs} == ptrs  # no pool moved
    assert c.caps[4] > 64 and c.caps[8] > 64 and c.caps[16] > 64
    # the reference's growth sequence for 16 / 16 / 8 frames of each precision
    expected = {4: 64, 8: 64, 16: 64}
    for f in range(40):
        bits = (4, 8, 16, 4, 8)[f % 5]
        used = sum(64 for g in range(f + 1) if (4, 8, 16, 4, 8)[g % 5] == bits)
        old = expected[bits]
        if used > old:
            expected[bits] = max(used, ((int(old * 1.5) + 63) // 64) * 64)
        assert caps_seen[f] == expected
    for i, (n, before) in enumerate(snapshots):
        assert torch.equal(c.pool_rows(n, 1, i % 2, 0, 64), before)  # rows stayed where they were


def test_attention_over_a_history_that_grew(cuda):
    from src.gpu_cache import GPUCache
    gen = torch.Generator().manual_seed(11)
    outliers = torch.randperm(64, generator=gen)[:4]
    past = 3000
    plan = [((4, 8, 16)[f % 3] if f % 7 else 8, min(64, past - 64 * f)) for f in range((past + 63) // 64)]
    hist_k, hist_v = outlier_kv(gen, 5, past, outliers)
    c = GPUCache(None, layers=1, heads=5, max_tokens=past + 64)
    start = 0
    for f, (b, n) in enumerate(plan):
        c.select(b, f)
        c.append(hist_k[:, :, start:start + n].cuda(), hist_v[:, :, start:start + n].cuda(), 0)
        start += n
    frames = oracle_frames(hist_k, hist_v, plan)
    for nq in (1, 64):
        q = torch.randn(1, 15, nq, 64, generator=gen).bfloat16()
        kn, vn = outlier_kv(gen, 5, nq, outliers)
        out = c.attend(q.cuda(), kn.cuda(), vn.cuda(), 0, past)
        c.check()
        assert_attention_close(out, oracle_attention(frames, q, kn, vn), atol=0.01, rtol=0.01)


def test_released_regions_are_reused(cuda):
    from src import gpu_kernels as K
    from src.gpu_cache import GPUCache
    K.release_pool_memory()
    a = GPUCache(None, layers=2, heads=3, max_tokens=1024)
    ptr = a.p16.data_ptr()
    del a
    b = GPUCache(None, layers=2, heads=3, max_tokens=1024)  # same geometry: a region from the free list
    assert b.p16.data_ptr() == ptr
    k = torch.randn(1, 3, 64, 64).bfloat16().cuda()
    b.select(16, 0)
    b.append(k, k, 0)
    b.check()
    assert torch.equal(b.pool_rows('p16', 0, 0, 0, 64), k[0])


def test_fork_growth_leaves_the_base(cuda):
    from src.gpu_cache import GPUCache
    c = GPUCache(None, layers=1, heads=3, max_tokens=2048)
    k = torch.randn(1, 3, 64, 64).bfloat16().cuda()
    c.select(8, 0)
    c.append(k, k, 0)
    base_rows = c.pool_rows('p8', 0, 0, 0, 64).clone()
    b = c.fork()
    for f in range(1, 6):  # the branch grows the shared 8-bit pool several times
        b.select(8, f)
        b.append(torch.randn(1, 3, 64, 64).bfloat16().cuda(), k, 0)
    assert b.caps[8] > 64 and c.caps[8] == 64 and c.p8.shape[0] == 1
    assert b.p8.data_ptr() == c.p8.data_ptr()  # one region, the branch's view is longer
    assert torch.equal(c.pool_rows('p8', 0, 0, 0, 64), base_rows)
    c.check()
    b.check()


def test_reserve_beyond_the_reservation_moves_once_and_keeps_rows(cuda):
    """An explicit reserve() past what the cache's token capacity can need (the
    reference allows any size) outgrows the reserved address space: the pool moves
    to a larger region once, its rows copied, and everything keeps working."""
    from src.gpu_cache import GPUCache
    gen = torch.Generator().manual_seed(21)
    c = GPUCache(None, layers=1, heads=5, max_tokens=256)
    k = torch.randn(1, 5, 64, 64, generator=gen).bfloat16().cuda()
    v = torch.randn(1, 5, 64, 64, generator=gen).bfloat16().cuda()
    c.select(16, 0)
    c.append(k, v, 0)
    before = c.pool_rows('p16', 0, 0, 0, 64).clone()
    ptr = c.p16.data_ptr()
    c.reserve(16, 5000)  # far beyond ceil64(1.5 * 256) rows
    assert c.caps[16] == 5000 and c.p16.data_ptr() != ptr and c.p16.shape[0] == (5000 + 63) // 64
    assert torch.equal(c.pool_rows('p16', 0, 0, 0, 64), before)
    q = torch.randn(1, 15, 8, 64, generator=gen).bfloat16().cuda()
    kn = torch.randn(1, 5, 8, 64, generator=gen).bfloat16().cuda()
    out = c.attend(q, kn, kn, 0, 64)
    ref = GPUCache(None, layers=1, heads=5, max_tokens=256)
    ref.select(16, 0)
    ref.append(k, v, 0)
    assert torch.equal(out, ref.attend(q, kn, kn, 0, 64))
    c.check()
