"""The C++ host binding (csrc/torch_ops.cpp) that GPUCache.append / attend /
append_attend use makes the same C-ABI calls as the ctypes binding: pools and
outputs must be bit-identical between the two paths, and argument errors must
keep the reference's exception type."""
import pytest
import torch

from dkv_testlib import outlier_kv

pytestmark = pytest.mark.gpu


def _cache_pair(seed, past, heads=5):
    from src.gpu_cache import GPUCache
    gen = torch.Generator().manual_seed(seed)
    outliers = torch.randperm(64, generator=gen)[:4]
    hk, hv = outlier_kv(gen, heads, past, outliers)
    caches = [GPUCache(None, layers=2, heads=heads, max_tokens=past + 128) for _ in range(2)]
    return gen, outliers, hk.cuda(), hv.cuda(), caches


@pytest.mark.parametrize('nq', [1, 5, 64])
def test_binding_matches_ctypes_path(cuda, nq):
    from src import gpu_kernels as K
    past = 1000
    gen, outliers, hk, hv, (a, b) = _cache_pair(nq, past)
    start = 0
    for f in range((past + 63) // 64):
        n = min(64, past - start)
        bits = (4, 8, 16)[f % 3]
        k, v = hk[:, :, start:start + n], hv[:, :, start:start + n]
        a.select(bits, f)
        a.append(k, v, 0)  # binding
        b.select(bits, f)
        past_b, n_b, row = b._claim(0, n)  # ctypes path, same bookkeeping
        K.pack_rows(k, v, *b._pools(), 0, row, n_b, b.caps[4], b.caps[8], b.caps[16], b.heads, b.dim,
                    b.pending_bits, b.layers, b.status)
        b.seen[0] = past_b + n_b
        start += n
    for name in ('p4', 'm4', 'p8', 'm8', 'p16'):
        rows = a.host_counts[(4, 4, 8, 8, 16)[('p4', 'm4', 'p8', 'm8', 'p16').index(name)]]  # rows in use
        assert torch.equal(a.pool_rows(name, 0, 1, 0, rows), b.pool_rows(name, 0, 1, 0, rows)), name
    q = torch.randn(1, 15, nq, 64, generator=gen).bfloat16().cuda()
    kn, vn = (x.cuda() for x in outlier_kv(gen, 5, nq, outliers))
    out_a = a.attend(q, kn, vn, 0, past)
    out_b = torch.empty_like(out_a)
    K.packed_attention(q, kn, vn, *b._pools(), b.rows, b.codes, out_b, 0, past, nq, b.caps[4], b.caps[8],
                       b.caps[16], 5, 3, 64, 16, 64, b.layers, b.status)
    assert torch.equal(out_a, out_b)
    # append + attend in one launch, against the ctypes binding of the same entry point
    a.select(8, 99)
    b.select(8, 99)
    fused_a = a.append_attend(q, kn, vn, 0)
    past_b, n_b, row = b._claim(0, nq, fill_map=False)
    fused_b = torch.empty_like(fused_a)
    K.append_attention(q, kn, vn, *b._pools(), b.rows, b.codes, fused_b, 0, past_b, n_b, row, 8, True, b.capacity,
                       b.caps[4], b.caps[8], b.caps[16], 5, 3, 64, 16, 64, b.layers, b.status)
    b.seen[0] = past_b + n_b
    a.check()
    b.check()
    assert torch.equal(fused_a, fused_b)
    assert torch.equal(a.pool_rows('p8', 0, 0, row, nq), b.pool_rows('p8', 0, 0, row, nq))
    assert torch.equal(a.rows[:past + nq], b.rows[:past + nq]) and torch.equal(a.codes[:past + nq], b.codes[:past + nq])


def test_binding_errors_keep_the_exception_type(cuda):
    from src.gpu_cache import GPUCache
    c = GPUCache(None, layers=1, heads=5)
    q = torch.randn(1, 15, 4, 64, device='cuda')  # float32, not bfloat16
    k = torch.randn(1, 5, 4, 64, device='cuda').bfloat16()
    with pytest.raises(ValueError, match='bfloat16'):
        c.attend(q, k, k, 0, 0)
    with pytest.raises(ValueError, match='requires CUDA'):
        c.attend(q.cpu().bfloat16(), k, k, 0, 0)
    with pytest.raises(ValueError, match='multiple of KV heads'):
        c.attend(torch.randn(1, 7, 4, 64, device='cuda').bfloat16(), k, k, 0, 0)
