"""Launch ordering of programmatic dependents. Every kernel of the library releases
its dependents only after its own griddepcontrol.wait, so when a kernel starts,
every kernel two or more launches back has completed. An attention call whose
preceding launch did not write its layer streams its history before its own
wait; it must still see rows that a pack two launches back wrote.

Pattern (an offline plan, as the reference's per-layer appends make it): pack
frame f of layer 0, pack frame f of layer 1, then attention over layer 0, whose
newest rows were written two launches before it, with no synchronisation in
between. Every output must equal the same call repeated after a device
synchronisation (the kernels are deterministic), over many fresh histories, for
the tensor-core kernel (64 queries) and the split-K kernel (1 query)."""
import pytest
import torch

from dkv_testlib import assert_attention_close, oracle_attention, oracle_frames, outlier_kv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('nq', [64, 1])
def test_attention_sees_rows_packed_two_launches_back(cuda, nq):
    from src.gpu_cache import GPUCache
    gen = torch.Generator().manual_seed(nq)
    outliers = torch.randperm(64, generator=gen)[:4]
    plan = [(8, 64), (4, 64), (16, 64), (4, 64)]
    past = sum(n for _, n in plan)
    for rep in range(24):
        cache = GPUCache(plan, layers=2, heads=5)
        hk, hv = outlier_kv(gen, 5, past, outliers)
        hk, hv = hk.cuda(), hv.cuda()
        q = torch.randn(1, 15, nq, 64, generator=gen).bfloat16().cuda()
        kn, vn = outlier_kv(gen, 5, nq, outliers)
        kn, vn = kn.cuda(), vn.cuda()
        start = 0
        for f, (bits, n) in enumerate(plan):
            cache.select(bits, f)
            for layer in (0, 1):
                cache.append(hk[:, :, start:start + n], hv[:, :, start:start + n], layer)
            start += n
        out = cache.attend(q, kn, vn, 0, past)  # right after the pack of layer 1
        torch.cuda.synchronize()
        again = cache.attend(q, kn, vn, 0, past)
        cache.check()
        assert torch.equal(out, again), rep
    expected = oracle_attention(oracle_frames(hk.cpu(), hv.cpu(), plan), q.cpu(), kn.cpu(), vn.cpu())
    assert_attention_close(out, expected, atol=0.01, rtol=0.01)
