"""Request batching: several independent caches stepped by one launch per layer
(dkv_pack_rows_many, dkv_packed_attention_many). Each request's pools and token
maps must come out bit-identical to its own GPUCache.append; each request's
attention must match the oracle over its own history (pasts may differ); the
batched model path must score like the oracle decoder's per-request protocol."""
import pytest
import torch

from dkv_testlib import assert_attention_close, frame_mix, oracle_attention, oracle_frames, outlier_kv
from oracle.decoder import OracleDecoder, decoder_params
from src import gpu_kernels as K
from src.decoder import DecoderConfig
from src.gpu_cache import GPUCache, append_many, attend_many
from src.streaming import StreamingModel, bits_for, synthetic_request

pytestmark = pytest.mark.gpu


def _history(seed, past, heads=5, layers=2):
    """A cache holding `past` seeded tokens in 64-token frames of mixed precision,
    on every layer, with its oracle frames of layer 0."""
    gen = torch.Generator().manual_seed(seed)
    outliers = torch.randperm(64, generator=gen)[:4]
    frames = max((past + 63) // 64, 0)
    plan = [(b, 64) for b in frame_mix(seed, frames)]
    if plan:
        plan[-1] = (plan[-1][0], past - 64 * (frames - 1))
    hist_k, hist_v = outlier_kv(gen, heads, past, outliers)
    c = GPUCache(None, layers=layers, heads=heads, device='cuda', max_tokens=past + 256)
    start = 0
    for f, (bits, m) in enumerate(plan):
        c.select(bits, f)
        for layer in range(layers):
            c.append(hist_k[:, :, start:start + m].cuda(), hist_v[:, :, start:start + m].cuda(), layer)
        start += m
    return c, oracle_frames(hist_k, hist_v, plan), gen, outliers


@pytest.mark.parametrize('pasts,bits', [((0, 100, 1000, 3000), (4, 8, 16, 4)), ((640, 640, 640), (16, 4, 8))])
def test_pack_many_matches_single_appends(cuda, pasts, bits):
    n, heads = 64, 5
    single = [_history(7 + i, p)[0] for i, p in enumerate(pasts)]
    batched = [_history(7 + i, p)[0] for i, p in enumerate(pasts)]
    gen = torch.Generator().manual_seed(99)
    k = torch.randn(len(pasts), heads, n, 64, generator=gen).bfloat16().cuda()
    v = torch.randn(len(pasts), heads, n, 64, generator=gen).bfloat16().cuda()
    for c, b in zip(single + batched, bits + bits):
        c.select(b, 1000)
    for layer in range(2):
        got = append_many(batched, k, v, layer)
        assert got == list(pasts)
        for r, c in enumerate(single):
            assert c.append(k[r:r + 1], v[r:r + 1], layer) == pasts[r]
    for s, b in zip(single, batched):
        s.check(), b.check()
        assert s.plan == b.plan and s.host_counts == b.host_counts and s.seen == b.seen
        total = s.seen[0]
        assert torch.equal(s.rows[:total], b.rows[:total]) and torch.equal(s.codes[:total], b.codes[:total])
        seg = s.plan[-1]
        rows = slice(seg[3], seg[3] + n)
        pool = {4: ('p4', 'm4'), 8: ('p8', 'm8'), 16: ('p16',)}[seg[2]]
        for name in pool:
            assert torch.equal(getattr(s, name)[:, :, :, rows], getattr(b, name)[:, :, :, rows]), name
        for layer in range(2):
            for x, y in zip(s.materialize(layer), b.materialize(layer)):
                assert torch.equal(x, y)


@pytest.mark.parametrize('pasts,n,group', [((0, 100, 1000, 3000), 64, 3), ((2048, 2048), 64, 3),
                                           ((513, 77, 4000), 5, 3), ((300,) * 9, 64, 4)])
def test_attend_many_matches_oracle_per_request(cuda, pasts, n, group):
    heads = 5
    hist = [_history(31 + i, p, heads=heads, layers=1) for i, p in enumerate(pasts)]
    caches = [h[0] for h in hist]
    gen = torch.Generator().manual_seed(sum(pasts) + n)
    b = len(pasts)
    q = torch.randn(b, heads * group, n, 64, generator=gen).bfloat16()
    kn = torch.cat([outlier_kv(gen, heads, n, hist[r][3])[0] for r in range(b)])
    vn = torch.randn(b, heads, n, 64, generator=gen).bfloat16()
    out = attend_many(caches, q.cuda(), kn.cuda(), vn.cuda(), 0, list(pasts))
    for c in caches:
        c.check()
    assert out.shape == (b, n, heads * group, 64)
    for r in range(b):
        expected = oracle_attention(hist[r][1], q[r:r + 1], kn[r:r + 1], vn[r:r + 1])
        assert_attention_close(out[r:r + 1], expected, atol=0.01, rtol=0.01)
        alone = caches[r].attend(q[r:r + 1].cuda(), kn[r:r + 1].cuda(), vn[r:r + 1].cuda(), 0, pasts[r])
        assert_attention_close(out[r:r + 1], alone, atol=0.01, rtol=0.01)
    again = attend_many(caches, q.cuda(), kn.cuda(), vn.cuda(), 0, list(pasts))
    assert torch.equal(out, again)  # deterministic


def test_more_requests_than_one_launch_takes(cuda):
    b, n, heads = K.MAX_REQUESTS + 3, 64, 5
    hist = [_history(200 + i, 64 + 7 * i, heads=heads, layers=1) for i in range(b)]
    caches = [h[0] for h in hist]
    pasts = [c.seen[0] for c in caches]
    gen = torch.Generator().manual_seed(5)
    q = torch.randn(b, heads * 3, n, 64, generator=gen).bfloat16()
    kn = torch.randn(b, heads, n, 64, generator=gen).bfloat16()
    vn = torch.randn(b, heads, n, 64, generator=gen).bfloat16()
    for c in caches:
        c.select(8, 500)
    assert append_many(caches, kn.cuda(), vn.cuda(), 0) == pasts
    out = attend_many(caches, q.cuda(), kn.cuda(), vn.cuda(), 0, pasts)
    for r in (0, K.MAX_REQUESTS - 1, K.MAX_REQUESTS, b - 1):
        caches[r].check()
        expected = oracle_attention(hist[r][1], q[r:r + 1], kn[r:r + 1], vn[r:r + 1])
        assert_attention_close(out[r:r + 1], expected, atol=0.01, rtol=0.01)
        assert caches[r].seen[0] == pasts[r] + n
        assert int(caches[r].codes[pasts[r]]) == 8


def test_append_many_rejects_shared_pools(cuda):
    c = _history(3, 128, layers=1)[0]
    k = torch.zeros(2, 5, 64, 64, dtype=torch.bfloat16, device='cuda')
    with pytest.raises(ValueError, match='own pools'):
        append_many([c, c.fork()], k, k, 0)


TINY = DecoderConfig(layers=2, hidden=384, q_heads=6, kv_heads=2, head_dim=64, intermediate=1024, vocab=1000,
                     init_std=0.05)


@pytest.mark.parametrize('mode', ['fused16', '4', 'dynamic'])
def test_batched_requests_match_oracle_decoder(cuda, mode):
    model = StreamingModel(TINY, device='cuda', seed=21)
    reqs = [synthetic_request(TINY, seed=s, frames=5, frame_tokens=64, question_tokens=12, candidates=3,
                              candidate_tokens=6, device='cuda') for s in (1, 2, 3)]
    bits = [bits_for(mode, 5, seed=s) for s in (1, 2, 3)]
    caches = model.ingest_many([r[0] for r in reqs], bits, mode, qa_reserve=64)
    got = model.answer_many([r[1] for r in reqs], [r[2] for r in reqs], caches)
    oracle = OracleDecoder(TINY, decoder_params(model.model))
    for r, (embeds, question, cands) in enumerate(reqs):
        caches[r].check()
        means, sums = oracle.request(model.prefix_ids, embeds, bits[r], question, cands)
        assert max(abs(a - b) for a, b in zip(got[r]['scores'], means)) < 2e-2, (got[r]['scores'], means)
        assert max(abs(a - b) for a, b in zip(got[r]['summed'], sums)) < 2e-2 * cands[0].shape[1]
        alone = model.answer(question, cands, model.ingest(embeds, bits[r], mode, qa_reserve=64))
        assert max(abs(a - b) for a, b in zip(got[r]['scores'], alone['scores'])) < 2e-2
        assert caches[r].seen[0] == model.prefix_ids.shape[1] + 5 * 64
        assert [s[2] for s in caches[r].plan[1:]] == bits[r]
