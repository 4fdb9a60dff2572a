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


def _device_tables(caches, pasts, rows=None):
    """Pack targets / histories of the caches in device memory (16-byte aligned)."""
    import ctypes
    from src.gpu_cache import _history, _pack_target
    b = len(caches)
    hist = (K.History * b)(*[_history(c, p) for c, p in zip(caches, pasts)])
    dev_h = torch.frombuffer(bytearray(bytes(hist)), dtype=torch.uint8).cuda()
    dev_t = None
    if rows is not None:
        tg = (K.PackTarget * b)(*[_pack_target(c, p, r, c.online) for c, p, r in zip(caches, pasts, rows)])
        dev_t = torch.frombuffer(bytearray(bytes(tg)), dtype=torch.uint8).cuda()
    assert ctypes.sizeof(K.History) * b == dev_h.numel()
    return dev_h, dev_t


@pytest.mark.parametrize('pasts,n', [((0, 100, 1000, 3000), 64), ((513, 77, 4000), 5)])
def test_device_descriptors_match_host_descriptors(cuda, pasts, n):
    """The device-table attention is bit-identical to the by-value one for the same
    plan bound, and the device-table pack to the host-table pack."""
    heads, group = 5, 3
    hist = [_history(71 + i, p, heads=heads, layers=1) for i, p in enumerate(pasts)]
    caches = [h[0] for h in hist]
    b = len(pasts)
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(b, heads * group, n, 64, generator=gen).bfloat16().cuda()
    kn = torch.randn(b, heads, n, 64, generator=gen).bfloat16().cuda()
    vn = torch.randn(b, heads, n, 64, generator=gen).bfloat16().cuda()
    ref = attend_many(caches, q, kn, vn, 0, list(pasts))
    dev_h, _ = _device_tables(caches, pasts)
    out = torch.empty_like(ref)
    K.packed_attention_many_device(q, kn, vn, dev_h.data_ptr(), b, max(pasts), out, 0, n, heads, group, 64, 1)
    torch.cuda.synchronize()
    for c in caches:
        c.check()
    assert torch.equal(out, ref)
    # a larger plan bound changes only the split count: still the oracle's result
    K.packed_attention_many_device(q, kn, vn, dev_h.data_ptr(), b, 8000, out, 0, n, heads, group, 64, 1)
    for r in range(b):
        expected = oracle_attention(hist[r][1], q[r:r + 1].cpu(), kn[r:r + 1].cpu(), vn[r:r + 1].cpu())
        assert_attention_close(out[r:r + 1], expected, atol=0.01, rtol=0.01)
    # pack through device tables: same pools as the host-table launch on twin caches
    twins = [_history(71 + i, p, heads=heads, layers=1)[0] for i, p in enumerate(pasts)]
    for c, bt in zip(caches + twins, (4, 8, 16, 4)[:b] * 2):
        c.select(bt, 77)
    append_many(twins, kn, vn, 0)
    claims = [c._claim_frame(n) for c in caches]
    _, dev_t = _device_tables(caches, [p for p, _ in claims], [r for _, r in claims])
    K.pack_rows_many_device(kn, vn, dev_t.data_ptr(), b, 0, n, heads, 64, 1)
    for c, t in zip(caches, twins):
        c.check()
        total = c.seen[0]
        assert torch.equal(c.rows[:total], t.rows[:total]) and torch.equal(c.codes[:total], t.codes[:total])
        for x, y in zip(c.materialize(0), t.materialize(0)):
            assert torch.equal(x, y)


def test_device_descriptor_errors_are_reported_not_used(cuda):
    """A history longer than its token map and a pack row range beyond the pool are
    reported to the request's status word; the kernels skip them."""
    c, _, _, _ = _history(5, 256, layers=1)
    h = (K.History * 1)(K.History(c.p4.data_ptr(), c.m4.data_ptr(), c.p8.data_ptr(), c.m8.data_ptr(),
                                   c.p16.data_ptr(), c.rows.data_ptr(), c.codes.data_ptr(), c.caps[4], c.caps[8],
                                   c.caps[16], c.capacity + 1, c.capacity, c.status.data_ptr()))
    dev_h = torch.frombuffer(bytearray(bytes(h)), dtype=torch.uint8).cuda()
    q = torch.zeros(1, 15, 64, 64, dtype=torch.bfloat16, device='cuda')
    kv = torch.zeros(1, 5, 64, 64, dtype=torch.bfloat16, device='cuda')
    out = torch.empty(1, 64, 15, 64, dtype=torch.bfloat16, device='cuda')
    K.packed_attention_many_device(q, kv, kv, dev_h.data_ptr(), 1, 256, out, 0, 64, 5, 3, 64, 1)
    with pytest.raises(ValueError, match='invalid argument'):
        c.check()
    h[0].past, h[0].p8 = 256, None  # a null pool in a device descriptor: reported, the history not read
    dev_h = torch.frombuffer(bytearray(bytes(h)), dtype=torch.uint8).cuda()
    K.packed_attention_many_device(q, kv, kv, dev_h.data_ptr(), 1, 256, out, 0, 64, 5, 3, 64, 1)
    with pytest.raises(ValueError, match='invalid argument'):
        c.check()
    from src.gpu_cache import _pack_target
    t = (K.PackTarget * 1)(_pack_target(c, 256, c.caps[16] - 10, False))
    t[0].bits = 16
    dev_t = torch.frombuffer(bytearray(bytes(t)), dtype=torch.uint8).cuda()
    K.pack_rows_many_device(kv, kv, dev_t.data_ptr(), 1, 0, 64, 5, 64, 1)
    with pytest.raises(ValueError, match='capacity'):
        c.check()


@pytest.mark.parametrize('mode', ['fused16', 'dynamic'])
def test_frame_graph_ingest_matches_eager_batched_ingest(cuda, mode):
    """Frames appended by replaying one captured graph give the same caches and
    scores as the eager batched ingest (the first frames' plan bound differs, so
    within floating-point order; then identical precision plans)."""
    model = StreamingModel(TINY, device='cuda', seed=21)
    reqs = [synthetic_request(TINY, seed=s, frames=6, frame_tokens=64, question_tokens=12, candidates=3,
                              candidate_tokens=6, device='cuda') for s in (1, 2, 3)]
    bits = [bits_for(mode, 6, seed=s) for s in (1, 2, 3)]
    eager = model.ingest_many([r[0] for r in reqs], bits, mode, qa_reserve=64)
    graphed = model.ingest_many([r[0] for r in reqs], bits, mode, qa_reserve=64, graph=True)
    oracle = OracleDecoder(TINY, decoder_params(model.model))
    got = model.answer_many([r[1] for r in reqs], [r[2] for r in reqs], graphed)
    want = model.answer_many([r[1] for r in reqs], [r[2] for r in reqs], eager)
    for r, (embeds, question, cands) in enumerate(reqs):
        graphed[r].check()
        assert graphed[r].plan == eager[r].plan and graphed[r].seen == eager[r].seen
        for x, y in zip(graphed[r].materialize(0), eager[r].materialize(0)):  # layer 0 K/V precede any attention
            assert torch.equal(x, y)
        means, _ = oracle.request(model.prefix_ids, embeds, bits[r], question, cands)
        assert max(abs(a - b) for a, b in zip(got[r]['scores'], means)) < 2e-2, (got[r]['scores'], means)
        assert max(abs(a - b) for a, b in zip(got[r]['scores'], want[r]['scores'])) < 2e-2


def test_frame_graph_replay_matches_its_eager_step(cuda):
    """Replaying the captured step computes exactly what the eager device-descriptor
    step computes for the same frame."""
    from src.decoder import FrameGraph
    model = StreamingModel(TINY, device='cuda', seed=3)
    gen = torch.Generator().manual_seed(8)
    frames = [(torch.randn(2, 64, TINY.hidden, generator=gen) * 0.02).bfloat16().cuda() for _ in range(4)]

    def caches():
        cs = [model.create_cache([64] * 4, 'dynamic', qa_reserve=64) for _ in range(2)]
        model.model.forward_many(cs, ids=model.prefix_ids.expand(2, -1))
        return cs

    a, b = caches(), caches()
    ga = FrameGraph(model.model, a, 64, logits=3, max_past=512)
    gb = FrameGraph(model.model, b, 64, logits=3, max_past=512)
    pools = ('p4', 'm4', 'p8', 'm8', 'p16')
    ptrs, caps = [[getattr(c, n).data_ptr() for n in pools] for c in a], [dict(c.caps) for c in a]
    with torch.inference_mode():
        for i, x in enumerate(frames):
            for c, bt in zip(a + b, (4, 16, 4, 16) if i % 2 else (8, 4, 8, 4)):
                c.select(bt, i)
            la = ga.step(embeds=x).clone()  # eager at i = 0, replayed afterwards
            if i == 1:
                graph = ga.graph
            gb.batch.prepare()             # b: the eager device-descriptor step every time
            gb.x.copy_(x)
            lb = model.model.forward_device(gb.batch, gb.x, 3)
            assert torch.equal(la, lb), i
    # the pools grew during replayed steps: the same graph kept serving them, at the
    # same addresses (growth maps pages behind the old rows)
    assert ga.graph is graph and all(c.caps != c0 for c, c0 in zip(a, caps))
    assert [[getattr(c, n).data_ptr() for n in pools] for c in a] == ptrs
    for x, y in zip(a, b):
        x.check()
        for layer in range(TINY.layers):
            for p, q in zip(x.materialize(layer), y.materialize(layer)):
                assert torch.equal(p, q)


def test_frame_graph_is_reused_for_the_next_batch(cuda):
    """The captured frame step is rebound to the next batch's caches: the second
    batch ingested through the same graph equals its eager ingest."""
    model = StreamingModel(TINY, device='cuda', seed=5)
    sets = [[synthetic_request(TINY, seed=s, frames=4, frame_tokens=64, question_tokens=12, candidates=2,
                               candidate_tokens=6, device='cuda') for s in seeds] for seeds in ((11, 12), (13, 14))]
    bits = [[bits_for('dynamic', 4, seed=s) for s in seeds] for seeds in ((11, 12), (13, 14))]
    model.ingest_many([r[0] for r in sets[0]], bits[0], 'dynamic', qa_reserve=64, graph=True)
    graph = model._frame_graphs[(2, 64, 0, True)].graph
    graphed = model.ingest_many([r[0] for r in sets[1]], bits[1], 'dynamic', qa_reserve=64, graph=True)
    assert model._frame_graphs[(2, 64, 0, True)].graph is graph  # captured once
    assert model._frame_graphs[(2, 64, 0, True)].batch.caches == []  # finished caches are not kept alive
    with pytest.raises(ValueError, match='no caches bound'):
        model._frame_graphs[(2, 64, 0, True)].step(embeds=torch.zeros(2, 64, TINY.hidden, dtype=torch.bfloat16,
                                                                device='cuda'))
    eager = model.ingest_many([r[0] for r in sets[1]], bits[1], 'dynamic', qa_reserve=64)
    got = model.answer_many([r[1] for r in sets[1]], [r[2] for r in sets[1]], graphed)
    want = model.answer_many([r[1] for r in sets[1]], [r[2] for r in sets[1]], eager)
    for g, e, a, b in zip(graphed, eager, got, want):
        g.check()
        assert g.plan == e.plan and g.seen == e.seen
        for x, y in zip(g.materialize(0), e.materialize(0)):
            assert torch.equal(x, y)
        assert max(abs(p - q) for p, q in zip(a['scores'], b['scores'])) < 2e-2


@pytest.mark.parametrize('mode', ['fused16', 'dynamic'])
def test_graph_replayed_scoring_matches_eager_scoring(cuda, mode):
    """The reference protocol with each candidate's forward replayed from a captured
    graph scores like the eager protocol and the oracle decoder, for one request and
    for a batch of requests; a second run through the cached graphs repeats it."""
    model = StreamingModel(TINY, device='cuda', seed=9)
    reqs = [synthetic_request(TINY, seed=s, frames=4, frame_tokens=64, question_tokens=12, candidates=3,
                              candidate_tokens=6, device='cuda') for s in (21, 22)]
    bits = [bits_for(mode, 4, seed=s) for s in (21, 22)]
    caches = model.ingest_many([r[0] for r in reqs], bits, mode, qa_reserve=64)
    oracle = OracleDecoder(TINY, decoder_params(model.model))
    for r, (embeds, question, cands) in enumerate(reqs):
        eager = model.answer(question, cands, caches[r])
        graphed = model.answer(question, cands, caches[r], graph=True)
        again = model.answer(question, cands, caches[r], graph=True)
        means, _ = oracle.request(model.prefix_ids, embeds, bits[r], question, cands)
        assert max(abs(a - b) for a, b in zip(graphed['scores'], eager['scores'])) < 2e-2
        assert max(abs(a - b) for a, b in zip(graphed['scores'], means)) < 2e-2
        assert graphed['scores'] == again['scores']
        caches[r].check()
    many = model.answer_many([r[1] for r in reqs], [r[2] for r in reqs], caches, graph=True)
    eager_many = model.answer_many([r[1] for r in reqs], [r[2] for r in reqs], caches)
    for a, b in zip(many, eager_many):
        assert max(abs(x - y) for x, y in zip(a['scores'], b['scores'])) < 2e-2
    assert all(c.seen == caches[0].seen for c in caches)  # scoring never moves the video caches


@pytest.mark.parametrize('mode', ['fused16', 'dynamic'])
def test_graph_replayed_batched_scoring_matches_eager(cuda, mode):
    """Batched scoring (question once, candidates side by side over one fork) with
    both steps replayed from captured graphs, the candidates' without appending."""
    model = StreamingModel(TINY, device='cuda', seed=13)
    embeds, question, cands = synthetic_request(TINY, seed=31, frames=4, frame_tokens=64, question_tokens=12,
                                                candidates=4, candidate_tokens=6, device='cuda')
    bits = bits_for(mode, 4, seed=31)
    cache = model.ingest(embeds, bits, mode, qa_reserve=64)
    eager = model.answer(question, cands, cache, batched=True)
    graphed = model.answer(question, cands, cache, batched=True, graph=True)
    again = model.answer(question, cands, cache, batched=True, graph=True)
    means, _ = OracleDecoder(TINY, decoder_params(model.model)).request(model.prefix_ids, embeds, bits, question,
                                                                        cands)
    assert max(abs(a - b) for a, b in zip(graphed['scores'], eager['scores'])) < 2e-2
    assert max(abs(a - b) for a, b in zip(graphed['scores'], means)) < 2e-2
    assert graphed['scores'] == again['scores']
    cache.check()
    assert cache.seen == [model.prefix_ids.shape[1] + 4 * 64] * TINY.layers
