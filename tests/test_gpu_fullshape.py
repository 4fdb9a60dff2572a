"""Model-level parity at the BASELINE model shape (random-init SmolLM2-360M:
32 layers, hidden 960, 15 query / 5 KV heads of 64, MLP 2560, vocab 49280, bf16)
against the fp32 oracle decoder with the reference's CPU cache semantics.

C4: a 96-frame (6144-token) mixed 4/8/16 packed prefix, a 32-token question and
4 x 24-token candidates, scored with the reference protocol (src/streaming.py:
209-225), its graph-replayed form, and the batched forms (question once, the
candidates side by side), eager and graph-replayed.
C5: one 64-frame request of the request-throughput configuration, ingested in a
batch of two requests with graph-replayed frame steps and scored with the
batched reference protocol.
Tolerance (stated): per-candidate mean log-likelihood within 2e-2 of the
oracle's, and the same argmax whenever the oracle's top-two margin exceeds 4e-2.
The attention calls of both shapes (56 queries after 6144 packed tokens, four
24-query chunks after 6176) are also checked on their own against the attention
oracle.
"""
import pytest
import torch

from dkv_testlib import assert_attention_close, frame_mix, oracle_attention, oracle_frames, outlier_kv
from oracle.decoder import OracleDecoder, decoder_params

pytestmark = pytest.mark.gpu
TOL, MARGIN = 2e-2, 4e-2


def _check(got, means):
    assert max(abs(a - b) for a, b in zip(got['scores'], means)) < TOL, (got['scores'], means)
    top = sorted(means, reverse=True)
    if top[0] - top[1] > MARGIN:
        assert got['prediction'] == max(range(len(means)), key=means.__getitem__)


@pytest.fixture(scope='module')
def smollm(cuda):
    from src.decoder import SMOLLM2_360M
    from src.streaming import StreamingModel
    model = StreamingModel(SMOLLM2_360M, device='cuda', seed=0)
    oracle = OracleDecoder(SMOLLM2_360M, decoder_params(model.model), memo=True)
    return model, oracle


def test_c4_candidate_scoring_full_shape(smollm):
    from src.streaming import bits_for, synthetic_request
    model, oracle = smollm
    embeds, question, cands = synthetic_request(model.cfg, seed=4, frames=96, device='cuda')
    bits = bits_for('dynamic', 96, seed=4)
    cache = model.ingest(embeds, bits, 'dynamic', qa_reserve=64)
    cache.check()
    assert cache.seen[0] == model.prefix_ids.shape[1] + 96 * 64
    means, _ = oracle.request(model.prefix_ids, embeds, bits, question, cands)
    for kw in (dict(), dict(graph=True), dict(batched=True), dict(batched=True, graph=True)):
        got = model.answer(question, cands, cache, **kw)
        cache.check()
        _check(got, means)


def test_c5_request_full_shape(smollm):
    from src.streaming import bits_for, synthetic_request
    model, oracle = smollm
    reqs = [synthetic_request(model.cfg, seed=r, frames=64, device='cuda') for r in (0, 1)]
    bits = [bits_for('dynamic', 64, seed=r) for r in (0, 1)]
    caches = model.ingest_many([r[0] for r in reqs], bits, 'dynamic', qa_reserve=64, graph=True)
    answers = model.answer_many([r[1] for r in reqs], [r[2] for r in reqs], caches, graph=True)
    for c in caches:
        c.check()
    embeds, question, cands = reqs[0]
    means, _ = oracle.request(model.prefix_ids, embeds, bits[0], question, cands)
    _check(answers[0], means)


@pytest.mark.parametrize('past,nq,chunks', [(6144, 56, 1), (6176, 24, 4)])
def test_c4_attention_shapes_vs_oracle(cuda, past, nq, chunks):
    from src.gpu_cache import GPUCache
    gen = torch.Generator().manual_seed(past + nq)
    outliers = torch.randperm(64, generator=gen)[:4]
    plan = [(b, min(64, past - 64 * f)) for f, b in enumerate(frame_mix(past, (past + 63) // 64))]
    cache = GPUCache(None, layers=1, heads=5, max_tokens=past + nq + 64)
    hist_k, hist_v = outlier_kv(gen, 5, past, outliers)
    start = 0
    for f, (b, n) in enumerate(plan):
        cache.select(b, f)
        cache.append(hist_k[:, :, start:start + n].cuda(), hist_v[:, :, start:start + n].cuda(), 0)
        start += n
    q = torch.randn(chunks, 15, nq, 64, generator=gen).bfloat16()
    kv = [outlier_kv(gen, 5, nq, outliers) for _ in range(chunks)]
    kn, vn = torch.cat([k for k, _ in kv]), torch.cat([v for _, v in kv])
    if chunks == 1:
        out = cache.attend(q.cuda(), kn.cuda(), vn.cuda(), 0, past)
    else:
        out = cache.attend_batched(q.cuda(), kn.cuda(), vn.cuda(), 0, past)
    cache.check()
    frames = oracle_frames(hist_k, hist_v, plan)
    for c in range(chunks):
        expected = oracle_attention(frames, q[c:c + 1], kn[c:c + 1], vn[c:c + 1])
        assert_attention_close(out[c:c + 1], expected, atol=0.01, rtol=0.01)
