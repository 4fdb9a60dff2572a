"""Batched query chunks over one packed history (dkv_packed_attention_batched) and
the batched candidate scoring built on it: every chunk matches the oracle on its
own (history + its own new K/V, bottom-right causal), and batched scoring matches
the oracle decoder's per-candidate protocol."""
import pytest
import torch

from dkv_testlib import assert_attention_close, frame_mix, oracle_attention, oracle_frames, outlier_kv
from oracle.decoder import OracleDecoder, decoder_params
from src.decoder import DecoderConfig
from src.gpu_cache import GPUCache
from src.streaming import StreamingModel, bits_for, synthetic_request

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('past,chunks,n,group', [(2048, 4, 24, 3), (640, 3, 64, 3), (5000, 2, 5, 3), (300, 4, 96, 4)])
def test_batched_chunks_match_oracle_per_chunk(cuda, past, chunks, n, group):
    gen = torch.Generator().manual_seed(past + chunks)
    outliers = torch.randperm(64, generator=gen)[:4]
    frames = (past + 63) // 64
    plan = [(b, 64) for b in frame_mix(past, frames)]
    plan[-1] = (plan[-1][0], past - 64 * (frames - 1))
    hist_k, hist_v = outlier_kv(gen, 5, past, outliers)
    c = GPUCache(None, layers=1, heads=5, device='cuda', max_tokens=past + 128)
    start = 0
    for f, (bits, m) in enumerate(plan):
        c.select(bits, f)
        c.append(hist_k[:, :, start:start + m].cuda(), hist_v[:, :, start:start + m].cuda(), 0)
        start += m
    q = torch.randn(chunks, 5 * group, n, 64, generator=gen).bfloat16()
    kn = torch.cat([outlier_kv(gen, 5, n, outliers)[0] for _ in range(chunks)])
    vn = torch.randn(chunks, 5, n, 64, generator=gen).bfloat16()
    out = c.attend_batched(q.cuda(), kn.cuda(), vn.cuda(), 0, past)
    c.check()
    assert out.shape == (chunks, n, 5 * group, 64)
    fr = oracle_frames(hist_k, hist_v, plan)
    for b in range(chunks):
        expected = oracle_attention(fr, q[b:b + 1], kn[b:b + 1], vn[b:b + 1])
        assert_attention_close(out[b:b + 1], expected, atol=0.01, rtol=0.01)
    again = c.attend_batched(q.cuda(), kn.cuda(), vn.cuda(), 0, past)
    assert torch.equal(out, again)  # deterministic
    c.check()


TINY = DecoderConfig(layers=2, hidden=384, q_heads=6, kv_heads=2, head_dim=64, intermediate=1024, vocab=1000,
                     init_std=0.05)


@pytest.mark.parametrize('mode', ['native', 'fused16', '8', '4', 'dynamic'])
def test_batched_candidate_scoring_matches_oracle(cuda, mode):
    model = StreamingModel(TINY, device='cuda', seed=21)
    embeds, question, cands = synthetic_request(TINY, seed=4, frames=6, frame_tokens=64, question_tokens=12,
                                                candidates=4, candidate_tokens=6, device='cuda')
    bits = bits_for(mode, len(embeds), seed=4)
    cache = model.ingest(embeds, bits, mode, qa_reserve=64)
    got = model.answer(question, cands, cache, batched=True)
    per_candidate = model.answer(question, cands, cache)
    means, sums = OracleDecoder(TINY, decoder_params(model.model)).request(model.prefix_ids, embeds, bits, question,
                                                                            cands)
    assert max(abs(a - b) for a, b in zip(got['scores'], means)) < 2e-2, (got['scores'], means)
    assert max(abs(a - b) for a, b in zip(got['summed'], sums)) < 2e-2 * cands[0].shape[1]
    assert max(abs(a - b) for a, b in zip(got['scores'], per_candidate['scores'])) < 2e-2
    if mode != 'native':
        cache.check()
