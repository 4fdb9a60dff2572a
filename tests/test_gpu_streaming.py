"""GPU parity of the model-level path: frame appends at each --mode's precisions
and candidate scoring (src/streaming.py:209-225) against the fp32 oracle decoder
with the reference's CPU cache semantics. Tolerance (stated): per-candidate mean
log-likelihood within 2e-2, and the same argmax whenever the oracle's top-two
margin exceeds 4e-2."""
import pytest
import torch

from oracle.decoder import OracleDecoder, decoder_params
from src.decoder import DecoderConfig
from src.streaming import StreamingModel, bits_for, synthetic_request

pytestmark = pytest.mark.gpu
TINY = DecoderConfig(layers=2, hidden=384, q_heads=6, kv_heads=2, head_dim=64, intermediate=1024, vocab=1000,
                     init_std=0.05)


@pytest.mark.parametrize('mode', ['native', 'fused16', '8', '4', 'dynamic'])
def test_candidate_scores_match_oracle(cuda, mode):
    model = StreamingModel(TINY, device='cuda', seed=21)
    embeds, question, cands = synthetic_request(TINY, seed=4, frames=6, frame_tokens=64, question_tokens=12,
                                                candidates=4, candidate_tokens=6, device='cuda')
    bits = bits_for(mode, len(embeds), seed=4)
    cache = model.ingest(embeds, bits, mode, qa_reserve=64)
    got = model.answer(question, cands, cache)
    oracle = OracleDecoder(TINY, decoder_params(model.model))
    means, sums = oracle.request(model.prefix_ids, embeds, bits, question, cands)
    assert max(abs(a - b) for a, b in zip(got['scores'], means)) < 2e-2, (got['scores'], means)
    assert max(abs(a - b) for a, b in zip(got['summed'], sums)) < 2e-2 * cands[0].shape[1]
    top = sorted(means, reverse=True)
    if top[0] - top[1] > 4e-2:
        assert got['prediction'] == max(range(len(means)), key=means.__getitem__)
    if mode != 'native':
        cache.check()
        again = model.answer(question, cands, cache)  # forks never move the base cache
        assert again['scores'] == got['scores']


def test_frame_append_accounting_matches_plan(cuda):
    model = StreamingModel(TINY, device='cuda', seed=2)
    embeds, _, _ = synthetic_request(TINY, seed=1, frames=5, device='cuda')
    bits = [4, 8, 16, 4, 8]
    cache = model.ingest(embeds, bits, 'dynamic', qa_reserve=32)
    a = cache.accounting()
    prefix = model.prefix_ids.shape[1]
    assert a['precision_token_counts'] == {4: 128, 8: 128, 16: 64 + prefix}
    assert a['used_tokens'] == prefix + 5 * 64 and cache.caps[16] >= cache.host_counts[16] + 32
    assert cache.plan[1] == (prefix, prefix + 64, 4, 0)
