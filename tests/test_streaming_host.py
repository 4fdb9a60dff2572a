"""CPU tests of the streaming engine's host logic: the --mode switch, the CLI
checks, and the decoder architecture (native bf16 cache on the CPU) against the
fp32 oracle decoder with every segment stored at 16 bits."""
import random

import pytest
import torch

from oracle.decoder import OracleDecoder, decoder_params
from src.decoder import Decoder, DecoderConfig, NativeCache
from src.inference import parse
from src.streaming import RANDOM_PROBABILITIES, bits_for, synthetic_request

TINY = DecoderConfig(layers=2, hidden=384, q_heads=6, kv_heads=2, head_dim=64, intermediate=1024, vocab=1000,
                     init_std=0.05)


def test_bits_for_matches_reference_mode_semantics():
    assert bits_for('native', 5) == [16] * 5 and bits_for('fused16', 3) == [16] * 3
    assert bits_for('4', 4) == [4] * 4 and bits_for('8', 2) == [8] * 2
    # random mode: random.Random(seed).choices with the reference's weights
    assert bits_for('random', 50, seed=7) == random.Random(7).choices([4, 8, 16], weights=RANDOM_PROBABILITIES, k=50)
    d = bits_for('dynamic', 2000, seed=3)
    assert bits_for('dynamic', 2000, seed=3) == d and set(d) == {4, 8, 16}
    assert 0.45 < d.count(4) / 2000 < 0.55 and 0.25 < d.count(8) / 2000 < 0.35
    with pytest.raises(ValueError):
        bits_for('fp8', 3)


def test_cli_checks_like_the_reference():
    assert parse(['--mode', '4', '--frames', '8']).mode == '4'
    with pytest.raises(SystemExit):
        parse(['--frames', '97'])
    with pytest.raises(SystemExit):
        parse(['--mode', 'bogus'])


def test_native_decoder_matches_oracle_decoder_on_cpu():
    torch.manual_seed(0)
    model = Decoder(TINY, device='cpu', seed=3)
    oracle = OracleDecoder(TINY, decoder_params(model))
    embeds, question, cands = synthetic_request(TINY, seed=5, frames=2, frame_tokens=16, question_tokens=6,
                                                candidates=3, candidate_tokens=4, device='cpu')
    prefix = torch.randint(0, TINY.vocab, (1, 5))
    cache = NativeCache(TINY.layers)
    with torch.inference_mode():
        model(cache, ids=prefix)
        for e in embeds:
            model(cache, embeds=e)
        got = []
        for c in cands:
            fork = cache.fork()
            logits = model(fork, ids=torch.cat((question, c), 1), logits=c.shape[1] + 1)
            got.append(float(logits[0, :-1].log_softmax(-1).gather(1, c[0][:, None]).mean()))
    means, _ = oracle.request(prefix, embeds, [16] * len(embeds), question, cands)
    assert max(abs(a - b) for a, b in zip(got, means)) < 2e-2
    assert cache.get_seq_length() == 5 + 2 * 16
