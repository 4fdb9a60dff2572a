"""One synthetic video-QA request through the packed-KV engine.

Keeps the reference CLI's switches (src/inference.py:9-14): --mode
{native,fused16,8,4,dynamic,original,random}, --sample, --frames (1..96),
--device. The reference reads a video and a checkpoint; this build has neither,
so a request is a seeded stand-in (random-init SmolLM2-360M-shape decoder, frame
embeddings, question and four candidates, see streaming.synthetic_request). All
modes need the GPU runtime; there is no CPU path.

    python -m src.inference --mode dynamic --frames 16
"""
import argparse
import json
import time

import torch

from .decoder import SMOLLM2_360M
from .gpu_cache import GPUCache
from .streaming import MODES, StreamingModel, bits_for, synthetic_request


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument('--sample', type=int, default=0)
    p.add_argument('--mode', choices=MODES, default='dynamic')
    p.add_argument('--device', choices=['auto', 'cpu', 'cuda'], default='auto')
    p.add_argument('--frames', type=int)
    args = p.parse_args(argv)
    if args.frames is not None and not 1 <= args.frames <= 96:
        p.error('--frames must be between 1 and 96')
    if args.sample < 0:
        p.error('--sample must be non-negative')
    return args


def timed_request(model, sample, frames, mode):
    """Decoder (frame appends) and QA timings of one request, with the cache's
    accounting (benchmarks/gpu_evaluate.py:69-111, without video decode / vision)."""
    embeds, question, cands = synthetic_request(model.cfg, sample, frames=frames)
    bits = bits_for(mode, frames, seed=sample)
    torch.cuda.synchronize()
    t = time.perf_counter()
    cache = model.ingest(embeds, bits, mode)
    torch.cuda.synchronize()
    decoder_seconds = time.perf_counter() - t
    t = time.perf_counter()
    answer = model.answer(question, cands, cache)
    torch.cuda.synchronize()
    qa_seconds = time.perf_counter() - t
    accounting = cache.accounting() if isinstance(cache, GPUCache) else dict(
        gpu_cache_used_bytes=sum(k.numel() * 2 * 2 for k in cache.k), used_tokens=cache.get_seq_length())
    return dict(sample=sample, mode=mode, frames=frames, bits=bits, decoder_seconds=decoder_seconds,
                qa_seconds=qa_seconds, frames_per_second=frames / (decoder_seconds + qa_seconds),
                answer=answer, cache=accounting)


def main(argv=None):
    args = parse(argv)
    if args.device == 'cpu' or not torch.cuda.is_available():
        raise RuntimeError('This mode requires the GPU runtime')
    model = StreamingModel(SMOLLM2_360M, device='cuda')
    print(json.dumps(timed_request(model, args.sample, args.frames or 16, args.mode), indent=2))


if __name__ == '__main__':
    main()
