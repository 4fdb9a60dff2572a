"""Streaming engine over the packed-KV cache: frame appends and candidate scoring.

Mirrors the cache-facing part of the reference engine (src/streaming.py):
create_cache (:155-165) builds a GPUCache (online plan, bf16) or a native cache;
ingest (:168-187) appends a prefix and then one frame at a time with the frame's
precision selected on the cache, and reserves the QA rows; answer with the
"candidate" protocol (:209-225) scores every candidate on a fork of the video
cache by its mean token log-likelihood (the reference's score) — the summed
log-likelihood is returned as well. Video decoding and the vision tower are not
part of this path: a frame arrives as its 64 visual-token embeddings.

bits_for restates the --mode switch of benchmarks/gpu_evaluate.py:23-31. The
reference's "dynamic"/"original" modes run an OpenCV feature policy on real video;
here they draw each frame's precision from a seeded categorical over {4, 8, 16}
(default weights 0.5 / 0.3 / 0.2), as the benchmark configurations specify.
"""
import random

import torch

from .decoder import SMOLLM2_360M, Decoder, FrameGraph, NativeCache
from .gpu_cache import GPUCache

MODES = ['native', 'fused16', '8', '4', 'dynamic', 'original', 'random']
# configs/gpu_selected.json:181-185 of the reference ("random" mode weights)
RANDOM_PROBABILITIES = [0.6834782608695652, 0.2991304347826087, 0.017391304347826087]
DYNAMIC_PROBABILITIES = [0.5, 0.3, 0.2]


def bits_for(mode, frames, seed=0):
    """Per-frame storage precision for --mode (benchmarks/gpu_evaluate.py:23-31)."""
    if mode not in MODES:
        raise ValueError(f'mode must be one of {MODES}')
    if mode in ('native', 'fused16'):
        return [16] * frames
    if mode in ('4', '8'):
        return [int(mode)] * frames
    weights = RANDOM_PROBABILITIES if mode == 'random' else DYNAMIC_PROBABILITIES
    return random.Random(seed).choices([4, 8, 16], weights=weights, k=frames)


class StreamingModel:
    def __init__(self, cfg=SMOLLM2_360M, device='cuda', seed=0, prefix_tokens=11):
        self.cfg = cfg
        self.device = torch.device(device)
        self.model = Decoder(cfg, device=device, seed=seed)
        gen = torch.Generator().manual_seed(seed + 1)
        self.prefix_ids = torch.randint(0, cfg.vocab, (1, prefix_tokens), generator=gen).to(self.device)
        self._frame_graphs = {}  # (requests, tokens, logits, append) -> FrameGraph, captured once and rebound

    def frame_graph(self, caches, n, logits=0, append=True):
        """The FrameGraph for len(caches) requests of n-token steps returning `logits`
        positions, captured on first use and rebound to `caches` afterwards."""
        key = (len(caches), n, logits, append)
        fg = self._frame_graphs.get(key)
        if fg is None:
            fg = self._frame_graphs[key] = FrameGraph(self.model, caches, n, logits=logits, append=append)
        else:
            fg.rebind(caches)
        return fg

    def create_cache(self, frame_lengths, mode, qa_reserve=192, max_tokens=8192):
        """GPUCache with an online plan (or a native cache for mode 'native'),
        checking the context limit like src/streaming.py:159-163."""
        if mode == 'native':
            return NativeCache(self.cfg.layers)
        total = self.prefix_ids.shape[1] + sum(frame_lengths) + qa_reserve
        if total > max_tokens:
            raise ValueError('Context exceeds the checkpoint limit')
        return GPUCache(None, layers=self.cfg.layers, heads=self.cfg.kv_heads, dim=self.cfg.head_dim,
                        device=self.device, max_tokens=max_tokens)

    @torch.inference_mode()
    def ingest(self, frames, bits, mode, qa_reserve=192):
        """Appends the prefix, then each frame ([1, n, hidden] embeddings) at its
        precision; returns the cache (src/streaming.py:168-187)."""
        cache = self.create_cache([f.shape[1] for f in frames], mode, qa_reserve)
        self.model(cache, ids=self.prefix_ids)
        for i, (emb, bit) in enumerate(zip(frames, bits)):
            if isinstance(cache, GPUCache):
                cache.select(bit, i)
            self.model(cache, embeds=emb)
        if isinstance(cache, GPUCache):
            cache.select(16, -1)
            cache.reserve(16, cache.host_counts[16] + qa_reserve)
            if len(set(cache.seen)) != 1:
                raise RuntimeError('Decoder layers disagree about the cache length')
        return cache

    @torch.inference_mode()
    def answer(self, question_ids, candidate_ids, cache, batched=False, graph=False):
        """Candidate protocol (src/streaming.py:209-225): per candidate, a fork of
        the cache sees question + candidate; the score is the mean log-likelihood
        of the candidate tokens. Returns scores (mean), summed log-likelihoods and
        the argmax. batched=True (equal-length candidates; not in the reference)
        appends the question to one fork once and runs every candidate in one
        forward over it: the same likelihoods up to floating-point order.
        graph=True (GPUCache; not in the reference) replays each candidate's
        forward from one captured CUDA graph (FrameGraph) instead of launching it."""
        if batched and len({c.shape[1] for c in candidate_ids}) == 1:
            return self._answer_batched(question_ids, candidate_ids, cache, graph and isinstance(cache, GPUCache))
        graph = graph and isinstance(cache, GPUCache)
        means, sums = [], []
        for answer_ids in candidate_ids:
            ids = torch.cat((question_ids, answer_ids), dim=1)
            fork = cache.fork()
            if graph:
                fg = self.frame_graph([fork], ids.shape[1], answer_ids.shape[1] + 1)
                logits = fg.step(ids=ids)
                fg.batch.release()
            else:
                logits = self.model(fork, ids=ids, logits=answer_ids.shape[1] + 1)
            ll = logits[0, :-1].log_softmax(-1).gather(1, answer_ids[0][:, None])[:, 0]
            means.append(ll.mean())
            sums.append(ll.sum())
        means, sums = torch.stack(means), torch.stack(sums)
        values = means.tolist()
        return dict(scores=values, summed=sums.tolist(), prediction=max(range(len(values)), key=values.__getitem__))

    @torch.inference_mode()
    def ingest_many(self, frames, bits, mode, qa_reserve=192, graph=False):
        """ingest() for B requests stepped together (request batching, not in the
        reference): frames[r] / bits[r] are request r's frame embeddings and
        precisions; every request has the same number of frames and frame
        lengths. Each frame step runs the B frames through the decoder at once,
        every request appended to its own cache. graph=True replays the frame
        steps from one captured CUDA graph (FrameGraph; frames of equal length).
        Returns the B caches."""
        b = len(frames)
        if b == 0 or len(bits) != b or len({len(f) for f in frames}) != 1:
            raise ValueError('request batching needs one bit list per request and equal frame counts')
        if mode == 'native':
            return [self.ingest(f, bt, mode, qa_reserve) for f, bt in zip(frames, bits)]
        caches = [self.create_cache([f.shape[1] for f in fr], mode, qa_reserve) for fr in frames]
        self.model.forward_many(caches, ids=self.prefix_ids.expand(b, -1))
        lengths = {e.shape[1] for fr in frames for e in fr}
        stepper = self.frame_graph(caches, lengths.pop()) if graph and len(lengths) == 1 else None
        for i in range(len(frames[0])):
            step = [fr[i] for fr in frames]
            if len({e.shape[1] for e in step}) != 1:
                raise ValueError('request batching needs equal frame lengths at each step')
            for cache, bt in zip(caches, bits):
                cache.select(bt[i], i)
            if stepper is not None:
                stepper.step(embeds=torch.cat(step, dim=0))
            else:
                self.model.forward_many(caches, embeds=torch.cat(step, dim=0))
        if stepper is not None:
            stepper.batch.release()  # the graph is kept for the next batch, the caches are not
        for cache in caches:
            cache.select(16, -1)
            cache.reserve(16, cache.host_counts[16] + qa_reserve)
            if len(set(cache.seen)) != 1:
                raise RuntimeError('Decoder layers disagree about the cache length')
        return caches

    @torch.inference_mode()
    def answer_many(self, questions, candidates, caches, graph=False):
        """answer() (the reference's candidate protocol) for B requests at once:
        candidate j of every request runs on a fork of that request's cache, the B
        forks in one batched forward. questions[r] [1, q], candidates[r] a list of
        [1, c] ids; every request has the same question and candidate lengths.
        graph=True replays each candidate step from one captured CUDA graph.
        Returns one answer() dict per request."""
        b = len(caches)
        if len(questions) != b or len(candidates) != b or len({len(c) for c in candidates}) != 1:
            raise ValueError('one question and the same number of candidates per request')
        if not all(isinstance(c, GPUCache) for c in caches):
            return [self.answer(q, c, cache) for q, c, cache in zip(questions, candidates, caches)]
        means = [[] for _ in range(b)]
        sums = [[] for _ in range(b)]
        for j in range(len(candidates[0])):
            answers = [c[j] for c in candidates]
            ids = torch.cat([torch.cat((q, a), dim=1) for q, a in zip(questions, answers)], dim=0)  # [B, q + c]
            forks = [cache.fork() for cache in caches]
            if graph:
                fg = self.frame_graph(forks, ids.shape[1], answers[0].shape[1] + 1)
                logits = fg.step(ids=ids)
                fg.batch.release()
            else:
                logits = self.model.forward_many(forks, ids=ids, logits=answers[0].shape[1] + 1)
            target = torch.cat(answers, dim=0)                                                  # [B, c]
            ll = logits[:, :-1].log_softmax(-1).gather(2, target[..., None])[..., 0]           # [B, c]
            for r in range(b):
                means[r].append(ll[r].mean())
                sums[r].append(ll[r].sum())
        out = []
        for r in range(b):
            values = torch.stack(means[r]).tolist()
            out.append(dict(scores=values, summed=torch.stack(sums[r]).tolist(),
                            prediction=max(range(len(values)), key=values.__getitem__)))
        return out

    def _answer_batched(self, question_ids, candidate_ids, cache, graph=False):
        fork = cache.fork()
        ids = torch.cat(candidate_ids, dim=0)                                         # [B, n]
        if graph:  # the question appended by one graph replay, the candidates attended by another
            fg = self.frame_graph([fork], question_ids.shape[1], 1)
            first = fg.step(ids=question_ids)[0, -1].log_softmax(-1)                  # predicts token 0
            fg.batch.release()
            fg = self.frame_graph([fork] * ids.shape[0], ids.shape[1], ids.shape[1], append=False)
            rest = fg.step(ids=ids)[:, :-1].log_softmax(-1)
            fg.batch.release()
        else:
            first = self.model(fork, ids=question_ids, logits=1)[0, -1].log_softmax(-1)  # predicts token 0
            rest = self.model.forward_chunks(fork, ids, logits=ids.shape[1])[:, :-1].log_softmax(-1)
        ll = torch.cat((first[ids[:, :1]], rest.gather(2, ids[:, 1:, None])[..., 0]), dim=1)  # [B, n]
        means, sums = ll.mean(1), ll.sum(1)
        values = means.tolist()
        return dict(scores=values, summed=sums.tolist(), prediction=max(range(len(values)), key=values.__getitem__))


def synthetic_request(cfg, seed, frames=64, frame_tokens=64, question_tokens=32, candidates=4,
                      candidate_tokens=24, device='cuda'):
    """Seeded stand-in for one video QA request: frame embeddings scaled like the
    decoder's token embeddings, question and candidate token ids."""
    gen = torch.Generator().manual_seed(10_000 + seed)
    embeds = [(torch.randn(1, frame_tokens, cfg.hidden, generator=gen) * cfg.init_std).to(torch.bfloat16).to(device)
              for _ in range(frames)]
    question = torch.randint(0, cfg.vocab, (1, question_tokens), generator=gen).to(device)
    cands = [torch.randint(0, cfg.vocab, (1, candidate_tokens), generator=gen).to(device) for _ in range(candidates)]
    return embeds, question, cands
