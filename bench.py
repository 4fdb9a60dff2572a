#!/usr/bin/env python
"""Benchmark of the packed-KV hot path on B200 (one process per GPU).

Workload (BASELINE config 3 at its 8K point, on a whole 32-layer cache): a
SmolLM2-360M-shape cache (32 layers, 5 KV heads, 15 query heads, head_dim 64)
holds P = 8128 packed history tokens in 64-token frames whose precision is drawn
from the seeded 50/30/20 int4/int8/bf16 mix; keys carry 4 seeded 8x outlier
channels. One STEP is the 64-token frame-append attention of all 32 layers
(GPUCache.attend per layer: 64 queries over 8128 packed + 64 native tokens). The
32 layers' caches (~185 MB) exceed the 126 MB L2, so every step streams its
history from HBM. Each rank builds its own independent request (seed = rank):
weak scaling, no collective on the data path.

Printed (rank 0, one JSON line):
  value      packed-KV attention HBM GB/s, algorithmic bytes of all ranks / max time
             (device-resident inputs; the 32-layer sweep replayed as a CUDA graph)
  e2e        same metric through the public API (GPUCache.attend) with pinned host
             buffers: per step one H2D copy of every layer's q, k and v and one D2H
             copy of the outputs inside the timing
  decode_us_per_layer_call   1 query after the same history, per layer call
  frame_append_tokens_per_s  pack + attend of a 64-token frame on all 32 layers (one fused launch each)
  c1..c5     the other BASELINE configurations (C3 also at past 1024 / 4096), each with
             a CPU baseline of the oracle port on a bounded, stated sample
  roofline   dominant op (attention) vs measured HBM peak; roofline_tensor vs bf16
  cpu_baseline  the reference CPU path (dequantise + torch SDPA, oracle port) on a
             bounded sample of the same workload, all host cores
`--impl reference` times only that CPU path and prints its own line.
"""
import argparse
import datetime
import json
import os
import random
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / 'dynamic-kv-cache_b200')):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

LAYERS, HEADS, GROUP, DIM = 32, 5, 3, 64
PAST, NQ, FRAME = 8128, 64, 64
MIX = ([4, 8, 16], [0.5, 0.3, 0.2])
ROW_BYTES = {4: 32 + 8, 8: 64 + 8, 16: 128}  # code bytes + (offset, scale) per row
METRIC = 'packed-KV attention HBM GB/s at 8K ctx'
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one attention_tc_kernel
# launch of this exact call shape (P = 8128, 64 queries, 15Q/5KV, the frame mix of
# seed 0), from an ncu capture of `bench.py --layers 2` (the first launch after six
# warm-up launches). It is a recorded figure, not measured by this run: a kernel
# change is re-captured and this constant updated with it.
NCU_TRAFFIC_BYTES = 5_800_192
# The same for the attention_combine_kernel launch that merges that call's splits
# (cold: ncu flushes the caches, so the partials come from DRAM; live they are in L2).
NCU_COMBINE_TRAFFIC_BYTES = 6_610_432
# The same for one attention_split_kernel launch of the decode shape (one query after
# the same 8128 tokens), from the matching capture with -k regex:attention_split.
NCU_DECODE_TRAFFIC_BYTES = 5_586_944
WORKLOAD = 'C3 frame-append attention, 8K ctx, 32-layer cache'
E2E_GROUPS = 2  # layer groups whose transfers overlap the other groups' attention calls


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=3000)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', choices=['ours', 'reference'], default='ours')
    ap.add_argument('--cpu-seconds', type=float, default=12.0, help='CPU-baseline sample budget')
    ap.add_argument('--e2e-steps', type=int, default=200)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--configs', default='c1,c2,c3,c4,c5',
                    help='extra BASELINE configurations reported in the same line (comma list, or "none")')
    ap.add_argument('--c5-requests', type=int, default=64, help='C5 requests in total, split across ranks')
    ap.add_argument('--c5-batch', type=int, default=8,
                    help='C5 requests stepped together per GPU (request batching); 8 divides 64 / 8 GPUs, so '
                         'every GPU count forms the same batches and the scores stay bit-identical')
    ap.add_argument('--c5-sequential', type=int, default=4,
                    help='C5 requests per rank also run one at a time (the reference protocol) for comparison')
    ap.add_argument('--layers', type=int, default=LAYERS,
                    help='cache layers (the per-call workload is unchanged; fewer layers only shrink '
                         'the set-up for profiler captures)')
    args = ap.parse_args()
    globals()['LAYERS'] = args.layers
    return args


def frame_plan(seed, past=None):
    past = PAST if past is None else past
    frames = (past + FRAME - 1) // FRAME
    bits = random.Random(seed).choices(MIX[0], weights=MIX[1], k=frames)
    sizes = [FRAME] * (frames - 1) + [past - FRAME * (frames - 1)]
    return list(zip(bits, sizes))


def attention_bytes(plan, nq=None):
    """Algorithmic HBM bytes of one attention call: each history row once (codes +
    metadata), the 5-byte token map entry per history token, Q and the output
    once, the native new K/V once."""
    nq = NQ if nq is None else nq
    hist = sum(2 * HEADS * n * ROW_BYTES[b] for b, n in plan)
    maps = 5 * sum(n for _, n in plan)
    q_out = 2 * nq * HEADS * GROUP * DIM * 2
    new_kv = 2 * nq * HEADS * DIM * 2
    return hist + maps + q_out + new_kv


def attention_flops(nq=None):
    nq = NQ if nq is None else nq
    return 4 * HEADS * GROUP * DIM * (nq * PAST + nq * (nq + 1) // 2)


def attention_exps(nq=None):
    """Exponentials of one call: one per visible (query row, key) pair."""
    return attention_flops(nq) // (4 * DIM)


def pack_bytes(bits):
    return 2 * HEADS * FRAME * DIM * 2 + 2 * HEADS * FRAME * ROW_BYTES[bits]


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, device_index):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ['nvidia-smi', f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits', '-lms', '200',
                 '-i', str(device_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['nvidia-smi unavailable']}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], [], set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(',')]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == 'active':
                    reasons.add(name)
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': max(smax) if smax else None,
                'reasons': sorted(reasons), 'samples': len(sm)}


def build_cache(seed, device, past=None, layers=None):
    from src.gpu_cache import GPUCache
    layers = LAYERS if layers is None else layers
    gen = torch.Generator(device=device).manual_seed(seed)
    outliers = torch.randperm(DIM, generator=torch.Generator().manual_seed(seed))[:4].to(device)
    plan = frame_plan(seed, past)
    cache = GPUCache(None, layers=layers, heads=HEADS, device=device)
    for f, (bits, n) in enumerate(plan):
        cache.select(bits, f)
        for layer in range(layers):
            k = torch.randn(1, HEADS, n, DIM, generator=gen, device=device)
            k[..., outliers] *= 8
            v = torch.randn(1, HEADS, n, DIM, generator=gen, device=device)
            cache.append(k.bfloat16(), v.bfloat16(), layer)
    for b in (4, 8, 16):  # room for the timed frame appends without growth
        cache.reserve(b, cache.host_counts[b] + FRAME)
    q = torch.randn(layers, 1, HEADS * GROUP, NQ, DIM, generator=gen, device=device).bfloat16()
    kn = torch.randn(layers, 1, HEADS, NQ, DIM, generator=gen, device=device)
    kn[..., outliers] *= 8
    kn = kn.bfloat16()
    vn = torch.randn(layers, 1, HEADS, NQ, DIM, generator=gen, device=device).bfloat16()
    cache.check()
    return cache, plan, q, kn, vn


def cpu_baseline(seconds, threads=None):
    """Times the reference CPU path (oracle port: unpack every stored frame, keep
    the current frame native, torch SDPA) on layers of the same workload."""
    import numpy as np
    from oracle import cpu_path, pools
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    plan = frame_plan(0)
    gen = torch.Generator().manual_seed(0)
    outliers = torch.randperm(DIM, generator=gen)[:4]

    def bits_np(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    frames = []
    for bits, n in plan:
        k = torch.randn(1, HEADS, n, DIM, generator=gen)
        k[..., outliers] *= 8
        v = torch.randn(1, HEADS, n, DIM, generator=gen)
        frames.append(pools.pack_frame(bits_np(k.bfloat16()), bits_np(v.bfloat16()), bits))
    q = torch.randn(1, HEADS * GROUP, NQ, DIM, generator=gen).bfloat16().float()
    kn = torch.randn(1, HEADS, NQ, DIM, generator=gen).bfloat16().float()
    vn = torch.randn(1, HEADS, NQ, DIM, generator=gen).bfloat16().float()
    bits = random.Random(0).choices(MIX[0], weights=MIX[1], k=len(plan) + 1)[-1]  # the appended frame's
    cpu_path.cpu_cache_update(frames, q, kn, vn, bits)  # warm-up
    calls, start = 0, time.perf_counter()
    while True:
        cpu_path.cpu_cache_update(frames, q, kn, vn, bits)
        calls += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds or calls >= 10000:
            break
    gbs = attention_bytes(plan) * calls / elapsed / 1e9
    return {'value': gbs, 'unit': 'GB/s', 'cores': threads, 'kind': 'port',
            'sample': f'{calls} single-layer calls (P={PAST}, n={NQ}, 15Q/5KV) of the reference CPU path '
                      f'(MixedPrecisionCache.update: unpack all frames + pack of the current frame\'s K and V at '
                      f'{bits} bits + cat, then torch SDPA) in {elapsed:.1f} s; ms/call {1e3 * elapsed / calls:.2f}'}


def measured_peaks():
    path = ROOT / 'MEASURED_PEAKS.json'
    if path.exists():
        d = json.loads(path.read_text())
        return d['hbm_gbs'], d['bf16_tflops'], 'measured'
    return 6650.0, 1590.0, 'fallback'


def run_reference(args, rank):
    if rank != 0:
        return
    base = cpu_baseline(args.cpu_seconds)
    line = {'impl': 'reference', 'metric': METRIC, 'value': base['value'], 'unit': 'GB/s', 'n_gpus': args.gpus,
            'steps': args.steps, 'warmup': args.warmup, 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic (seeded, BASELINE config 3 shapes)',
            'config': {'workload': WORKLOAD + ' (CPU reference path)', 'past': PAST, 'nq': NQ,
                       'layers_sampled': 'single-layer calls', 'heads': '15Q/5KV', 'head_dim': DIM},
            'cpu_baseline': base,
            'e2e': {'value': base['value'], 'unit': 'GB/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


def bench_c1(seconds=2.0):
    """C1: the reference CPU path, one layer, P = 1024 (16 frames of the 50/30/20 mix), fp32."""
    import numpy as np
    from oracle import cpu_path, pools
    torch.set_num_threads(os.cpu_count())
    gen = torch.Generator().manual_seed(1)
    outliers = torch.randperm(DIM, generator=gen)[:4]
    bits = random.Random(1).choices(MIX[0], weights=MIX[1], k=16)
    frames = []
    for b in bits:
        k = torch.randn(1, HEADS, FRAME, DIM, generator=gen)
        k[..., outliers] *= 8
        v = torch.randn(1, HEADS, FRAME, DIM, generator=gen)
        to_bits = lambda t: t.bfloat16().contiguous().view(torch.int16).numpy().view(np.uint16)
        frames.append(pools.pack_frame(to_bits(k), to_bits(v), b))
    q = torch.randn(1, HEADS * GROUP, NQ, DIM, generator=gen)
    kn, vn = torch.randn(1, HEADS, NQ, DIM, generator=gen), torch.randn(1, HEADS, NQ, DIM, generator=gen)
    new_bits = random.Random(1).choices(MIX[0], weights=MIX[1], k=17)[-1]
    cpu_path.cpu_cache_update(frames, q, kn, vn, new_bits)
    calls, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        cpu_path.cpu_cache_update(frames, q, kn, vn, new_bits)
        calls += 1
    return {'ms_per_call': 1e3 * (time.perf_counter() - t0) / calls, 'cores': os.cpu_count(), 'past': 1024,
            'what': 'reference CPU path (unpack + pack of the current frame + cat + SDPA), one layer, '
                    '64-token append'}


def bench_c3_sweep(device, cases=((1024, 256), (4096, 64))):
    """C3 at the shorter histories of the configuration (past 1024 and 4096; 8128 is the
    headline): as many layers as keep the packed history above L2 (~180 MB), every
    layer's call replayed from one CUDA graph."""
    out = {}
    for past, layers in cases:
        cache, plan, q, kn, vn = build_cache(1100 + past, device, past=past, layers=layers)
        outs = [None] * layers
        stream = torch.cuda.Stream(device)

        def sweep():
            for layer in range(layers):
                outs[layer] = cache.attend(q[layer], kn[layer], vn[layer], layer, past)

        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            sweep()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                sweep()
            for _ in range(3):
                graph.replay()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for _ in range(20):
                graph.replay()
            end.record(stream)
        torch.cuda.synchronize(device)
        cache.check()
        us = 1e3 * start.elapsed_time(end) / 20 / layers
        nbytes = attention_bytes(plan)
        out[str(past)] = {'us_per_layer_call': us, 'GB_per_s': nbytes / (us * 1e-6) / 1e9, 'layers': layers,
                          'bytes_per_call': nbytes, 'working_set_MB': layers * nbytes // 2**20}
        del graph, cache, q, kn, vn, outs
    return out


def bench_c2(device):
    """C2: pack sweep, 32 layers x 5 KV heads, 64-token frames appended one at a time from 0
    to 8192 tokens at fixed 4 / 8 / 16 bits, pool growth included (as in the reference).
    Each sweep runs twice on a new cache: cold (the process maps pool memory of this size
    for the first time) and warm (growth maps pages of regions that earlier caches left,
    as in a serving process); the warm pass is the headline figure, the cold one is
    reported beside it."""
    from src.gpu_cache import GPUCache
    gen = torch.Generator(device=device).manual_seed(2)
    k = torch.randn(LAYERS, 1, HEADS, FRAME, DIM, generator=gen, device=device).bfloat16()
    v = torch.randn(LAYERS, 1, HEADS, FRAME, DIM, generator=gen, device=device).bfloat16()
    out = {}
    launches = (8192 // FRAME) * LAYERS
    for bits in (4, 8, 16):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ms = []
        for _ in range(2):  # cold (first pools of this size in the process), then warm
            cache = None  # the previous cache's pool regions return to the free list first
            cache = GPUCache(None, layers=LAYERS, heads=HEADS, device=device)
            torch.cuda.synchronize(device)
            start.record()
            for f in range(8192 // FRAME):
                cache.select(bits, f)
                for layer in range(LAYERS):
                    cache.append(k[layer], v[layer], layer)
            end.record()
            torch.cuda.synchronize(device)
            ms.append(start.elapsed_time(end))
            cache.check()
        out[str(bits)] = {'GB_per_s': launches * pack_bytes(bits) / (ms[1] * 1e-3) / 1e9,
                          'us_per_layer_append': 1e3 * ms[1] / launches,
                          'us_per_layer_append_cold': 1e3 * ms[0] / launches, 'final_cap': cache.caps[bits]}
        # the same 32 per-layer pack launches of one frame replayed from a CUDA graph
        # (rows 0..63 rewritten each time): the kernel without the eager Python calls
        from src import gpu_kernels as K
        stream = torch.cuda.Stream(device)

        def frame():
            for layer in range(LAYERS):
                K.pack_rows(k[layer], v[layer], *cache._pools(), layer, 0, FRAME, cache.caps[4], cache.caps[8],
                            cache.caps[16], HEADS, DIM, bits, LAYERS, cache.status)

        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            frame()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                frame()
            for _ in range(3):
                graph.replay()
            start.record(stream)
            for _ in range(50):
                graph.replay()
            end.record(stream)
        torch.cuda.synchronize(device)
        gms = start.elapsed_time(end) / 50
        out[str(bits)].update({'GB_per_s_graph': LAYERS * pack_bytes(bits) / (gms * 1e-3) / 1e9,
                               'us_per_layer_append_graph': 1e3 * gms / LAYERS})
        del graph
        cache.check()
    return out


def cpu_config_baselines(model, seconds=2.0):
    """CPU baselines of C2, C4 and C5 (rank 0, all host threads): the oracle port of
    the reference CPU path on bounded samples, extrapolated as stated in each entry."""
    import dataclasses
    import numpy as np
    from oracle import kvq
    from oracle.decoder import OracleDecoder, decoder_params
    torch.set_num_threads(os.cpu_count())
    gen = torch.Generator().manual_seed(5)
    to_bits = lambda t: t.bfloat16().contiguous().view(torch.int16).numpy().view(np.uint16)
    out = {'cores': os.cpu_count(), 'kind': 'port'}
    # C2: the reference quantiser on one (layer, 64-token append): K and V of 5 heads
    k, v = to_bits(torch.randn(1, HEADS, FRAME, DIM, generator=gen)), to_bits(torch.randn(1, HEADS, FRAME, DIM, generator=gen))
    c2 = {}
    for bits in (4, 8, 16):
        kvq.pack(k, bits)
        calls, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds / 3:
            kvq.pack(k, bits), kvq.pack(v, bits)
            calls += 1
        dt = (time.perf_counter() - t0) / calls
        c2[str(bits)] = {'GB_per_s': pack_bytes(bits) / dt / 1e9, 'us_per_layer_append': 1e6 * dt}
    out['c2'] = dict(c2, sample='kv_quantization.pack port (numpy) on the K and V of one (layer, 64-token append)')
    # C4 / C5: the decoder restatement on 2 of the 32 layers over a synthetic packed history
    cfg = dataclasses.replace(model.cfg, layers=2)
    params = {n: t for n, t in decoder_params(model.model).items()
              if not (n.split('.')[-1].isdigit() and int(n.split('.')[-1]) >= 2)}
    oracle = OracleDecoder(cfg, params)
    rnd = random.Random(5)

    def history(frames):
        hist = [[] for _ in range(cfg.layers)]
        for _ in range(frames):
            b = rnd.choices(MIX[0], weights=MIX[1])[0]
            for layer in range(cfg.layers):
                hist[layer].append((kvq.pack(to_bits(torch.randn(1, HEADS, FRAME, DIM, generator=gen)), b),
                                    kvq.pack(to_bits(torch.randn(1, HEADS, FRAME, DIM, generator=gen)), b)))
        return hist

    def timed(hist, n, past, logits):
        x = oracle.p['embed'][torch.randint(0, cfg.vocab, (n,), generator=gen)][None]
        oracle.forward(hist, x, past, logits=logits)
        reps, t0 = 0, time.perf_counter()
        while reps < 1 or time.perf_counter() - t0 < seconds / 3:
            oracle.forward(hist, x, past, logits=logits)
            reps += 1
        return (time.perf_counter() - t0) / reps * model.cfg.layers / cfg.layers

    scaled = f'{cfg.layers} of {model.cfg.layers} layers timed and scaled by {model.cfg.layers / cfg.layers:g}'
    cand = timed(history(96), 56, 96 * FRAME, 25)
    out['c4'] = {'ms_per_4_candidates': 4e3 * cand,
                 'sample': f'one 56-token question + candidate forward over a 6144-token packed history, {scaled}; '
                           'x4 candidates (the reference protocol)'}
    frame = timed(history(32), FRAME, 32 * FRAME, 0)
    out['c5'] = {'frame_append_tokens_per_s': FRAME / frame,
                 'sample': 'one 64-token frame forward over a 2048-token packed history (the mean history of '
                           f'a 64-frame request), {scaled}; one request on all host cores, the same rate for the '
                           '64-request set'}
    return out


def bench_c4(device):
    """C4: candidate scoring over a 96-frame (6144-token) mixed 4/8/16 packed prefix with the
    random-init SmolLM2-360M-shape decoder: 32-token question, 4 x 24-token candidates."""
    from src.decoder import SMOLLM2_360M
    from src.streaming import StreamingModel, bits_for, synthetic_request
    model = StreamingModel(SMOLLM2_360M, device=device, seed=0)
    embeds, question, cands = synthetic_request(SMOLLM2_360M, seed=4, frames=96, device=device)
    cache = model.ingest(embeds, bits_for('dynamic', 96, seed=4), 'dynamic', qa_reserve=64)
    model.answer(question, cands, cache)
    model.answer(question, cands, cache, batched=True)
    model.answer(question, cands, cache, graph=True)  # captures the candidate step once
    model.answer(question, cands, cache, batched=True, graph=True)
    torch.cuda.synchronize(device)
    reps, t0 = 5, time.perf_counter()
    for _ in range(reps):
        ans = model.answer(question, cands, cache)
    torch.cuda.synchronize(device)
    ms = 1e3 * (time.perf_counter() - t0) / reps
    t0 = time.perf_counter()
    for _ in range(reps):
        graphed = model.answer(question, cands, cache, graph=True)
    torch.cuda.synchronize(device)
    ms_graph = 1e3 * (time.perf_counter() - t0) / reps
    t0 = time.perf_counter()
    for _ in range(reps):
        batched_graph = model.answer(question, cands, cache, batched=True, graph=True)
    torch.cuda.synchronize(device)
    ms_batched_graph = 1e3 * (time.perf_counter() - t0) / reps
    t0 = time.perf_counter()
    for _ in range(reps):
        batched = model.answer(question, cands, cache, batched=True)
    torch.cuda.synchronize(device)
    ms_batched = 1e3 * (time.perf_counter() - t0) / reps
    return {'ms_per_4_candidates': ms, 'prefix_tokens': cache.seen[0],
            'scores_mean_ll': ans['scores'], 'summed_ll': ans['summed'],
            'ms_per_4_candidates_batched': ms_batched, 'batched_scores_mean_ll': batched['scores'],
            'ms_per_4_candidates_graph': ms_graph, 'graph_scores_mean_ll': graphed['scores'],
            'ms_per_4_candidates_batched_graph': ms_batched_graph,
            'batched_graph_scores_mean_ll': batched_graph['scores'],
            'note': 'wall time of StreamingModel.answer: the reference protocol (4 forks x question + candidate) '
                    'eager and with each candidate forward replayed from a captured CUDA graph, and batched '
                    '(question once, 4 candidates in one forward) eager and graph-replayed'}, model


def rank_requests(total, world, rank):
    """Request ids of one rank: a contiguous slice of `total` // `world`."""
    per = total // world
    return list(range(rank * per, (rank + 1) * per))


def rank_batches(total, world, rank, batch):
    """The request batches one rank steps together: fixed-size slices of its requests,
    so whenever `batch` divides total // world every GPU count forms the same batches
    (and, with deterministic kernels, the same scores)."""
    mine = rank_requests(total, world, rank)
    return [mine[s:s + batch] for s in range(0, len(mine), batch)]


def max_over_ranks(values, dist):
    """Element-wise max over ranks of a 1-D tensor (the job's time is its slowest rank's)."""
    if dist is not None:
        dist.all_reduce(values, op=dist.ReduceOp.MAX)
    return values


def gather_scores(local, dist, world):
    """Every rank's score rows, in rank order (one all_gather of a few KiB)."""
    if dist is None:
        return local
    gathered = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(gathered, local)
    return torch.cat(gathered)


def scores_digest(scores):
    """SHA-256 of fp32 score rows: equal digests = bit-identical scores."""
    import hashlib
    return hashlib.sha256(scores.detach().float().cpu().contiguous().numpy().tobytes()).hexdigest()


def bench_c5(model, device, rank, world, total, dist, batch, sequential):
    """C5: `total` independent requests (64 frames x 64 tokens, dynamic 4/8/16, seed = request
    id, then 4-candidate scoring) split across ranks; on each rank the requests are stepped
    `batch` at a time through one batched decoder forward per frame (request batching: one
    pack and one attention launch per layer for the whole batch). Scores gathered with NCCL.
    The first `sequential` requests of each rank are also run one at a time through the
    reference's per-request protocol, timed separately, and their scores compared."""
    from src.streaming import bits_for, synthetic_request
    per = total // world
    mine = rank_requests(total, world, rank)
    # inputs (frame embeddings as a vision tower would hand them over, question and
    # candidates) are made on the device before the clock starts
    reqs = {r: synthetic_request(model.cfg, seed=r, frames=64, device=device) for r in mine}
    bits = {r: bits_for('dynamic', 64, seed=r) for r in mine}
    warm = mine[:batch]  # captures the frame-step graph and loads every kernel once
    model.answer_many([reqs[r][1] for r in warm], [reqs[r][2] for r in warm],
                      model.ingest_many([reqs[r][0] for r in warm], [bits[r] for r in warm], 'dynamic',
                                        qa_reserve=64, graph=True), graph=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    scores = []
    for ids in rank_batches(total, world, rank, batch):
        caches = model.ingest_many([reqs[r][0] for r in ids], [bits[r] for r in ids], 'dynamic', qa_reserve=64,
                                   graph=True)
        scores += [a['scores'] for a in model.answer_many([reqs[r][1] for r in ids], [reqs[r][2] for r in ids],
                                                          caches, graph=True)]
        del caches
    torch.cuda.synchronize(device)
    secs = torch.tensor([time.perf_counter() - t0], device=device)
    seq = min(sequential, per)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    seq_scores = []
    for r in mine[:seq]:
        embeds, question, cands = reqs[r]
        cache = model.ingest(embeds, bits[r], 'dynamic', qa_reserve=64)
        seq_scores.append(model.answer(question, cands, cache)['scores'])
    torch.cuda.synchronize(device)
    seq_secs = torch.tensor([time.perf_counter() - t0], device=device)
    diff = torch.tensor([max((abs(a - b) for x, y in zip(seq_scores, scores) for a, b in zip(x, y)), default=0.0)],
                        device=device)
    local = torch.tensor(scores, dtype=torch.float32, device=device)
    secs, seq_secs, diff = max_over_ranks(torch.cat((secs, seq_secs, diff)), dist).split(1)
    all_scores = gather_scores(local, dist, world)
    return {'frame_append_tokens_per_s': per * world * 64 * 64 / float(secs.item()),
            'requests': per * world, 'seconds': float(secs.item()), 'batch_per_gpu': batch,
            'scaling': 'strong (fixed request set)',
            'scores_sha256': scores_digest(all_scores),
            'sequential': {'requests_per_gpu': seq, 'seconds': float(seq_secs.item()),
                           'frame_append_tokens_per_s': seq * world * 64 * 64 / max(float(seq_secs.item()), 1e-9),
                           'max_abs_score_diff_vs_batched': float(diff.item())},
            'note': 'wall time of ingest + scoring with inputs already on the device (one warm-up batch first); '
                    'batched: requests stepped together, each frame step and each candidate step one replay of '
                    'a captured CUDA graph (FrameGraph: one append+attention launch per layer for the whole '
                    'batch); '
                    'sequential: the reference protocol, one request at a time, eager; scores gathered with NCCL '
                    'all_gather'}


def main():
    os.environ.setdefault('CUBLAS_WORKSPACE_CONFIG', ':4096:8')  # deterministic GEMMs for C5
    args = parse()
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if args.impl == 'reference':  # CPU path on rank 0 only; other ranks leave at once
        run_reference(args, rank)
        return
    dist = None
    if world > 1:
        import torch.distributed as dist
        os.environ['NCCL_DEBUG'] = 'WARN'  # keep stdout to the one JSON line
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device('cuda', local))

    device = torch.device('cuda', local)
    torch.cuda.set_device(device)
    cache, plan, q, kn, vn = build_cache(1000 + rank, device)
    stream = torch.cuda.Stream(device)

    # ---- 32-layer attention sweep, captured once and replayed ----
    outs = [None] * LAYERS

    def sweep():
        for layer in range(LAYERS):
            outs[layer] = cache.attend(q[layer], kn[layer], vn[layer], layer, PAST)

    with torch.cuda.stream(stream):
        for _ in range(3):
            sweep()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        sweep()
    torch.cuda.synchronize(device)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(device)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    barrier()
    clocks = ClockSampler(device.index)
    time.sleep(0.25)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        end.record(stream)
    barrier()
    clock = clocks.stop()
    ms_total = start.elapsed_time(end)
    t = torch.tensor([ms_total], device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total = float(t.item())
    ms_step = ms_total / args.steps
    bytes_call = attention_bytes(plan)
    value = world * LAYERS * bytes_call * args.steps / (ms_total * 1e-3) / 1e9
    us_call = 1e3 * ms_step / LAYERS

    # ---- decode-shaped calls: 1 query after the same history, 32 layers, graph replay ----
    dq1, dk1, dv1 = q[:, :, :, :1].contiguous(), kn[:, :, :, :1].contiguous(), vn[:, :, :, :1].contiguous()
    douts = [None] * LAYERS

    def decode_sweep():
        for layer in range(LAYERS):
            douts[layer] = cache.attend(dq1[layer], dk1[layer], dv1[layer], layer, PAST)

    with torch.cuda.stream(stream):
        decode_sweep()
        dgraph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(dgraph, stream=stream):
            decode_sweep()
        for _ in range(args.warmup):
            dgraph.replay()
        start.record(stream)
        for _ in range(20):
            dgraph.replay()
        end.record(stream)
    torch.cuda.synchronize(device)
    decode_us = 1e3 * start.elapsed_time(end) / 20 / LAYERS
    del dgraph

    # ---- frame append (fused pack + attend on a fork, 32 layers), captured and replayed ----
    branch = cache.fork()
    branch.select(16)
    fa_outs = [None] * LAYERS

    def frame_sweep():
        b = branch.fork()
        b.select(16)
        for layer in range(LAYERS):  # append + attend of the frame: one fused launch per layer
            fa_outs[layer] = b.append_attend(q[layer], kn[layer], vn[layer], layer)

    with torch.cuda.stream(stream):
        for _ in range(2):
            frame_sweep()
    torch.cuda.synchronize(device)
    fgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(fgraph, stream=stream):
        frame_sweep()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            fgraph.replay()
    barrier()
    fsteps = max(1, args.steps // 2)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(fsteps):
            fgraph.replay()
        end.record(stream)
    barrier()
    t = torch.tensor([start.elapsed_time(end)], device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    fa_ms_step = float(t.item()) / fsteps
    fa_tokens_s = world * FRAME / (fa_ms_step * 1e-3)

    # ---- e2e through the public API with pinned host buffers ----
    hq = q.cpu().pin_memory()
    hk = kn.cpu().pin_memory()
    hv = vn.cpu().pin_memory()
    hout = torch.empty((LAYERS, 1, NQ, HEADS * GROUP, DIM), dtype=torch.bfloat16).pin_memory()

    # Transfers overlap the attention calls, as a serving loop would do it. Every step
    # copies in all its q / k / v from pinned host memory and copies all its outputs
    # back; the layers come in E2E_GROUPS groups, each group's calls starting once its
    # inputs have landed and its outputs leaving while the next group computes. Inputs
    # and outputs are double-buffered on the device, with uploads and downloads on
    # streams of their own, so step s + 1's uploads only wait for step s - 1's reads of
    # the same buffers and run while step s still computes.
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    dins = [(torch.empty_like(q), torch.empty_like(kn), torch.empty_like(vn)) for _ in range(2)]
    layer_ins = [[(dq[layer], dk[layer], dv[layer]) for layer in range(LAYERS)] for dq, dk, dv in dins]
    e2e_outs = [torch.empty((LAYERS, 1, NQ, HEADS * GROUP, DIM), dtype=torch.bfloat16, device=device)
                for _ in range(2)]
    per = (LAYERS + E2E_GROUPS - 1) // E2E_GROUPS
    groups = [(g, min(g + per, LAYERS)) for g in range(0, LAYERS, per)]
    # per buffer and group: the (device, host) input slices and the output slices
    uploads = [[[(d[lo:hi], h[lo:hi]) for d, h in zip(dins[b], (hq, hk, hv))] for lo, hi in groups] for b in range(2)]
    downloads = [[(e2e_outs[b][lo:hi], hout[lo:hi]) for lo, hi in groups] for b in range(2)]
    read = [None, None]     # per buffer: the calls that read its inputs are done
    fetched = [None, None]  # per buffer: its outputs are in host memory
    steps_done = [0]

    def e2e_step():
        b = steps_done[0] & 1
        steps_done[0] += 1
        compute = torch.cuda.current_stream(device)
        arrived = []
        with torch.cuda.stream(up):
            if read[b] is not None:
                up.wait_event(read[b])
            for group in uploads[b]:
                for d, h in group:
                    d.copy_(h, non_blocking=True)
                arrived.append(up.record_event())
        if fetched[b] is not None:
            compute.wait_event(fetched[b])  # the previous outputs of this buffer have left
        ins = layer_ins[b]
        for (lo, hi), ev, (dout, hdst) in zip(groups, arrived, downloads[b]):
            compute.wait_event(ev)
            torch.stack([cache.attend(*ins[layer], layer, PAST) for layer in range(lo, hi)], out=dout)
            done = compute.record_event()
            with torch.cuda.stream(down):
                down.wait_event(done)
                hdst.copy_(dout, non_blocking=True)
        read[b] = compute.record_event()
        fetched[b] = down.record_event()

    with torch.cuda.stream(stream):
        for _ in range(20):  # warm-up: the host side of the calls and the copies settle
            e2e_step()
        stream.wait_stream(down)
    barrier()
    with torch.cuda.stream(stream):
        start.record(stream)
        up.wait_stream(stream)  # the first timed upload starts inside the timed region
        for _ in range(args.e2e_steps):
            e2e_step()
        stream.wait_stream(down)  # the last step ends when its outputs are in host memory
        end.record(stream)
    barrier()
    t = torch.tensor([start.elapsed_time(end)], device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item()) / args.e2e_steps
    torch.cuda.synchronize(device)
    for layer in range(LAYERS):  # the outputs that reached the host are the graph-replayed ones
        if not torch.equal(hout[layer], outs[layer].cpu()):
            raise RuntimeError(f'e2e output of layer {layer} differs from the graph-replayed call')
    e2e_value = world * LAYERS * bytes_call / (e2e_ms * 1e-3) / 1e9
    h2d = LAYERS * (q[0].numel() + kn[0].numel() + vn[0].numel()) * 2
    d2h = LAYERS * hout[0].numel() * 2
    cache.check()

    from src import gpu_kernels as K
    launches_per_call = K.attention_launches(PAST, NQ, HEADS, GROUP)
    hbm, tflops, peak_kind = measured_peaks()
    achieved = bytes_call / (us_call * 1e-6) / 1e9
    achieved_tf = attention_flops() / (us_call * 1e-6) / 1e12
    sm_mhz = clock.get('sm_mhz') or 1965.0
    mufu_peak = 16 * torch.cuda.get_device_properties(device).multi_processor_count * sm_mhz * 1e6 / 1e12  # T ex2/s
    achieved_ex = attention_exps() / (us_call * 1e-6) / 1e12
    decode_bytes = attention_bytes(plan, nq=1)
    line = {
        'metric': METRIC, 'value': value, 'unit': 'GB/s', 'n_gpus': world, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': ms_step, 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (seeded; BASELINE config 3 shapes and mix)',
        'config': {'workload': WORKLOAD, 'layers': LAYERS, 'kv_heads': HEADS, 'q_heads': HEADS * GROUP,
                   'head_dim': DIM, 'past': PAST, 'nq': NQ, 'mix': '50/30/20 int4/int8/bf16 per frame',
                   'step': '32 x GPUCache.attend (one layer each), CUDA-graph replay',
                   'l2': f'{LAYERS}-layer working set ~{LAYERS * bytes_call // 2**20} MB vs 126 MB L2 '
                         '(larger than L2 at the default 32 layers: no flush needed)',
                   'requests': f'one independent request per rank (seed 1000+rank)', 'parallelism': f'dp{world}'},
        'us_per_layer_call': us_call,
        'decode_us_per_layer_call': decode_us,
        'decode': {'us_per_layer_call': decode_us, 'GB_per_s': decode_bytes / (decode_us * 1e-6) / 1e9,
                   'hbm_frac': decode_bytes / (decode_us * 1e-6) / 1e9 / hbm, 'bytes_per_call': decode_bytes,
                   'traffic': NCU_DECODE_TRAFFIC_BYTES,
                   'kernel': 'attention_split_kernel (split-K, mma.sync, cluster merge; 3 stacked rows per KV head)'},
        'frame_append_tokens_per_s': fa_tokens_s,
        'frame_append_ms_per_frame': fa_ms_step,
        'e2e': {'value': e2e_value, 'unit': 'GB/s', 'h2d_bytes_per_step': h2d, 'd2h_bytes_per_step': d2h,
                'ms_per_step': e2e_ms, 'api': f'per step: q/k/v of all layers copied in from pinned host memory and '
                                              f'32 GPUCache.attend calls (eager), their outputs copied back to pinned '
                                              f'host memory; transfers in {E2E_GROUPS} layer groups on upload and '
                                              f'download streams, overlapping the attention calls (device buffers '
                                              f'double-buffered across steps)'},
        'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': hbm, 'unit': 'GB/s', 'frac': achieved / hbm,
                     'traffic': NCU_TRAFFIC_BYTES, 'peak_kind': peak_kind,
                     'traffic_combine_cold': NCU_COMBINE_TRAFFIC_BYTES if launches_per_call == 2 else None,
                     'bytes_per_launch': bytes_call,
                     'note': 'attention op per layer call: attention_tc_kernel (tcgen05 / TMEM) + '
                             'attention_combine_kernel (merge of the history splits)' if launches_per_call == 2 else
                             'attention op per layer call: attention_tc_kernel (tcgen05 / TMEM), history splits '
                             'merged in the same cooperative launch'},
        'roofline_tensor': {'bound': 'tensor', 'achieved': achieved_tf, 'peak': tflops, 'unit': 'TFLOP/s',
                            'frac': achieved_tf / tflops, 'peak_kind': peak_kind,
                            'flops_per_launch': attention_flops()},
        'roofline_mufu': {'bound': 'mufu', 'achieved': achieved_ex, 'peak': mufu_peak, 'unit': 'T ex2/s',
                          'frac': achieved_ex / mufu_peak, 'exps_per_launch': attention_exps(),
                          'note': 'every exponential on MUFU ex2 at 16 per clock per SM at the sampled SM clock; '
                                  'the kernel moves one pair in four to the FMA pipes'},
        'gpu_launches': args.steps * LAYERS * launches_per_call,
        'clocks': clock,
    }
    configs = set() if args.configs == 'none' else set(args.configs.split(','))
    if 'c2' in configs:
        line['c2_pack_sweep'] = bench_c2(device)
    if 'c3' in configs:
        line['c3_past_sweep'] = bench_c3_sweep(device)
    model = None
    if 'c4' in configs:
        line['c4_candidate_scoring'], model = bench_c4(device)
    elif 'c5' in configs:
        from src.decoder import SMOLLM2_360M
        from src.streaming import StreamingModel
        model = StreamingModel(SMOLLM2_360M, device=device, seed=0)
    if 'c5' in configs:
        line['c5_request_throughput'] = bench_c5(model, device, rank, world, args.c5_requests, dist, args.c5_batch,
                                                 args.c5_sequential)
    if rank == 0 and 'c1' in configs:
        line['c1_cpu_reference_path'] = bench_c1()
    if rank == 0 and model is not None and not args.no_cpu_baseline:
        cpu = cpu_config_baselines(model)
        meta = {'cores': cpu['cores'], 'kind': cpu['kind']}
        if 'c2' in configs:
            line['c2_pack_sweep']['cpu_baseline'] = dict(cpu['c2'], **meta)
        if 'c4' in configs:
            line['c4_candidate_scoring']['cpu_baseline'] = dict(cpu['c4'], **meta)
        if 'c5' in configs:
            line['c5_request_throughput']['cpu_baseline'] = dict(cpu['c5'], **meta)
    if rank == 0 and not args.no_cpu_baseline:
        line['cpu_baseline'] = cpu_baseline(args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph, fgraph
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
