"""The multi-GPU host logic of bench.py on CPU, as world-size-2 gloo ranks: request
partitioning, the fixed request batches (the same at every GPU count), the
max-over-ranks timing reduction and the all_gather + SHA-256 of the scores that
checks bit-identity across GPU counts."""
import datetime
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT

import bench


def _scores(ids):
    """Deterministic stand-in scores of requests `ids` (4 candidates each)."""
    return torch.tensor([[r * 0.25 + j / 8 for j in range(4)] for r in ids], dtype=torch.float32)


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank(rank, world, port, queue):
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist
    import bench as b
    dist.init_process_group('gloo', init_method=f'tcp://127.0.0.1:{port}', rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        gathered = b.gather_scores(_scores(b.rank_requests(64, world, rank)), dist, world)
        slowest = b.max_over_ranks(torch.tensor([1.0 + rank, 5.0 - rank]), dist)
        queue.put((rank, b.scores_digest(gathered), tuple(gathered.shape), slowest.tolist()))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_gather_the_single_process_scores():
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    single = bench.scores_digest(_scores(range(64)))
    for rank, digest, shape, slowest in results:
        assert digest == single and shape == (64, 4)
        assert slowest == [2.0, 5.0]


@pytest.mark.parametrize('world', [1, 2, 4, 8])
def test_every_gpu_count_forms_the_same_request_batches(world):
    one_gpu = bench.rank_batches(64, 1, 0, 8)
    batches = [b for r in range(world) for b in bench.rank_batches(64, world, r, 8)]
    assert batches == one_gpu
    assert sorted(i for r in range(world) for i in bench.rank_requests(64, world, r)) == list(range(64))
