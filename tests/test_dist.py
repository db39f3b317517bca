"""Multi-rank host logic of the request-sharded step, on CPU with gloo.

The data path has no collective; what crosses ranks is the request slice
each rank owns and the reductions of a timed run (slowest rank's time, sum of
tokens).  These run as two gloo processes on 127.0.0.1.
"""
import os
import socket

import pytest

from specdec.dist import shard_range, step_throughput


@pytest.mark.parametrize("n,world", [(0, 1), (5, 1), (32, 2), (33, 2), (7, 4), (64, 8), (3, 8)])
def test_shard_range_covers_each_request_once(n, world):
    seen = []
    sizes = []
    for r in range(world):
        lo, hi = shard_range(n, world, r)
        assert 0 <= lo <= hi <= n
        seen.extend(range(lo, hi))
        sizes.append(hi - lo)
    assert seen == list(range(n))
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)
    with pytest.raises(ValueError):
        shard_range(4, 0, 0)


def test_single_process_throughput_needs_no_group():
    r = step_throughput(None, 250.0, 1000)
    assert r == {"ms_max": 250.0, "tokens": 1000.0, "value": 4000.0}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # rank r: a slower device time and its own token count
        ms = 100.0 + 25.0 * rank
        tokens = 40 + rank
        lo, hi = shard_range(64, world, rank)
        out = step_throughput(dist, ms, tokens, "cpu")
        q.put((rank, lo, hi, out))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_reductions():
    import torch.multiprocessing as mp

    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    # disjoint halves of the 64 requests
    assert [(lo, hi) for _, lo, hi, _ in res] == [(0, 32), (32, 64)]
    # every rank sees the same aggregate: tokens of both ranks over the slowest time
    for _, _, _, out in res:
        assert out["ms_max"] == 125.0
        assert out["tokens"] == 81.0
        assert out["value"] == pytest.approx(81.0 / 0.125)


# ---- collectives of the vocabulary-sharded acceptance (host side)
def _comm_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from specdec.dist import TorchComm, vocab_shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        comm = TorchComm(dist)
        g = comm.all_gather(torch.tensor([rank * 10, rank * 10 + 1], dtype=torch.int64))
        s = comm.all_reduce_sum(torch.tensor([1 << 40, rank], dtype=torch.int64))
        m = comm.all_reduce_max(torch.tensor([-1, rank], dtype=torch.int32))
        q.put((rank, comm.world, comm.rank, g.tolist(), s.tolist(), m.tolist(), vocab_shard(10, world, rank)))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_shard_collectives():
    """TorchComm's all-gather (rank order), int64 sum (exact above 2^32) and
    int32 max across two gloo ranks, and the vocabulary split they use."""
    import torch.multiprocessing as mp

    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_comm_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, (rank, w, crank, g, s, m, shard) in enumerate(res):
        assert (rank, w, crank) == (r, 2, r)
        assert g == [[0, 1], [10, 11]]
        assert s == [2 << 40, 1]
        assert m == [-1, 1]
    assert [x[-1] for x in res] == [(0, 5), (5, 5)]


def test_thread_comm_matches_the_collectives():
    """ThreadComm (virtual ranks as threads, used to test the sharded
    acceptance on one GPU) gathers in rank order and reduces like NCCL."""
    import threading

    import torch

    from specdec.dist import ThreadComm

    world = 3
    comm = ThreadComm(world)
    out = [None] * world

    def run(r):
        v = comm.rank_view(r)
        g = v.all_gather(torch.tensor([r, -r], dtype=torch.int64))
        s = v.all_reduce_sum(torch.tensor([r + 1], dtype=torch.int64))
        m = v.all_reduce_max(torch.tensor([3 - r], dtype=torch.int32))
        out[r] = (v.world, v.rank, g.tolist(), s.tolist(), m.tolist())

    ths = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in ths:
        t.start()
    for t in ths:
        t.join(timeout=60)
    for r in range(world):
        assert out[r] == (3, r, [[0, 0], [1, -1], [2, -2]], [6], [3])
