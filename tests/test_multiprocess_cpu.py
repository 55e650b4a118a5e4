"""Multi-process host logic on CPU (gloo, world size 2): the (batch, head)
sharding that bench.py uses across GPUs covers every pair exactly once with
no overlap, and the job time is the maximum over ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_partition_the_pairs(world):
    seen = []
    for r in range(world):
        a, b = bench.shard(bench.PAIRS, world, r)
        assert b - a in (bench.PAIRS // world, bench.PAIRS // world + 1)
        seen.extend(range(a, b))
    assert seen == list(range(bench.PAIRS))


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ms = 10.0 + 5.0 * rank  # rank 1 is the slow one
        got = bench.max_over_ranks(ms, dist, world, torch.device("cpu"))
        a, b = bench.shard(bench.PAIRS, world, rank)
        sizes = torch.tensor([b - a], dtype=torch.int64)
        dist.all_reduce(sizes)
        q.put((rank, got, int(sizes.item())))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    assert [r[1] for r in res] == [15.0, 15.0]
    assert all(r[2] == bench.PAIRS for r in res)


def _gpt_worker(rank, world, port, q):
    """One gloo rank of the data-parallel GPT driver's host logic: per-rank
    token streams, the weak-scaling token count and the max-over-ranks time."""
    from cuda_transformer_b200 import gpt_case

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, y = gpt_case.rank_batches(1000 + rank, 1, 4, 32, 65)[0]
        got = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(got, x)
        distinct = all(not torch.equal(got[i], got[j])
                       for i in range(world) for j in range(i + 1, world))
        ms = gpt_case.max_over_ranks(20.0 + rank, dist, world, torch.device("cpu"))
        q.put((rank, distinct, ms, gpt_case.tokens_per_step(world, 64, 256)))
    finally:
        dist.destroy_process_group()


def test_gpt_case_host_logic_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gpt_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    assert all(r[1] for r in res)                      # every rank trains on its own tokens
    assert [r[2] for r in res] == [21.0, 21.0]         # the job time is the slowest rank's
    assert all(r[3] == 2 * 64 * 256 for r in res)      # global batch = ranks x 64 sequences
