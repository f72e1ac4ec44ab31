"""Request sharding and multi-rank aggregation of the serving sweep, on CPU.

World-size-2 gloo ranks run the same static-batch serving loop as the GPU
sweep with a CPU stand-in for the prefill; their gathered records must equal
a single-process run over all requests (the data path has no collective, so
sharding may not change any request's result).
"""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tokengate_b200.serving import gather_records, serve_static, shard_requests, static_batches, summarize


def fake_prefill(ids, starts, ends, K):
    first = torch.tensor([[int(sum(x.tolist()) % 997)] for x in ids])
    n_kepts = [s + min(K, e - s) + (len(x) - e) for x, s, e in zip(ids, starts, ends)]
    return first, n_kepts


def _requests(n):
    g = torch.Generator().manual_seed(0)
    return {i: dict(ids=torch.randint(0, 50, (int(30 + 7 * i),), generator=g), start=3, end=20 + i)
            for i in range(n)}


def test_shard_requests_partition():
    for n in (0, 1, 7, 64):
        for world in (1, 2, 4, 8):
            shards = [shard_requests(n, world, r) for r in range(world)]
            flat = sorted(i for s in shards for i in s)
            assert flat == list(range(n))
            assert max(map(len, shards)) - min(map(len, shards)) <= 1
    with pytest.raises(ValueError):
        shard_requests(4, 2, 2)


def test_static_batches():
    assert static_batches(list(range(10)), 4) == [[0, 1, 2, 3], [4, 5, 6, 7], [8, 9]]
    assert static_batches([], 3) == []
    with pytest.raises(ValueError):
        static_batches([1], 0)


def _rank_main(rank, world, port, n, K, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        reqs = _requests(n)
        recs = serve_static(fake_prefill, reqs, shard_requests(n, world, rank), 3, K)
        merged, wall = gather_records(recs, 0.5 + rank)
        if rank == 0:
            q.put((merged, wall))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_equals_single():
    n, K = 11, 5
    single = serve_static(fake_prefill, _requests(n), list(range(n)), 3, K)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, n, K, q)) for r in range(2)]
    for p in procs:
        p.start()
    merged, wall = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    key = lambda r: (r["idx"], r["first_token"], r["n_kept"], r["n_tokens"])
    assert [key(r) for r in merged] == [key(r) for r in sorted(single, key=lambda r: r["idx"])]
    assert wall == 1.5   # slowest rank's wall time
    s = summarize(merged, wall)
    assert s["requests"] == n and s["tokens"] == sum(30 + 7 * i for i in range(n))
