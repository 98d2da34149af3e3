"""Multi-process host logic of the request-sharded replicas, on CPU with the gloo backend.

Each rank of ``bench.py`` is an independent engine replica; the only cross-rank step is the
aggregation after the timed region (max of the times, sum of the tokens), tested here with two
gloo ranks. The ranks share one seeded trace, request i on rank i mod N: their shards are disjoint
and together are the whole trace (config 1 per rank and the config-4 Poisson trace alike).
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench

        dev, wall, tok = bench.aggregate(1.0 + rank, 2.0 + 3 * rank, 100.0 * (rank + 1), torch.device("cpu"))
        prompts, max_new, depths = bench.rank_workload(0, 4, 16, rank, world)
        _p, _m, _d, arrivals = bench.config4_trace(0, 10, 200.0, 16)
        mine = bench.shard(arrivals, rank, world)
        out.put((rank, dev, wall, tok, [p[:5] for p in prompts], sum(max_new), mine))
    finally:
        dist.destroy_process_group()


def test_two_rank_aggregation_and_distinct_shards():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, dev, wall, tok, _heads, _n, _arr in results:
        assert dev == 2.0 and wall == 5.0 and tok == 300.0, rank
    import bench

    whole, _m, _d = bench.workload(bench.replica_seed(0, 0), 8, 16)
    assert results[0][4] == [p[:5] for p in whole[0::2]] and results[1][4] == [p[:5] for p in whole[1::2]]
    _p, _m, _d, arrivals = bench.config4_trace(0, 10, 200.0, 16)
    assert sorted(results[0][6] + results[1][6]) == sorted(arrivals)
    assert arrivals == sorted(arrivals) and arrivals[0] == 0.0


def test_single_process_aggregation_is_identity():
    import bench

    if dist.is_initialized():
        pytest.skip("process group already initialised")
    assert bench.aggregate(1.5, 2.5, 7.0, torch.device("cpu")) == (1.5, 2.5, 7.0)
