"""Multi-rank logic of bench.py on CPU: two gloo ranks (world size 2)
exchange their step times (max over ranks), gather each other's output
statistics and split the decode-stress sequences by cached keys.  No GPU
involved."""
from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    slowest = bench.max_over_ranks(10.0 + 5.0 * rank, world)
    y = torch.full((3, 4), float(rank + 1))
    y[0, 0] = -2.0 * (rank + 1)
    if rank == 1:
        y[2, 3] = float("nan")
    stats = bench.gather_output_stats([y], world)
    lens = [128 + (i * 977) % 3969 for i in range(256)]
    shards = bench.shard_sequences(lens, world)
    mine = torch.tensor([sum(lens[i] for i in shards[rank])], dtype=torch.float64)
    total = mine.clone()
    dist.all_reduce(total)
    q.put((rank, slowest, shards[rank], float(mine.item()), float(total.item()), stats))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_step_time_and_shards():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, t0, s0, l0, tot0, st0), (r1, t1, s1, l1, tot1, st1) = out
    assert t0 == t1 == 15.0
    # output statistics: both ranks see both ranks' [sum, sum_abs, max_abs, non_finite]
    assert st0 == st1
    assert st0[0] == [9.0, 13.0, 2.0, 0.0]
    assert st0[1] == [16.0, 24.0, 4.0, 1.0]
    assert sorted(s0 + s1) == list(range(256))
    assert tot0 == tot1 == l0 + l1
    assert abs(l0 - l1) <= 4096  # balanced to within one sequence


def test_shard_sequences_single_rank_and_empty():
    import bench
    assert bench.shard_sequences([5, 1, 3], 1) == [[0, 1, 2]]
    assert bench.shard_sequences([], 4) == [[], [], [], []]
    assert bench.max_over_ranks(3.5, 1) == 3.5
