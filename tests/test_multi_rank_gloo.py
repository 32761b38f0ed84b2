"""Host-side logic of the data-parallel path on CPU: two gloo ranks each
process their row shard (oracle stands in for the device kernel), the
per-rank times reduce with MAX like bench.py, and the gathered shards equal
the single-process result. No collective is on the data path; the gather
here is only the optional final gather."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cutile_b200.shard import shard_range, weak_offset


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, rows, length, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import oracle as O

    x = (4 * O.normal(rows * length, 7)).reshape(rows, length)
    lo, hi = shard_range(rows, rank, world)
    y = O.softmax(x[lo:hi])
    t = torch.tensor([float(rank + 1)])  # this rank's "kernel time"
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    parts = [None] * world
    dist.all_gather_object(parts, (lo, hi, y))
    if rank == 0:
        q.put((t.item(), parts))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_row_shards_match_single_process():
    from oracle import oracle as O

    rows, length, world = 37, 256, 2
    q = mp.get_context("spawn").SimpleQueue()
    mp.spawn(_worker, args=(world, _free_port(), rows, length, q), nprocs=world, join=True)
    tmax, parts = q.get()
    assert tmax == float(world)  # max over ranks, not rank 0's own time
    parts.sort(key=lambda p: p[0])
    assert parts[0][0] == 0 and parts[-1][1] == rows
    full = O.softmax((4 * O.normal(rows * length, 7)).reshape(rows, length))
    np.testing.assert_array_equal(np.concatenate([p[2] for p in parts]), full)


def test_shard_range_partitions():
    for total in (0, 1, 7, 4096, 131072):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert shard_range(4096, 1, 8, align=128) == (512, 1024)
    assert weak_offset(4096 * 16384, 3) == 3 * 4096 * 16384


def _gather_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from cutile_b200.shard import gather_shards

    local = torch.arange(6, dtype=torch.float32).reshape(3, 2) + 100 * rank
    full = gather_shards(local)
    if rank == 1:
        q.put(full.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_gather_shards_concatenates_in_rank_order():
    q = mp.get_context("spawn").SimpleQueue()
    mp.spawn(_gather_worker, args=(2, _free_port(), q), nprocs=2, join=True)
    full = q.get()
    expect = np.concatenate([np.arange(6, dtype=np.float32).reshape(3, 2) + 100 * r for r in range(2)])
    np.testing.assert_array_equal(full, expect)
