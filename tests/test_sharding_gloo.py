"""KV-head sharding host logic on CPU with world_size-2 gloo process groups."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from utmist_bigger_bird_b200.sharding import gather_heads, kv_head_shard, query_heads_of, reduce_step


def test_partition_covers_every_head_once():
    for world in (1, 2, 4, 8):
        owned = [h for r in range(world) for h in kv_head_shard(r, world, 8)]
        assert owned == list(range(8))
        q = [h for r in range(world) for h in query_heads_of(kv_head_shard(r, world, 8), 4)]
        assert q == list(range(32))
    with pytest.raises(ValueError):
        kv_head_shard(0, 3, 8)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, per, d = 5, 2, 3
        kv = kv_head_shard(rank, world, 4)
        heads = query_heads_of(kv, 2)
        # each rank's output columns hold its query heads' ids: the gather must restore head order
        local = torch.tensor([[float(h) for h in heads for _ in range(d)]] * n)
        full = gather_heads(local)
        ms, fl = reduce_step(10.0 + rank, 100.0 * (rank + 1), "cpu")
        q.put((rank, full.tolist(), ms, fl))
    finally:
        dist.destroy_process_group()


def test_gather_and_step_reduction_over_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want_row = [float(h) for h in range(8) for _ in range(3)]
    for rank, full, ms, fl in results:
        assert all(row == want_row for row in full)
        assert ms == 11.0 and fl == 300.0
