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


def _model_worker(rank, world, port, q, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from transformers import LlamaConfig, LlamaForCausalLM
        from utmist_bigger_bird_b200.sharding import shard_llama
        cfg = LlamaConfig(vocab_size=256, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                          num_attention_heads=8, num_key_value_heads=4, max_position_embeddings=1024)
        cfg._attn_implementation = "sdpa"
        torch.manual_seed(0)
        model = LlamaForCausalLM(cfg).eval()
        ids = torch.randint(0, 256, (1, 40), generator=torch.Generator().manual_seed(1))
        with torch.no_grad():
            want = model(ids).logits
        shard_llama(model, rank, world, mode=mode, dense=True)
        a = model.model.layers[0].self_attn
        # grad mode on (parameters require grad): the attention rotates with HF's apply_rotary_pos_emb
        got = model(ids).logits.detach()
        q.put((rank, a.num_heads, a.num_kv_heads, tuple(a.q_proj.weight.shape), (got - want).abs().max().item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["gather", "tensor"])
def test_head_sharded_llama_matches_unsharded_over_gloo(mode):
    """Each rank keeps the q/k/v rows of its KV heads and attends over them; the all-gather before
    o_proj ("gather") or the row-parallel o_proj and tensor-parallel MLP with all-reduces
    ("tensor") rebuild the full layer output: logits equal the unsharded model's on every rank."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_model_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, heads, kv_heads, qshape, err in results:
        assert heads == 4 and kv_heads == 2 and qshape == (4 * 16, 128)
        assert err < 1e-4, err
