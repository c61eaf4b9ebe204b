"""KV-head sharding of the sparse-prefill layer across ranks (one process per GPU).

Routes and attention of query head h touch only KV head h // g (modal_rd/attention.py:157-168,
kernels/bigger_bird_flash.py:56), so a layer splits across P ranks by KV heads with no data
exchange: rank p owns KV heads [p*Hk/P, (p+1)*Hk/P) and their g query heads each. A whole-model
prefill then recombines the per-rank head outputs with one all-gather before o_proj.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["kv_head_shard", "query_heads_of", "reduce_step", "gather_heads"]


def kv_head_shard(rank: int, world: int, kv_heads: int) -> list[int]:
    """KV heads owned by ``rank``: a contiguous, equal block (``kv_heads`` must divide evenly)."""
    if world <= 0 or kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads do not split evenly over {world} ranks")
    per = kv_heads // world
    return list(range(rank * per, (rank + 1) * per))


def query_heads_of(kv_heads: list[int], groups: int) -> list[int]:
    """Query heads served by the given KV heads (GQA group size ``groups``)."""
    return [h * groups + j for h in kv_heads for j in range(groups)]


def reduce_step(ms: float, flops: float, device, group=None) -> tuple[float, float]:
    """(max of the ranks' times, sum of their FLOPs): the whole-job step time and work."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return ms, flops
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    f = torch.tensor([flops], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    dist.all_reduce(f, op=dist.ReduceOp.SUM, group=group)
    return t.item(), f.item()


def gather_heads(out_local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather per-rank attention outputs ``[n, H_local*d]`` (rank order = head order) into
    ``[n, H*d]``, the input layout of o_proj."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return out_local
    n, w = out_local.shape
    buf = torch.empty((world * n, w), dtype=out_local.dtype, device=out_local.device)
    dist.all_gather_into_tensor(buf, out_local.contiguous(), group=group)
    return buf.view(world, n, w).permute(1, 0, 2).reshape(n, world * w)
