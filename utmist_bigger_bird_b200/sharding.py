"""KV-head sharding of the sparse-prefill layer across ranks (one process per GPU).

Routes and attention of query head h touch only KV head h // g (modal_rd/attention.py:157-168,
kernels/bigger_bird_flash.py:56), so a layer splits across P ranks by KV heads with no data
exchange: rank p owns KV heads [p*Hk/P, (p+1)*Hk/P) and their g query heads each. A whole-model
prefill then recombines the per-rank head outputs with one all-gather before o_proj.
"""
from __future__ import annotations

from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.nn as nn

__all__ = ["kv_head_shard", "query_heads_of", "reduce_step", "gather_heads", "GatheredOProj", "RowParallelLinear",
           "shard_llama"]


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


class GatheredOProj(nn.Module):
    """``o_proj`` of a head-sharded attention layer: one all-gather of the ranks' head outputs
    ``[n, H_local*d]`` into a ``[P, n, H_local*d]`` buffer, then the full projection as the sum
    of the P column blocks of the weight (``out = sum_p x_p W_p^T``), so the gathered heads never
    need a transposing copy into ``[n, H*d]``. Every rank ends with the full ``[n, hidden]``."""

    def __init__(self, o_proj: nn.Module, world: int, group=None):
        super().__init__()
        if getattr(o_proj, "bias", None) is not None:
            raise ValueError("GatheredOProj: o_proj with bias is not supported")
        self.weight = o_proj.weight
        self.world, self.group = world, group

    @torch.no_grad()
    def forward(self, x):
        # Inference only: the collective carries no gradient.
        lead, w = x.shape[:-1], x.shape[-1]
        rows = x.reshape(-1, w)
        out = torch.empty((rows.shape[0], self.weight.shape[0]), dtype=x.dtype, device=x.device)
        if self.world == 1:
            torch.mm(rows, self.weight.t(), out=out)
            return out.view(*lead, -1)
        buf = torch.empty((self.world * rows.shape[0], w), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(buf, rows.contiguous(), group=self.group)
        buf = buf.view(self.world, rows.shape[0], w)
        for p in range(self.world):
            wp = self.weight[:, p * w:(p + 1) * w].t()
            if p == 0:
                torch.mm(buf[0], wp, out=out)
            else:
                out.addmm_(buf[p], wp)
        return out.view(*lead, -1)


class RowParallelLinear(nn.Module):
    """The input-column block [lo, hi) of a linear layer: ``y = x_local W[:, lo:hi]^T`` summed over
    the ranks with one NCCL all-reduce (the row-parallel half of a tensor-parallel pair). The
    chunked MLP forward calls ``matmul`` on ``weight`` itself and then ``all_reduce_`` once on its
    whole output."""

    def __init__(self, linear: nn.Linear, lo: int, hi: int, world: int, group=None):
        super().__init__()
        if getattr(linear, "bias", None) is not None:
            raise ValueError("RowParallelLinear: bias is not supported")
        self.weight = nn.Parameter(linear.weight[:, lo:hi].detach().clone(), requires_grad=False)
        self.world, self.group = world, group

    def all_reduce_(self, y):
        if self.world > 1:
            dist.all_reduce(y, group=self.group)
        return y

    @torch.no_grad()
    def forward(self, x):
        return self.all_reduce_(torch.matmul(x, self.weight.t()))


def _rows(linear: nn.Linear, lo: int, hi: int) -> nn.Linear:
    new = nn.Linear(linear.in_features, hi - lo, bias=linear.bias is not None,
                    device=linear.weight.device, dtype=linear.weight.dtype)
    with torch.no_grad():
        new.weight.copy_(linear.weight[lo:hi])
        if linear.bias is not None:
            new.bias.copy_(linear.bias[lo:hi])
    return new


def shard_llama(model, rank: int, world: int, group=None, mode: str = "gather", **attn_kw):
    """Head-shard every decoder layer's attention of a Llama-architecture model over ``world``
    ranks (one process per GPU): rank ``rank`` keeps the q/k/v projection rows of its KV heads and
    their query heads (column-parallel) and runs routes and the sparse attention on those heads
    only. Hidden states and norms stay replicated.

    ``mode="gather"``: ``GatheredOProj`` all-gathers the head outputs before the replicated
    ``o_proj``; the MLP is replicated (one all-gather per layer).
    ``mode="tensor"``: ``o_proj`` is row-parallel over the rank's heads and the SwiGLU MLP is
    tensor-parallel (gate/up column blocks, down row block), each followed by one all-reduce: every
    GEMM of the layer is split over the ranks (two all-reduces per layer).

    ``attn_kw`` go to ``RDAttention`` (e.g. sink, window, vertical, exact_tail). Every rank must
    hold identical weights and call this with the same arguments."""
    if mode not in ("gather", "tensor"):
        raise ValueError("shard_llama: mode must be 'gather' or 'tensor'")
    from .attention import RDAttention
    cfg = model.config
    H, Hk = cfg.num_attention_heads, cfg.num_key_value_heads
    d = getattr(cfg, "head_dim", None) or cfg.hidden_size // H
    kvs = kv_head_shard(rank, world, Hk)
    qh = query_heads_of(kvs, H // Hk)
    q0, q1 = qh[0] * d, (qh[-1] + 1) * d
    k0, k1 = kvs[0] * d, (kvs[-1] + 1) * d
    for layer in model.model.layers:
        base = layer.self_attn
        base = getattr(base, "_rd_base", base)
        local = SimpleNamespace(
            config=SimpleNamespace(num_attention_heads=len(qh), num_key_value_heads=len(kvs)),
            layer_idx=base.layer_idx, head_dim=d, scaling=base.scaling,
            q_proj=_rows(base.q_proj, q0, q1), k_proj=_rows(base.k_proj, k0, k1), v_proj=_rows(base.v_proj, k0, k1),
            o_proj=(GatheredOProj(base.o_proj, world, group) if mode == "gather"
                    else RowParallelLinear(base.o_proj, q0, q1, world, group)))
        layer.self_attn = RDAttention(local, **attn_kw)
        if mode == "tensor":
            mlp = layer.mlp
            inter = mlp.gate_proj.out_features
            if inter % world:
                raise ValueError(f"intermediate size {inter} does not split over {world} ranks")
            i0, i1 = rank * inter // world, (rank + 1) * inter // world
            mlp.gate_proj = _rows(mlp.gate_proj, i0, i1)
            mlp.up_proj = _rows(mlp.up_proj, i0, i1)
            mlp.down_proj = RowParallelLinear(mlp.down_proj, i0, i1, world, group)
    return model

