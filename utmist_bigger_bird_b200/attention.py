"""Drop-in for ``modal_rd/attention.py``: Bigger Bird v3 sparse prefill / dense decode attention.

``RDAttention`` keeps the reference's constructor keywords (lines 79-83), forward signature
(112-135), ``routes`` (143-174), ``sparse_prefill`` (176-206), ``last_routes`` / ``kept``
attributes and ``install`` (262-270). The sparse prefill path (RoPE, routing, sink + window +
routed attention, exact tail) runs in libbb_b200.so on sm_100a; there is no CPU or Triton path,
so CUDA FP16/BF16 inputs are required there. Exact attention for decode, dense layers and short
prompts stays on ``F.scaled_dot_product_attention`` as in the reference (137-141).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _ops
from .bigger_bird_flash import bigger_bird_flash, next_power_of_2

__all__ = ["RDAttention", "install", "rope_inplace", "vertical_budget", "forward_pool",
           "bigger_bird_flash", "route_query_positions", "ROPE_CHUNK"]

ROPE_CHUNK = 8192  # kept for signature compatibility; the kernel is position-wise in one launch


def rope_inplace(x, cos, sin, chunk=ROPE_CHUNK):
    """``apply_rotary_pos_emb`` on x [b, h, t, d] in place (reference lines 51-60), bit-identical
    to the torch expression ``x*cos + rotate_half(x)*sin``; one kernel launch, no transients."""
    return _ops.rope_inplace_(x, cos, sin)


def vertical_budget(n, vertical, vertical_sqrt):
    """Fixed budget, or c*sqrt(n) (rounded to 64) when vertical_sqrt=c > 0 (reference 63-67)."""
    if vertical_sqrt > 0:
        return int(math.ceil(vertical_sqrt * math.sqrt(n) / 64) * 64)
    return vertical


def forward_pool(score, p, back=0):
    """[H, n] -> [H, n]: each key takes the best score among itself, the p - 1 keys before it and
    the ``back`` keys after it (reference 70-75)."""
    p = max(p, 1)
    return F.max_pool1d(F.pad(score[:, None], (p - 1, back), value=-float("inf")), p + back, stride=1)[:, 0]


def route_query_positions(n, r, mode, sink, window, device):
    """Positions of the routing queries (reference 151-155): the last r, or ``linspace`` spread."""
    if mode == "spread":
        if sink + window > n - 1:
            # torch.linspace would produce positions >= n; the reference's q[0][:, qpos] raises.
            raise IndexError(f"spread routing positions reach {sink + window} >= n = {n}")
        return torch.linspace(sink + window, n - 1, r, device=device).long()
    return torch.arange(n - r, n, device=device)


class RDAttention(nn.Module):
    def __init__(self, base, *, sink=64, window=4096, vertical=2048, vertical_sqrt=0.0,
                 n_route=64, route_pool="mean", route_queries="last", exact_tail=0,
                 vertical_scope=0, scope_chunk=4096, kv_evict=False, evict_keep=0, evict_pool=0, evict_obs=0,
                 evict_obs_max=False, evict_pool_back=0, evict_window=0, evict_full_layers=0, dense=False,
                 block_m=64, block_n=64, num_warps=4, num_stages=2):
        super().__init__()
        cfg = base.config
        self.layer_idx = base.layer_idx
        self.head_dim = base.head_dim
        self.num_heads = cfg.num_attention_heads
        self.num_kv_heads = cfg.num_key_value_heads
        self.groups = self.num_heads // self.num_kv_heads
        self.scaling = base.scaling
        self.q_proj, self.k_proj, self.v_proj, self.o_proj = base.q_proj, base.k_proj, base.v_proj, base.o_proj
        self.sink, self.window, self.vertical, self.vertical_sqrt = sink, window, vertical, vertical_sqrt
        if route_pool not in ("mean", "max"):
            raise ValueError("route_pool must be mean or max")
        self.n_route, self.route_pool, self.dense, self.block_m, self.block_n = n_route, route_pool, dense, block_m, block_n
        if route_queries not in ("last", "spread"):
            raise ValueError("route_queries must be last or spread")
        if scope_chunk % block_m or scope_chunk & (scope_chunk - 1):
            raise ValueError("scope_chunk must be a power of two multiple of block_m")
        self.exact_tail, self.route_queries = exact_tail, route_queries
        self.vertical_scope, self.scope_chunk = vertical_scope, scope_chunk
        self.num_warps, self.num_stages = num_warps, num_stages
        self.kv_evict = kv_evict
        self.evict_keep, self.evict_pool, self.evict_obs = evict_keep, evict_pool, evict_obs
        self.evict_full_layers, self.evict_window = evict_full_layers, evict_window
        self.evict_obs_max, self.evict_pool_back = evict_obs_max, evict_pool_back
        self.last_routes = None
        self.kept = None            # [Hkv, m] absolute positions left in the cache after eviction
        self._col = None

    def forward(self, hidden_states, position_embeddings=None, attention_mask=None,
                past_key_values=None, **kwargs):
        b, t, _ = hidden_states.shape
        q = self.q_proj(hidden_states).view(b, t, self.num_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(hidden_states).view(b, t, self.num_kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(hidden_states).view(b, t, self.num_kv_heads, self.head_dim).transpose(1, 2)
        if torch.is_grad_enabled() and q.requires_grad:
            from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
            q, k = apply_rotary_pos_emb(q, k, *position_embeddings)
        else:
            q, k = rope_inplace(q, *position_embeddings), rope_inplace(k, *position_embeddings)
        if past_key_values is not None:
            k, v = past_key_values.update(k, v, self.layer_idx)
        n = k.shape[-2]
        if b != 1:
            raise ValueError("batch size 1 only")
        if self.dense or t < n or n <= self.sink + self.window:
            out = self.exact_attention(q, k, v, t, n)
        else:
            out = self.sparse_prefill(q, k, v)
            if self.kv_evict and past_key_values is not None:
                self.evict(past_key_values, q, k, v)
        out = out.transpose(1, 2).reshape(b, t, -1)
        return self.o_proj(out), None

    def exact_attention(self, q, k, v, t, n):
        if getattr(k, "turbo", None) is not None:
            return k.attend(q, self.scaling)
        return F.scaled_dot_product_attention(q, k, v, is_causal=t == n and t > 1,
                                              scale=self.scaling, enable_gqa=True)

    def route_budget(self, n):
        return min(vertical_budget(n, self.vertical, self.vertical_sqrt), max(0, n - self.sink - self.window))

    def routes(self, q, k):
        """Per-head top-V key columns by mean (or max) softmax prob of the routing queries,
        sorted ascending, int32 ``[H, budget]`` (reference 143-174). One fused router launch
        sequence; K stays at KV-head width."""
        if not q.is_cuda or q.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("Bigger Bird (sm_100a) requires CUDA FP16/BF16")
        n = k.shape[-2]
        budget = self.route_budget(n)
        r = min(self.n_route, n)
        qpos = route_query_positions(n, r, self.route_queries, self.sink, self.window, q.device)
        col = torch.empty(self.num_heads, n, device=q.device, dtype=torch.float32) if self.kv_evict else None
        idx = _ops.routes_(q[0], k[0], qpos, sink=self.sink, window=self.window, budget=budget,
                           scaling=self.scaling, pool=self.route_pool, out_col=col)
        if self.kv_evict:
            self._col = col
        return idx

    def sparse_prefill(self, q, k, v):
        """Routes, then the main sparse pass over rows [0, n - r) and the exact causal tail over
        the last r = min(exact_tail, n) rows (reference 176-206). Output ``[1, H, n, d]`` with
        ``[n, H, d]`` storage, so ``transpose(1, 2).reshape`` is free."""
        n = k.shape[-2]
        idx = self.routes(q, k)
        self.last_routes = idx
        bh = self.num_heads
        Q, K, V = q[0], k[0], v[0]
        if self.vertical_scope:
            chunk = self.scope_chunk
            groups = -(-n // chunk)
            starts = torch.arange(groups, device=q.device) * chunk
            active = (starts + chunk > n - self.vertical_scope)[None, :, None]
            routed = torch.where(active, idx[:, None, :], torch.full_like(idx[:, None, :], -1)).contiguous()
        else:
            chunk, routed = max(self.block_m, next_power_of_2(n)), idx.view(bh, 1, -1)
        out = torch.empty((n, bh, self.head_dim), dtype=q.dtype, device=q.device).permute(1, 0, 2)
        r = min(self.exact_tail, n)
        _ops.flash_(Q, K, V, routed, out, front=min(self.sink, n), window=self.window, num_heads=bh,
                    kv_groups=self.groups, route_chunk=chunk, scale=self.scaling, row_begin=0,
                    row_end=n - r)
        if r:
            none = torch.full((bh, 1, 1), -1, dtype=torch.int32, device=q.device)
            _ops.flash_(Q[:, n - r:], K, V, none[:, :, :0], out[:, n - r:], front=0, window=n,
                        num_heads=bh, kv_groups=self.groups, route_chunk=max(64, next_power_of_2(n)),
                        scale=self.scaling)
        return out[None]

    def _evict_col(self, q, k):
        """[H, n] exact-attention column scores of the last ``evict_obs`` queries: per query head,
        the softmax over all keys of each of those queries (bf16/fp16 matmul output, then fp32),
        pooled by mean or, with ``evict_obs_max``, max (reference 214-222). Computed by the routing
        kernels with no sink/window columns and no top-k."""
        n = k.shape[-2]
        r = min(self.evict_obs, n)
        qpos = torch.arange(n - r, n, device=q.device)
        col = torch.empty(self.num_heads, n, device=q.device, dtype=torch.float32)
        _ops.routes_(q[0], k[0], qpos, sink=0, window=0, budget=0, scaling=self.scaling,
                     pool="max" if self.evict_obs_max else "mean", out_col=col)
        return col

    def evict_scores(self, q, k):
        """[Hkv, n] key importance from the last ``evict_obs`` queries: exact softmax, mean (or
        max) over those queries, max over each KV head's query group (reference 209-224)."""
        hk, g = self.num_kv_heads, self.groups
        return self._evict_col(q, k).view(hk, g, -1).amax(1)

    def evict(self, cache, q, k, v):
        """Rewrite this layer's cache to sink + kept middle + window keys per KV head (reference
        226-259): one native call computes the priorities (routed columns first, then the pooled
        routing or exact-attention scores), selects the kept middle keys and gathers K/V."""
        n = k.shape[-2]
        g, hk = self.groups, self.num_kv_heads
        idx, col, self._col = self.last_routes, self._col, None
        if self.layer_idx < self.evict_full_layers:
            self.kept = torch.arange(n, device=k.device)[None].expand(hk, -1)
            return
        if self.evict_obs:
            col = self._evict_col(q, k)
        w = min(max(self.window, self.evict_window), n - self.sink)
        extra = min(max(self.evict_keep, g * idx.shape[-1]) if self.evict_keep else g * idx.shape[-1],
                    n - self.sink - w)
        pool = self.evict_pool if (self.evict_pool > 1 or self.evict_pool_back) else 0
        kk, vv, pos = _ops.kv_evict_(idx, col, k[0], v[0], sink=self.sink, window=w, keep=extra,
                                     pool=pool, pool_back=self.evict_pool_back)
        layer = cache.layers[self.layer_idx]
        layer.keys, layer.values = kk[None], vv[None]
        self.kept = pos


def install(model, arm, dense_layers=(), **kw):
    """Patch every decoder layer; ``dense_layers`` stay exact (reference 262-270)."""
    for i, layer in enumerate(model.model.layers):
        base = layer.self_attn
        base = getattr(base, "_rd_base", base)
        new = RDAttention(base, dense=(arm == "dense_rd" or i in dense_layers), **kw)
        new._rd_base = base
        layer.self_attn = new
    return model
