"""Drop-in for ``kernels/bigger_bird_flash.py`` (reference lines 99-138): same signature, same
validation errors, same output layout, computed by libbb_b200.so on sm_100a.

Semantics (reference ``_attention``, lines 42-96): one softmax over the unique union of the
``front`` sink keys, a causal local window of ``window`` keys, and routed keys ``indices[bh,
group(q), :]`` beyond the window (-1 marks an empty slot). Query j of T sits at absolute
position ``n - T + j``. Query head h reads KV head ``(h // num_heads) * (num_heads //
kv_groups) + (h % num_heads) // kv_groups``. ``block_m``/``block_n``/``num_warps``/
``num_stages`` are tiling hints of the Triton kernel: they are validated (``route_chunk %
block_m``) and otherwise ignored, since the sm_100a kernels pick their own tiles.
"""
from __future__ import annotations

import torch

from . import _ops

__all__ = ["bigger_bird_flash", "next_power_of_2"]


def next_power_of_2(n: int) -> int:
    return 1 if n <= 1 else 1 << (int(n) - 1).bit_length()


def _cdiv(a, b):
    return -(-a // b)


def bigger_bird_flash(q, k, v, indices, *, front=64, window=256, token_mask=None, num_heads=32,
                      route_chunk=None, kv_groups=1, scale=1.0, block_m=64, block_n=64,
                      num_warps=4, num_stages=2):
    """Q [BH,T,D], K/V [BH/kv_groups,N,D]; unique route indices [BH,G,K], -1 marks invalid.

    ``kv_groups`` > 1 reads grouped-query K/V in place (query head h uses KV head h // kv_groups),
    so callers never materialise a repeat_interleave'd copy of K/V. Routing groups must align
    with query tiles. Returns ``[BH,T,D]`` whose storage is ``[T,BH,D]``."""
    if not q.is_cuda or q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("Bigger Bird (sm_100a) requires CUDA FP16/BF16")
    if (k.shape != v.shape or q.ndim != 3 or q.shape[0] != k.shape[0] * kv_groups
            or q.shape[-1] != k.shape[-1] or num_heads % kv_groups):
        raise ValueError("Q [BH,T,D] and K/V [BH/kv_groups,N,D] must have matching heads and dimensions")
    if k.dtype != q.dtype or v.dtype != q.dtype or not (k.is_cuda and v.is_cuda):
        raise ValueError("Q, K and V must be CUDA tensors of one dtype")
    if front < 0 or window < 1:
        raise ValueError("front >= 0 and window >= 1 required")
    bh, t, d = q.shape
    n = k.shape[1]
    if n - t < 0:
        raise ValueError("Key sequence must be at least as long as query sequence")
    if indices.ndim == 2:
        indices = indices[:, None, :]
    route_chunk = route_chunk or max(block_m, next_power_of_2(n))
    if route_chunk % block_m or tuple(indices.shape[:2]) != (bh, _cdiv(n, route_chunk)):
        raise ValueError("Routing groups must cover the sequence and align with query tiles")
    indices = indices.to(device=q.device, dtype=torch.int32).contiguous()
    if token_mask is not None:
        if tuple(token_mask.shape) != (bh // num_heads, n) or token_mask.dtype != torch.bool:
            raise ValueError("token_mask must be boolean [batch,N]")
        token_mask = token_mask.to(q.device).contiguous()
    out = torch.empty((t, bh, d), dtype=q.dtype, device=q.device).permute(1, 0, 2)
    _ops.flash_(q, k, v, indices, out, front=min(front, n), window=window, num_heads=num_heads,
                kv_groups=kv_groups, route_chunk=route_chunk, scale=scale, token_mask=token_mask)
    return out
