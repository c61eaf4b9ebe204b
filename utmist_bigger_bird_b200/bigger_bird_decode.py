"""Split-K sparse decode attention for one new query token (drop-in for
``kernels/bigger_bird_decode.py:bigger_bird_decode``), on the library's CUDA kernels.

Each query head attends to the front (sink) keys, the last ``window`` keys and its routed keys; the
virtual key list front | window | routed is cut into ``splits`` chunks whose partial softmaxes are
merged (flash-decoding). Keys and values are read in place from the cache. ``n`` may be a 1-element
GPU integer tensor holding the current cache length, read by the kernels at run time, so a CUDA
graph captured once stays valid as the cache grows inside a fixed-capacity buffer. With front=0,
window=capacity and no routed keys this is plain (dense) flash-decoding over the first n keys.

Route groups: pooled routes (``indices`` [Hkv, R]) are shared by the query heads of a KV head;
per-head routes (``indices`` [H, R]) give each query head its own key list. Routed positions must
lie in [front, n - window) and be unique per row.
"""
from __future__ import annotations

import torch

from . import _ops

__all__ = ["bigger_bird_decode"]


def bigger_bird_decode(q, k, v, indices, *, front=64, window=4096, scale=1.0, n=None, splits=None,
                       block_n=64, num_warps=4, num_stages=2):
    """q [H, D] (one token), k / v [Hkv, N, D] (any strides, e.g. a cache view), indices int [Hkv or H, R].
    ``n``: current length as a 1-element GPU int tensor (CUDA-graph safe); default all N keys.

    Returns [H, D] in q's dtype. ``splits`` defaults to enough chunks for ~4 CTAs per SM;
    ``block_n``, ``num_warps`` and ``num_stages`` are accepted for compatibility (tiling is fixed)."""
    if not q.is_cuda or q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("bigger_bird_decode requires CUDA FP16/BF16")
    h, d = q.shape
    hk, cap, _ = k.shape
    if k.shape != v.shape or h % hk or k.shape[-1] != d:
        raise ValueError("q [H,D] and k/v [Hkv,N,D] must match")
    if n is None and cap < front + window:
        raise ValueError("cache shorter than front + window: use dense attention")
    if indices.shape[0] not in (hk, h):
        raise ValueError("indices must be [Hkv, R] (pooled) or [H, R] (per head)")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k and v must share one dtype")
    # int32 and int64 (the routes' dtype) are read as they are; other integer dtypes are widened.
    idx = indices if indices.dtype in (torch.int32, torch.int64) else indices.to(torch.int64)
    if idx.numel() and idx.stride(-1) != 1:
        idx = idx.contiguous()
    q = q if q.stride(-1) == 1 else q.contiguous()
    out = torch.empty((h, d), dtype=q.dtype, device=q.device)
    _ops.decode_(q, k, v, idx if idx.shape[1] else None, out, front=front, window=window, scale=scale, n=n,
                 splits=splits or 0)
    return out
