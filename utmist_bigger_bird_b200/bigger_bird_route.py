"""Fused decode routing for one new query token (drop-in for ``kernels/bigger_bird_route.py``):
per KV head, the ``k_route`` cached keys with the highest pooled attention probability (softmax
over all n cached keys separately for each query head, averaged over the query heads that share
the KV head), with the first ``front`` keys and the last ``window`` keys excluded.

  pass 1  split-K over the keys: log2-scaled scores of every key for all query heads of the group
          (each key read once), plus per-chunk softmax statistics
  pass 2  merged statistics -> probabilities averaged over the group, front / window / length masks
  top-k   the routing top-k over [Hkv, capacity] (positions come out ascending)

``n`` may be a 1-element GPU int tensor holding the current cache length, as in
``bigger_bird_decode``.
"""
from __future__ import annotations

import torch

from . import _ops

__all__ = ["pooled_probs", "bigger_bird_route"]


def _check(q, k):
    if not q.is_cuda or q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("bigger_bird_route requires CUDA FP16/BF16")
    h, d = q.shape
    hk, cap, _ = k.shape
    if h % hk or k.shape[-1] != d:
        raise ValueError("q [H,D] and k [Hkv,CAP,D] must match")
    if k.dtype != q.dtype:
        raise ValueError("q and k must share one dtype")
    return q if q.stride(-1) == 1 else q.contiguous()


def pooled_probs(q, k, *, front=64, window=4096, scale=1.0, n=None, splits=None, block_n=64, num_warps=4):
    """q [H, D], k [Hkv, CAP, D] -> [Hkv, CAP] fp32 pooled probabilities; -1 outside [front, n - window)."""
    q = _check(q, k)
    hk, cap, _ = k.shape
    p = torch.empty(hk, cap, device=q.device, dtype=torch.float32)
    _ops.decode_route_(q, k, front=front, window=window, scale=scale, n=n, probs=p, splits=splits or 0)
    return p


def bigger_bird_route(q, k, k_route, *, front=64, window=4096, scale=1.0, n=None, **kw):
    """Indices [Hkv, k_route] (int64, positions ascending) of the highest pooled-probability keys in
    [front, n - window)."""
    q = _check(q, k)
    hk, cap, _ = k.shape
    if not 0 <= k_route <= cap:
        raise ValueError("k_route must lie in [0, capacity]")
    idx = torch.empty(hk, k_route, device=q.device, dtype=torch.int64)  # written as int64 by the top-k
    _ops.decode_route_(q, k, front=front, window=window, scale=scale, n=n, k_route=k_route, idx_out=idx,
                       splits=kw.get("splits") or 0)
    return idx
