"""CPU oracle for the Bigger Bird v3 sparse-prefill path (TEST INFRASTRUCTURE ONLY).

This module is a numpy restatement of the reference's algorithm. It exists so that the
tests, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of ``bench.py`` can check
the CUDA path; the product (``utmist_bigger_bird_b200``) never imports it.

What it restates (paths inside the reference project derkychen/utmist-bigger-bird):

* ``rope``           -- ``modal_rd/attention.py:51-60`` (``rope_inplace``), i.e. Hugging Face
                        ``apply_rotary_pos_emb`` / ``rotate_half`` (transformers, pinned 5.15.1 in
                        ``modal_rd/app.py:24``; the formula is unchanged in 5.5): each op of
                        ``x*cos + rotate_half(x)*sin`` rounds to the tensor dtype.
* ``vertical_budget`` -- ``modal_rd/attention.py:63-67``.
* ``route_query_positions`` -- ``modal_rd/attention.py:151-155`` (``torch.linspace`` in float32,
                        truncated by ``.long()``; ATen's symmetric linspace formula).
* ``route_scores`` / ``routes`` -- ``modal_rd/attention.py:143-174``: bf16/fp16 scores are the
                        matmul output rounded to the input dtype, then ``.float() * scaling``,
                        causal mask, fp32 softmax over all keys, mean (or max) over the routing
                        queries, sink and window columns forced to -1, top-``budget`` sorted.
* ``flash``          -- ``kernels/bigger_bird_flash_ref.py:10-52`` (same masks: sink, causal
                        window, routed columns beyond the window, route groups, token mask;
                        fully masked rows give 0), computed in fp32, optionally on a subset of
                        query rows so long sequences stay tractable.
* ``sparse_prefill`` -- ``modal_rd/attention.py:176-206`` (routes, optional ``vertical_scope``
                        groups, main pass, exact tail overwriting the last ``exact_tail`` rows).
                        ``route_scores_at`` / ``flash_at`` / ``sparse_prefill_at`` are the same
                        arithmetic given only the query rows to evaluate (long prompts).
* ``decode``         -- ``kernels/bigger_bird_decode.py:21-107``: one query per head over the virtual
                        key list front | window | routed (positions outside [0, n) skipped; a key
                        listed twice counts twice, as in the kernel), exact softmax in fp32.
* ``pooled_probs``   -- ``kernels/bigger_bird_route.py:24-106``: per-head base-2 softmax of the
                        fp32 scores over the first n keys, mean over the KV head's query heads, -1
                        outside [front, n - window).
* ``forward_pool`` / ``evict_positions`` -- ``modal_rd/attention.py:70-75`` and ``:226-259``
                        (``RDAttention.evict``): routed columns first, then the group-max (pooled)
                        column scores, sink and kept window excluded, top-``keep`` sorted; the
                        kept cache is the K/V rows at [sink | selected | window].

Parity is pinned by ``tests/test_oracle_golden.py`` against vectors produced by the reference
itself (``tests/golden/make_golden.py`` imports the reference read-only).
"""
from __future__ import annotations

import math

import numpy as np

__all__ = [
    "bf16_round", "f16_round", "rounder", "rope", "vertical_budget", "route_query_positions",
    "route_scores", "route_scores_at", "routes", "topk_sorted", "route_sets_match", "flash", "flash_at",
    "sparse_prefill", "sparse_prefill_at",
    "forward_pool", "evict_positions", "decode", "pooled_probs",
]


# ----------------------------------------------------------------------------- rounding helpers

def bf16_round(x):
    """float32 -> float32 holding the bfloat16 round-to-nearest-even value (NaN kept)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    out = b.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out)


def f16_round(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def rounder(dtype):
    """Rounding applied by a torch op whose output dtype is ``dtype`` ("bf16", "f16", "f32")."""
    if dtype == "bf16":
        return bf16_round
    if dtype == "f16":
        return f16_round
    if dtype == "f32":
        return lambda a: np.asarray(a, dtype=np.float32)
    raise ValueError(f"unknown dtype {dtype}")


# ----------------------------------------------------------------------------- RoPE

def rope(x, cos, sin, dtype):
    """``x*cos + rotate_half(x)*sin`` with each op rounded to ``dtype``.

    x: [..., T, D] float32 (values representable in ``dtype``); cos/sin: [T, D] float32
    (already in ``dtype``). Restates ``modal_rd/attention.py:51-60`` (chunking there is
    position-wise and does not change results)."""
    rnd = rounder(dtype)
    x = np.asarray(x, dtype=np.float32)
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return rnd(rnd(x * cos) + rnd(rot * sin))


# ----------------------------------------------------------------------------- routing

def vertical_budget(n, vertical, vertical_sqrt):
    """``modal_rd/attention.py:63-67``."""
    if vertical_sqrt > 0:
        return int(math.ceil(vertical_sqrt * math.sqrt(n) / 64) * 64)
    return vertical


def route_query_positions(n, r, mode, sink, window):
    """Routing query positions (``modal_rd/attention.py:151-155``).

    "spread" restates ``torch.linspace(sink + window, n - 1, r).long()``: float32 endpoints,
    ``step = (end - start) / (steps - 1)``, the first ``steps // 2`` values are
    ``start + step * i`` and the rest ``end - step * (steps - 1 - i)``, then truncation."""
    if mode == "spread":
        start, end = np.float32(sink + window), np.float32(n - 1)
        if r == 1:
            vals = np.array([start], dtype=np.float32)
        else:
            step = np.float32((end - start) / np.float32(r - 1))
            i = np.arange(r)
            lo = start + step * i.astype(np.float32)
            hi = end - step * (r - 1 - i).astype(np.float32)
            vals = np.where(i < r // 2, lo, hi).astype(np.float32)
        return vals.astype(np.int64)
    if mode == "last":
        return np.arange(n - r, n, dtype=np.int64)
    raise ValueError("route_queries must be last or spread")


def route_scores(q, k, *, scaling, sink, window, n_route=64, pool="mean", queries="last",
                 dtype="bf16", qpos=None):
    """Per-Q-head column scores ``col [H, n]`` (fp32) before top-k.

    q: [H, n, d], k: [Hk, n, d] float32 arrays holding ``dtype`` values (post-RoPE).
    ``modal_rd/attention.py:148-170``."""
    q = np.asarray(q, dtype=np.float32)
    H, n, d = q.shape
    r = min(n_route, n)
    if qpos is None:
        qpos = route_query_positions(n, r, queries, sink, window)
    qpos = np.asarray(qpos, dtype=np.int64)
    return route_scores_at(q[:, qpos, :], k, qpos, scaling=scaling, sink=sink, window=window, pool=pool,
                           dtype=dtype)


def route_scores_at(q_sel, k, qpos, *, scaling, sink, window, pool="mean", dtype="bf16"):
    """``route_scores`` given only the routing query rows: q_sel [H, r, d] holds the rows at
    positions ``qpos`` (so a long prompt's full Q is not needed); k: [Hk, n, d]."""
    q_sel = np.asarray(q_sel, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    H, r, d = q_sel.shape
    hk, n, _ = k.shape
    g = H // hk
    qpos = np.asarray(qpos, dtype=np.int64)
    rnd = rounder(dtype)
    keypos = np.arange(n)
    qpos_g = np.tile(qpos, g)
    masked = keypos[None, :] > qpos_g[:, None]
    col = np.zeros((H, n), dtype=np.float32)
    for h in range(hk):
        qa = q_sel[h * g:(h + 1) * g].reshape(g * r, d)
        s = (qa.astype(np.float64) @ k[h].astype(np.float64).T).astype(np.float32)
        s = rnd(s) * np.float32(scaling)
        s[masked] = -np.inf
        m = s.max(-1, keepdims=True)
        e = np.exp(s - m)
        p = (e / e.sum(-1, keepdims=True, dtype=np.float32)).reshape(g, r, n)
        if pool == "max":
            pooled = p.max(1)
        elif pool == "mean":
            pooled = p.sum(1, dtype=np.float32) / np.float32(r)
        else:
            raise ValueError("route_pool must be mean or max")
        col[h * g:(h + 1) * g] = pooled
    col[:, :sink] = -1
    col[:, n - window:] = -1          # Python slice semantics, as in the reference
    return col


def topk_sorted(col, budget):
    """``col.topk(budget).indices.sort(-1).values.to(int32)``; ties resolved to lower index."""
    H, n = col.shape
    out = np.empty((H, budget), dtype=np.int32)
    for h in range(H):
        order = np.lexsort((np.arange(n), -col[h].astype(np.float64)))
        out[h] = np.sort(order[:budget])
    return out


def routes(q, k, *, scaling, sink, window, vertical, vertical_sqrt=0.0, n_route=64, pool="mean",
           queries="last", dtype="bf16", qpos=None, return_scores=False):
    """``RDAttention.routes`` (``modal_rd/attention.py:143-174``) -> int32 [H, budget]."""
    n = k.shape[-2]
    budget = min(vertical_budget(n, vertical, vertical_sqrt), max(0, n - sink - window))
    col = route_scores(q, k, scaling=scaling, sink=sink, window=window, n_route=n_route, pool=pool,
                       queries=queries, dtype=dtype, qpos=qpos)
    idx = topk_sorted(col, budget)
    return (idx, col) if return_scores else idx


def route_sets_match(got, want, col, tol=1e-6):
    """True when every head's route set equals the oracle's, except indices whose oracle score
    lies within ``tol`` of that head's ``budget``-th score (a tie at the selection boundary).

    Returns (ok, n_swapped, worst_gap)."""
    got = np.asarray(got)
    want = np.asarray(want)
    if got.shape != want.shape:
        return False, -1, float("inf")
    swapped, worst = 0, 0.0
    for h in range(want.shape[0]):
        a, b = set(got[h].tolist()), set(want[h].tolist())
        diff = a ^ b
        if not diff:
            continue
        if any(i < 0 or i >= col.shape[1] for i in diff):
            return False, len(diff), float("inf")
        kth = col[h, want[h]].min()
        gap = max(abs(float(col[h, i]) - float(kth)) for i in diff)
        worst = max(worst, gap)
        swapped += len(diff) // 2
        if gap > tol:
            return False, swapped, worst
    return True, swapped, worst


# ----------------------------------------------------------------------------- attention

def _kv_head(h, num_heads, kv_groups):
    return (h // num_heads) * (num_heads // kv_groups) + (h % num_heads) // kv_groups


def flash(q, k, v, indices, *, front=64, window=256, token_mask=None, num_heads=32, route_chunk=None,
          kv_groups=1, scale=1.0, rows=None, heads=None):
    """fp32 restatement of ``bigger_bird_flash_ref`` (``kernels/bigger_bird_flash_ref.py:10-52``).

    q [BH, T, D], k/v [BH/kv_groups, N, D] (float32 arrays), indices [BH, G, K] or [BH, K]
    (-1 = empty slot; out-of-range indices are treated as empty). ``rows`` selects query rows
    (local indices into T) and ``heads`` selects query heads; the result is
    ``[len(heads), len(rows), D]`` float32 (not rounded to the input dtype)."""
    q = np.asarray(q, dtype=np.float32)
    bh, t, d = q.shape
    n = np.shape(k)[1]
    offset = n - t
    if offset < 0:
        raise ValueError("Key sequence must be at least as long as query sequence")
    rows = np.arange(t) if rows is None else np.asarray(rows, dtype=np.int64)
    heads = np.arange(bh) if heads is None else np.asarray(heads, dtype=np.int64)
    return flash_at(q[heads][:, rows], rows + offset, k, v, indices, heads=heads, front=front, window=window,
                    token_mask=token_mask, num_heads=num_heads, route_chunk=route_chunk, kv_groups=kv_groups,
                    scale=scale)


def flash_at(q_rows, qs, k, v, indices, *, heads, front=64, window=256, token_mask=None, num_heads=32,
             route_chunk=None, kv_groups=1, scale=1.0):
    """``flash`` given only the query rows to compute: q_rows [len(heads), R, D] are the rows of
    query heads ``heads`` at absolute positions ``qs`` [R]; k/v [BH/kv_groups, N, D]; indices as in
    ``flash`` (indexed by query head). Returns [len(heads), R, D] float32."""
    q_rows = np.asarray(q_rows, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    n = k.shape[1]
    d = q_rows.shape[-1]
    idx_all = np.asarray(indices)
    if idx_all.ndim == 2:
        idx_all = idx_all[:, None, :]
    route_chunk = route_chunk or n
    front = min(front, n)
    qs = np.asarray(qs, dtype=np.int64)
    heads = np.asarray(heads, dtype=np.int64)
    kp = np.arange(n)
    causal = kp[None, :] <= qs[:, None]
    base = causal & ((kp[None, :] < front) | (kp[None, :] > qs[:, None] - window))
    beyond = kp[None, :] < qs[:, None] - window + 1
    group = qs // route_chunk
    out = np.zeros((len(heads), len(qs), d), dtype=np.float32)
    for oi, h in enumerate(heads):
        kv = _kv_head(int(h), num_heads, kv_groups)
        idx = idx_all[h].astype(np.int64)                         # [G, K]
        routed = np.zeros((idx.shape[0], n + 1), dtype=bool)
        valid = (idx >= 0) & (idx < n)
        gi, _ = np.nonzero(valid)
        routed[gi, idx[valid]] = True
        routed = routed[:, :n][group]                               # [R, N]
        mask = base | (routed & causal & (kp[None, :] >= front) & beyond)
        if token_mask is not None:
            b = int(h) // num_heads
            mask &= np.asarray(token_mask[b], dtype=bool)[None, :]
        s = (q_rows[oi] @ k[kv].T) * np.float32(scale)
        s = np.where(mask, s, -np.inf).astype(np.float32)
        m = s.max(-1, keepdims=True)
        m = np.where(np.isfinite(m), m, 0.0).astype(np.float32)
        e = np.exp(s - m)
        den = e.sum(-1, keepdims=True, dtype=np.float32)
        p = np.where(den > 0, e / np.where(den > 0, den, 1), 0).astype(np.float32)
        o = p @ v[kv]
        if token_mask is not None:
            o *= np.asarray(token_mask[b], dtype=np.float32)[qs][:, None]
        out[oi] = o
    return out


def sparse_prefill(q, k, v, *, scaling, sink, window, vertical, vertical_sqrt=0.0, n_route=64,
                   pool="mean", queries="last", exact_tail=0, vertical_scope=0, scope_chunk=4096,
                   dtype="bf16", rows=None, heads=None, idx=None, qpos=None):
    """``RDAttention.sparse_prefill`` (``modal_rd/attention.py:176-206``) on post-RoPE inputs.

    q [H, n, d], k/v [Hk, n, d]. Returns ``(out [len(heads), len(rows), d] fp32, idx [H, budget])``.
    ``idx`` may be given to reuse routes already computed."""
    H, n, d = np.shape(q)
    hk = np.shape(k)[0]
    g = H // hk
    if idx is None:
        idx = routes(q, k, scaling=scaling, sink=sink, window=window, vertical=vertical,
                     vertical_sqrt=vertical_sqrt, n_route=n_route, pool=pool, queries=queries,
                     dtype=dtype, qpos=qpos)
    if vertical_scope:
        chunk = scope_chunk
        groups = -(-n // chunk)
        starts = np.arange(groups) * chunk
        active = (starts + chunk > n - vertical_scope)[None, :, None]
        routed = np.where(active, idx[:, None, :], -1)
    else:
        chunk, routed = None, idx[:, None, :]
    rows = np.arange(n) if rows is None else np.asarray(rows, dtype=np.int64)
    heads = np.arange(H) if heads is None else np.asarray(heads, dtype=np.int64)
    out = flash(q, k, v, routed, front=sink, window=window, num_heads=H, route_chunk=chunk,
                kv_groups=g, scale=scaling, rows=rows, heads=heads)
    r = min(exact_tail, n)
    if r:
        tail_rows = rows >= n - r
        if tail_rows.any():
            none = -np.ones((H, 1, 1), dtype=np.int32)
            tail = flash(np.asarray(q)[:, n - r:], k, v, none, front=0, window=n, num_heads=H,
                         kv_groups=g, scale=scaling, rows=rows[tail_rows] - (n - r), heads=heads)
            out[:, tail_rows] = tail
    return out, idx


def sparse_prefill_at(q_rows, qs, k, v, idx, *, heads, scaling, sink, window, exact_tail=0,
                      vertical_scope=0, scope_chunk=4096):
    """``sparse_prefill`` output for the query rows ``q_rows [len(heads), R, d]`` at absolute
    positions ``qs`` with routes ``idx [H, budget]`` given: rows at or after ``n - exact_tail``
    take the exact causal tail, the others the main pass. Returns [len(heads), R, d] fp32."""
    H = np.shape(idx)[0]
    hk, n, _ = np.shape(k)
    g = H // hk
    qs = np.asarray(qs, dtype=np.int64)
    idx = np.asarray(idx)
    if vertical_scope:
        chunk = scope_chunk
        groups = -(-n // chunk)
        starts = np.arange(groups) * chunk
        active = (starts + chunk > n - vertical_scope)[None, :, None]
        routed = np.where(active, idx[:, None, :], -1)
    else:
        chunk, routed = None, idx[:, None, :]
    q_rows = np.asarray(q_rows, dtype=np.float32)
    out = flash_at(q_rows, qs, k, v, routed, heads=heads, front=sink, window=window, num_heads=H,
                   route_chunk=chunk, kv_groups=g, scale=scaling)
    r = min(exact_tail, n)
    tail = qs >= n - r
    if r and tail.any():
        none = -np.ones((H, 1, 1), dtype=np.int32)
        out[:, tail] = flash_at(q_rows[:, tail], qs[tail], k, v, none, heads=heads, front=0, window=n,
                                num_heads=H, kv_groups=g, scale=scaling)
    return out


# ----------------------------------------------------------------------------- KV eviction
def forward_pool(score, p, back=0):
    """``modal_rd/attention.py:70-75``: [H, n] -> [H, n], each key takes the max of the scores of
    keys j - p + 1 .. j + back (-inf beyond the ends; p is taken as at least 1)."""
    score = np.asarray(score, dtype=np.float32)
    p = max(int(p), 1)
    H, n = score.shape
    padded = np.full((H, n + p - 1 + back), -np.inf, dtype=np.float32)
    padded[:, p - 1:p - 1 + n] = score
    out = np.full((H, n), -np.inf, dtype=np.float32)
    for o in range(p + back):
        out = np.maximum(out, padded[:, o:o + n])
    return out


def evict_positions(idx, col, *, kv_heads, sink, window, evict_keep=0, evict_window=0, evict_pool=0,
                    evict_pool_back=0):
    """Kept positions ``[Hk, sink + keep + w]`` of ``RDAttention.evict`` (``modal_rd/attention.py:
    226-259``) and the priorities they were selected by.

    idx: [H, budget] routes; col: [H, n] fp32 per-query-head column scores (the routing scores, or
    the ``evict_obs`` exact-attention scores before the group max). The middle keys are the top-
    ``keep`` priorities sorted ascending; equal priorities at the cut go to the lower position."""
    idx = np.asarray(idx)
    col = np.asarray(col, dtype=np.float32)
    H, n = col.shape
    hk = kv_heads
    g = H // hk
    member = np.zeros((H, n), dtype=bool)
    for h in range(H):
        member[h, idx[h]] = True
    score = col.reshape(hk, g, n).max(1)
    if evict_pool > 1 or evict_pool_back:
        score = forward_pool(score, evict_pool, evict_pool_back)
    prio = member.reshape(hk, g, n).any(1).astype(np.float32) * np.float32(2) + score
    w = min(max(window, evict_window), n - sink)
    prio[:, :sink] = -np.inf
    prio[:, n - w:] = -np.inf
    budget = idx.shape[-1]
    extra = min(max(evict_keep, g * budget) if evict_keep else g * budget, n - sink - w)
    sel = topk_sorted(prio, extra).astype(np.int64)
    ar = np.arange(n, dtype=np.int64)
    pos = np.concatenate([np.tile(ar[:sink], (hk, 1)), sel, np.tile(ar[n - w:], (hk, 1))], axis=1)
    return pos, prio


# ----------------------------------------------------------------------------- decode
def decode(q, k, v, indices, *, front, window, scale, n=None):
    """``bigger_bird_decode`` (``kernels/bigger_bird_decode.py:67-107``) in fp32: q [H, D], k/v
    [Hkv, cap, D], indices [Hkv or H, R] -> [H, D]."""
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    idx = np.asarray(indices, dtype=np.int64).reshape(np.asarray(indices).shape[0], -1)
    H, D = q.shape
    hk, cap, _ = k.shape
    g = H // hk
    n = cap if n is None else int(n)
    pooled = idx.shape[0] == hk and hk != H
    out = np.zeros((H, D), dtype=np.float32)
    for h in range(H):
        kv = h // g
        row = idx[kv] if pooled else idx[h]
        pos = np.concatenate([np.arange(front), n - window + np.arange(window), row])
        pos = pos[(pos >= 0) & (pos < n)]
        s = (k[kv, pos].astype(np.float64) @ q[h].astype(np.float64)) * scale
        if s.size == 0:
            out[h] = np.nan
            continue
        p = np.exp(s - s.max())
        out[h] = ((p / p.sum()) @ v[kv, pos].astype(np.float64)).astype(np.float32)
    return out


def pooled_probs(q, k, *, front, window, scale, n=None):
    """``pooled_probs`` (``kernels/bigger_bird_route.py:80-106``): [Hkv, cap] fp32."""
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    H, D = q.shape
    hk, cap, _ = k.shape
    g = H // hk
    n = cap if n is None else int(n)
    out = np.full((hk, cap), -1.0, dtype=np.float32)
    for kv in range(hk):
        s = (q[kv * g:(kv + 1) * g].astype(np.float64) @ k[kv, :n].astype(np.float64).T) * scale
        e = np.exp(s - s.max(-1, keepdims=True))
        p = (e / e.sum(-1, keepdims=True)).mean(0)
        keep = np.zeros(cap, dtype=bool)
        keep[front:max(front, n - window)] = True
        out[kv, :n] = np.where(keep[:n], p, -1.0)
    return out
