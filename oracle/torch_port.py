"""The reference's sparse-prefill path restated with torch CPU ops in fp32 on all host threads: the
CPU leg of ``bench.py`` (its ``cpu_baseline`` and ``--impl reference`` arm).

Test infrastructure, like ``bigbird_oracle``: only ``bench.py``'s CPU legs and ``tests/`` use it, and
its results equal the numpy restatement's (``tests/test_torch_port_cpu.py``). It follows the same
reference lines as ``bigbird_oracle`` (cited per function) in the reference's own CPU contract, fp32
(``modal_rd/attention.py:41-45`` sends CPU tensors to ``bigger_bird_flash_ref``), with batched matrix
products and one softmax per row, so its speed on a host is that of the reference's own CPU path
(``oracle/time_reference_cpu.py`` measures both on one sample).
"""
from __future__ import annotations

import torch


def rope(x, cos, sin):
    """``x * cos + rotate_half(x) * sin`` (``modal_rd/attention.py:51-60``); x [..., T, D], cos/sin [T, D]."""
    half = x.shape[-1] // 2
    return x * cos + torch.cat((-x[..., half:], x[..., :half]), dim=-1) * sin


def route_scores(q_sel, k, qpos, *, scaling, sink, window, pool="mean"):
    """Column scores ``col [H, n]`` from the routing rows ``q_sel [H, r, d]`` at positions ``qpos``
    (``modal_rd/attention.py:148-170``): per KV head, scores of its query heads' rows against every
    key, causal at the routing rows, softmax per row, pooled over the rows; sink and window columns -1."""
    H, r, d = q_sel.shape
    hk, n, _ = k.shape
    g = H // hk
    blocked = torch.arange(n)[None, :] > qpos.repeat(g)[:, None]
    col = torch.empty(H, n)
    for h in range(hk):
        s = (q_sel[h * g:(h + 1) * g].reshape(g * r, d) @ k[h].T) * scaling
        s.masked_fill_(blocked, float("-inf"))
        p = torch.softmax(s, dim=-1).view(g, r, n)
        col[h * g:(h + 1) * g] = p.amax(1) if pool == "max" else p.sum(1) / r
    col[:, :sink] = -1
    col[:, n - window:] = -1
    return col


def routes(q, k, *, scaling, sink, window, vertical, n_route=64):
    """``RDAttention.routes`` with the last ``n_route`` queries (``modal_rd/attention.py:143-174``):
    q [H, n, d], k [Hk, n, d] -> int64 [H, budget], positions ascending."""
    n = k.shape[1]
    r = min(n_route, n)
    budget = min(vertical, max(0, n - sink - window))
    qpos = torch.arange(n - r, n)
    col = route_scores(q[:, qpos], k, qpos, scaling=scaling, sink=sink, window=window)
    return col.topk(budget, dim=-1).indices.sort(dim=-1).values


def attend_rows(q_rows, qs, k, v, idx, *, heads, kv_groups, scaling, sink, window, exact_tail):
    """``sparse_prefill`` output of the query rows ``q_rows [len(heads), R, d]`` at absolute positions
    ``qs`` (``modal_rd/attention.py:176-206``, ``kernels/bigger_bird_flash_ref.py:10-52``): rows before
    ``n - exact_tail`` attend the sink, their causal window and their head's routed keys in
    [sink, q - window]; later rows attend every causal key. Returns [len(heads), R, d] fp32."""
    n = k.shape[1]
    kp = torch.arange(n)
    causal = kp[None, :] <= qs[:, None]
    local = causal & ((kp[None, :] < sink) | (kp[None, :] > qs[:, None] - window))
    tail = (qs >= n - exact_tail)[:, None]
    out = torch.empty(q_rows.shape)
    for i, h in enumerate(heads):
        kv = int(h) // kv_groups
        routed = torch.zeros(n, dtype=torch.bool)
        ids = idx[int(h)]
        routed[ids[(ids >= 0) & (ids < n)]] = True
        far = routed[None, :] & (kp[None, :] >= sink) & (kp[None, :] <= qs[:, None] - window)
        allowed = torch.where(tail, causal, local | far)
        s = (q_rows[i] @ k[kv].T) * scaling
        s.masked_fill_(~allowed, float("-inf"))
        out[i] = torch.softmax(s, dim=-1) @ v[kv]
    return out
