"""Seeded inputs of the golden cases (shared by ``make_golden.py`` and the tests).

Inputs are drawn with torch's CPU generator, which is deterministic for a given torch build, so
only the reference's OUTPUTS are stored in the ``.npz`` files next to this module; each record
also stores a checksum of its inputs so that a generator change is caught instead of silently
comparing different data. Shapes follow the reference's own tests
(``tests/test_rd_attention_gqa.py``, ``tests/test_bigger_bird_flash.py``,
``tests/test_exact_memory_savers.py``).
"""
from __future__ import annotations

import numpy as np
import torch

RNG_TORCH = torch.__version__


def checksum(*tensors) -> np.ndarray:
    return np.array([float(t.double().abs().sum()) for t in tensors] +
                    [float(t.double().flatten()[:7].sum()) for t in tensors])


def rope_cases():
    """(name, dtype, n, q_heads, kv_heads, d, theta) -> q [1,hq,n,d], k [1,hk,n,d]."""
    out = []
    for name, dt, n, hq, hk, d, theta in (("bf16_d32", torch.bfloat16, 100, 8, 2, 32, 10000.0),
                                            ("f32_d32", torch.float32, 100, 8, 2, 32, 10000.0),
                                            ("f16_d64", torch.float16, 65, 4, 2, 64, 10000.0),
                                            ("bf16_d128", torch.bfloat16, 80, 4, 1, 128, 500000.0)):
        g = torch.Generator().manual_seed(11)
        q = torch.randn(1, hq, n, d, generator=g).to(dt)
        k = torch.randn(1, hk, n, d, generator=g).to(dt)
        out.append(dict(name=name, dtype=dt, n=n, d=d, theta=theta, q=q, k=k))
    return out


def flash_cases():
    """Kernel-level cases: (name, q, k, v, idx, kwargs, token_mask, rows). Values are bf16-representable
    so one set of inputs serves both the fp32 and the bf16 runs."""
    bf = lambda t: t.to(torch.bfloat16).float()  # noqa: E731
    cases = []
    g = torch.Generator().manual_seed(1)
    h, gq, n, d = 8, 4, 384, 32
    q, k, v = bf(torch.randn(h, n, d, generator=g)), bf(torch.randn(h // gq, n, d, generator=g)), bf(torch.randn(h // gq, n, d, generator=g))
    idx = torch.stack([torch.randperm(n - 160, generator=g)[:24] + 16 for _ in range(h)]).sort(-1).values.int()
    cases.append(("grouped", q, k, v, idx[:, None], dict(front=16, window=64, num_heads=h, kv_groups=gq, scale=0.2), None))
    g = torch.Generator().manual_seed(2)
    h, n, d, front, window = 4, 256, 32, 8, 48
    q, k, v = (bf(torch.randn(h, n, d, generator=g)) for _ in range(3))
    idx = torch.stack([torch.randperm(n - window - front, generator=g)[:20] + front for _ in range(h)]).sort(-1).values.int()
    cases.append(("union", q, k, v, idx[:, None], dict(front=front, window=window, num_heads=h), None))
    g = torch.Generator().manual_seed(3)
    h, gq, n, d, r = 8, 4, 300, 32, 37
    q, k, v = bf(torch.randn(h, n, d, generator=g)), bf(torch.randn(h // gq, n, d, generator=g)), bf(torch.randn(h // gq, n, d, generator=g))
    none = torch.full((h, 1, 1), -1, dtype=torch.int32)
    cases.append(("tail", q[:, n - r:].contiguous(), k, v, none, dict(front=0, window=n, num_heads=h, kv_groups=gq, scale=0.3), None))
    for name, n, d, window, front, chunk, masked in (("groups_n97", 97, 64, 17, 7, 128, False),
                                                      ("groups_mask_n257", 257, 128, 33, 0, 128, True),
                                                      ("groups_n513", 513, 128, 128, 0, 1024, False),
                                                      ("groups_c64_n300", 300, 64, 40, 5, 64, False)):
        g = torch.Generator().manual_seed(53 + n)
        q = bf(torch.randn(4, n, d, generator=g) / d ** 0.5)
        k, v = bf(torch.randn(4, n, d, generator=g)), bf(torch.randn(4, n, d, generator=g))
        G = (n + chunk - 1) // chunk
        kk = min(63, n)
        idx = torch.stack([torch.randperm(n, generator=g)[:kk] for _ in range(4 * G)]).reshape(4, G, kk).to(torch.int32)
        idx[0, 0, :5] = -1
        mask = None
        if masked:
            mask = torch.ones(2, n, dtype=torch.bool)
            mask[0, 15:23] = False
            mask[1, -17:] = False
        cases.append((name, q, k, v, idx, dict(front=front, window=window, route_chunk=chunk, num_heads=2), mask))
    g = torch.Generator().manual_seed(7)
    h, gq, n, t, d = 4, 2, 200, 70, 64
    q, k, v = bf(torch.randn(h, t, d, generator=g)), bf(torch.randn(h // gq, n, d, generator=g)), bf(torch.randn(h // gq, n, d, generator=g))
    idx = torch.stack([torch.randperm(n, generator=g)[:16] for _ in range(h)]).int()
    cases.append(("suffix", q, k, v, idx[:, None], dict(front=4, window=30, num_heads=h, kv_groups=gq, scale=0.125), None))
    out = []
    for name, q, k, v, idx, kw, mask in cases:
        t = q.shape[1]
        rows = torch.unique(torch.cat([torch.arange(0, t, max(1, t // 24)), torch.arange(max(0, t - 8), t)]))
        out.append(dict(name=name, q=q, k=k, v=v, idx=idx, kw=kw, token_mask=mask, rows=rows))
    return out


PREFILL_SHAPE = dict(H=8, hk=2, d=32, n=300)
PREFILL_BASE_KW = dict(sink=8, window=96, vertical=24, n_route=16, scope_chunk=64)


def prefill_inputs(dtype):
    s = PREFILL_SHAPE
    g = torch.Generator().manual_seed(4)
    q = torch.randn(1, s["H"], s["n"], s["d"], generator=g).to(dtype)
    k = torch.randn(1, s["hk"], s["n"], s["d"], generator=g).to(dtype)
    v = torch.randn(1, s["hk"], s["n"], s["d"], generator=g).to(dtype)
    n = s["n"]
    rows = torch.cat([torch.arange(0, n - 100, 23), torch.arange(n - 100, n, 9), torch.arange(n - 3, n)])
    return q, k, v, torch.unique(rows)


def prefill_configs():
    import itertools
    for pool, rq, tail, vs in itertools.product(["mean", "max"], ["last", "spread"], [0, 24, 96], [0, 128]):
        yield f"{pool}_{rq}_t{tail}_s{vs}", dict(PREFILL_BASE_KW, route_pool=pool, route_queries=rq,
                                                  exact_tail=tail, vertical_scope=vs)


EXTRA_ROUTE_CONFIGS = {
    "sqrt": dict(sink=8, window=96, vertical=24, vertical_sqrt=1.5, n_route=16),
    "bigbudget": dict(sink=8, window=96, vertical=500, n_route=16),
    "short": dict(sink=8, window=250, vertical=24, n_route=16),
    "nobudget": dict(sink=8, window=400, vertical=24, n_route=16),
}


# KV eviction after the prefill (RDAttention.evict, modal_rd/attention.py:226-259): the default
# policy and each tuning knob of the reference's eviction tests, on the PREFILL_SHAPE inputs.
EVICT_BASE_KW = dict(sink=8, window=96, vertical=24, n_route=16)
EVICT_CONFIGS = {
    "default": {},
    "keep160": dict(evict_keep=160),
    "window160": dict(evict_window=160),
    "pool8": dict(evict_pool=8),
    "back8": dict(evict_pool_back=8),
    "obs24": dict(evict_obs=24),
    "obs24max": dict(evict_obs=24, evict_obs_max=True),
    "full1": dict(evict_full_layers=1),
    "all": dict(evict_keep=160, evict_window=160, evict_pool=8, evict_obs=24, evict_pool_back=4),
}


# Decode (one new token): pinned through the reference's own functions that run on the CPU. A
# one-query decode over front | window | routed equals bigger_bird_flash_ref for the last query
# row with the same routes; in fp32, pooled_probs equals the mean over a KV head's query heads of
# RDAttention.routes' column scores with n_route=1 (the same masks).
DECODE_SHAPE = dict(H=8, hk=2, d=32, n=300, front=8, window=64, R=24)


def decode_inputs():
    s = DECODE_SHAPE
    g = torch.Generator().manual_seed(11)
    q = torch.randn(1, s["H"], s["n"], s["d"], generator=g)
    k = torch.randn(1, s["hk"], s["n"], s["d"], generator=g)
    v = torch.randn(1, s["hk"], s["n"], s["d"], generator=g)
    lo, hi = s["front"], s["n"] - s["window"]
    pooled = torch.stack([torch.randperm(hi - lo, generator=g)[:s["R"]] + lo for _ in range(s["hk"])])
    pooled = pooled.sort(-1).values.to(torch.int32)
    return q, k, v, pooled


def config1_rows(n):
    return torch.cat([torch.linspace(0, n - 300, 12).long(), torch.arange(n - 258, n - 254),
                      torch.arange(n - 4, n)])
