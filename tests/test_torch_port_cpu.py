"""The torch CPU restatement that bench.py times as its CPU leg (``oracle/torch_port.py``) against the
numpy restatement pinned to the reference's golden vectors (``oracle/bigbird_oracle.py``), fp32."""
import numpy as np
import pytest
import torch

from oracle import bigbird_oracle as orc
from oracle import torch_port as tp


@pytest.mark.parametrize("pool", ["mean", "max"])
def test_torch_port_matches_oracle(pool):
    g = torch.Generator().manual_seed(21)
    H, hk, n, d = 8, 2, 2304, 64
    sink, window, vertical, n_route, tail, scaling = 16, 256, 96, 32, 64, 64 ** -0.5
    q = torch.randn(H, n, d, generator=g)
    k = torch.randn(hk, n, d, generator=g)
    v = torch.randn(hk, n, d, generator=g)
    pos = torch.arange(n, dtype=torch.float32)[:, None]
    freq = 10000.0 ** (-torch.arange(0, d, 2, dtype=torch.float32) / d)
    ang = torch.cat([pos * freq, pos * freq], dim=-1)
    cos, sin = ang.cos(), ang.sin()

    qr, kr = tp.rope(q, cos, sin), tp.rope(k, cos, sin)
    np.testing.assert_allclose(qr.numpy(), orc.rope(q.numpy(), cos.numpy(), sin.numpy(), "f32"), atol=1e-6)
    np.testing.assert_allclose(kr.numpy(), orc.rope(k.numpy(), cos.numpy(), sin.numpy(), "f32"), atol=1e-6)
    qn, kn = qr.numpy(), kr.numpy()

    qpos = torch.arange(n - n_route, n)
    col_t = tp.route_scores(qr[:, qpos], kr, qpos, scaling=scaling, sink=sink, window=window, pool=pool)
    col_o = orc.route_scores(qn, kn, scaling=scaling, sink=sink, window=window, n_route=n_route, pool=pool,
                             dtype="f32")
    np.testing.assert_allclose(col_t.numpy(), col_o, rtol=1e-4, atol=1e-7)
    if pool == "mean":
        idx_t = tp.routes(qr, kr, scaling=scaling, sink=sink, window=window, vertical=vertical, n_route=n_route)
        idx_o = orc.routes(qn, kn, scaling=scaling, sink=sink, window=window, vertical=vertical, n_route=n_route,
                           dtype="f32")
        ok, swapped, gap = orc.route_sets_match(idx_t.numpy(), idx_o, col_o)
        assert ok, (swapped, gap)

        rows = np.unique(np.concatenate([np.arange(0, n, 97), np.arange(n - tail - 3, n - tail + 3), [n - 1]]))
        heads = np.array([0, 3, 5])
        got = tp.attend_rows(qr[heads][:, rows], torch.from_numpy(rows), kr, v, torch.from_numpy(idx_o).long(),
                             heads=heads, kv_groups=H // hk, scaling=scaling, sink=sink, window=window,
                             exact_tail=tail)
        want = orc.sparse_prefill_at(qn[heads][:, rows], rows, kn, v.numpy(), idx_o, heads=heads, scaling=scaling,
                                     sink=sink, window=window, exact_tail=tail)
        np.testing.assert_allclose(got.numpy(), want, atol=2e-5)
