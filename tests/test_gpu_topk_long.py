"""Top-k over rows longer than one thread-block cluster holds (> 16 x 49152 keys), on the GPU.

Such rows (1M-token prompts: the routing top-k of modal_rd/attention.py:173, the eviction top-k of
:253, decode routing over a 1M-key cache, kernels/bigger_bird_route.py:115) are selected in two
levels: per-segment top-k, then a top-k over the candidates. The selection must equal the
one-level rule exactly: the k largest values, ties at the cut going to the lowest positions, so
the tests compare against the oracle's top-k of the SAME values (no tolerance), including rows of
massive ties.
"""
import numpy as np
import pytest
import torch

from oracle import bigbird_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib_loaded():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from utmist_bigger_bird_b200 import _lib
    _lib.lib()


@pytest.mark.parametrize("n", [1 << 20, 1000003, 800000])
def test_routing_topk_long_rows_exact(n):
    """Routes of 8 query heads over n keys equal the oracle's top-512 of the GPU's own column
    scores, position for position."""
    from utmist_bigger_bird_b200 import _ops
    from utmist_bigger_bird_b200.attention import route_query_positions
    H, hk, d, sink, window, budget = 8, 2, 128, 64, 16384, 512
    g = torch.Generator(device=DEV).manual_seed(n % 1000)
    q = torch.randn(H, n, d, device=DEV, dtype=torch.bfloat16, generator=g)
    k = torch.randn(hk, n, d, device=DEV, dtype=torch.bfloat16, generator=g)
    qpos = route_query_positions(n, 64, "last", sink, window, DEV)
    col = torch.empty(H, n, device=DEV, dtype=torch.float32)
    idx = _ops.routes_(q, k, qpos, sink=sink, window=window, budget=budget, scaling=d ** -0.5, out_col=col)
    torch.cuda.synchronize()
    want = orc.topk_sorted(col.cpu().numpy(), budget)
    assert np.array_equal(idx.cpu().numpy(), want)


@pytest.mark.parametrize("n,keep,levels", [((1 << 20) + 4097, 2048, 50), (1 << 20, 4096, 3), (900000, 1000, 1),
                                           (1 << 20, 5000, 50)],
                         ids=["ragged_50_values", "keep4096_3_values", "all_equal", "keep5000_one_level"])
def test_evict_topk_long_rows_with_ties(n, keep, levels):
    """KV eviction with priorities of only `levels` distinct values (most keys tie at the cut):
    the kept middle keys are the oracle's, i.e. the lowest positions among the tied ones. keep >
    4096 takes the one-CTA-per-row kernel instead of the two-level path."""
    from utmist_bigger_bird_b200 import _ops
    H, hk, d, sink, window = 8, 2, 64, 64, 16384
    g = torch.Generator(device=DEV).manual_seed(keep)
    lv = torch.randint(0, levels, (hk, n), device=DEV, generator=g).float() / levels
    col = lv.repeat_interleave(H // hk, 0).contiguous()
    k = torch.randn(hk, n, d, device=DEV, dtype=torch.bfloat16, generator=g)
    v = torch.randn(hk, n, d, device=DEV, dtype=torch.bfloat16, generator=g)
    idx = torch.empty(H, 0, device=DEV, dtype=torch.int32)
    kk, vv, pos = _ops.kv_evict_(idx, col, k, v, sink=sink, window=window, keep=keep)
    torch.cuda.synchronize()
    want, _ = orc.evict_positions(np.zeros((H, 0), dtype=np.int32), col.cpu().numpy(), kv_heads=hk, sink=sink,
                                  window=window, evict_keep=keep)
    assert np.array_equal(pos.cpu().numpy(), want)
    gi = pos[:, :, None].expand(-1, -1, d)
    assert torch.equal(kk, k.gather(1, gi)) and torch.equal(vv, v.gather(1, gi))


def test_decode_route_topk_1m_cache_exact():
    """Decode routing over a 1M-key cache: the int64 routes equal the oracle's top-k of the GPU's
    own pooled probabilities."""
    from utmist_bigger_bird_b200 import bigger_bird_route, pooled_probs
    H, hk, d, cap, kr = 32, 8, 128, 1 << 20, 512
    g = torch.Generator(device=DEV).manual_seed(3)
    q = torch.randn(H, d, device=DEV, dtype=torch.bfloat16, generator=g)
    k = torch.randn(hk, cap, d, device=DEV, dtype=torch.bfloat16, generator=g)
    kw = dict(front=64, window=16384, scale=d ** -0.5)
    probs = pooled_probs(q, k, **kw)
    idx = bigger_bird_route(q, k, kr, **kw)
    torch.cuda.synchronize()
    want = orc.topk_sorted(probs.cpu().numpy(), kr)
    assert np.array_equal(idx.cpu().numpy(), want)
