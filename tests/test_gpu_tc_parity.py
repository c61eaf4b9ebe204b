"""The head_dim-128 path that ships, against the numpy oracle (needs an sm_100a GPU).

With head_dim 128 and no token mask every attention call runs on the tcgen05/TMEM kernels
(``flash_tc_pair_kernel`` for even GQA groups, ``flash_tc_kernel`` for odd ones), and routing
with 4 query heads x 64 routing rows runs on the tcgen05 score passes (``rt_stats_kernel``,
``rt_col_kernel``) and the cluster top-k. The d = 32 product in ``test_gpu_parity.py`` exercises
the mma.sync kernels instead, so the reference's router-variant product
(``tests/test_rd_attention_gqa.py:105-128``) is repeated here at Llama shapes (32 query / 8 KV
heads), with ``vertical_scope`` producing several route groups, in bf16 and fp16; then config 3's
window-4096 arm at 128K, a 512K layer, a 1M layer whose element offsets pass 2^32, and odd GQA
groups.

Tolerances (north star): attention within max-abs 2e-2 / mean-abs 2e-3 of the fp32 oracle computed
with the SAME routes; routes identical except keys whose oracle scores lie within 1e-6 of the
budget-th score.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import bigbird_oracle as orc

pytestmark = pytest.mark.gpu

ATOL_MAX, ATOL_MEAN, TIE_TOL = 2e-2, 2e-3, 1e-6
DEV = "cuda"
TAG = {torch.bfloat16: "bf16", torch.float16: "f16"}


def np32(t):
    return t.detach().float().cpu().numpy()


def close(got, want, what=""):
    got = np.asarray(got, dtype=np.float32)
    err = np.abs(got - np.asarray(want, dtype=np.float32))
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    assert err.max() <= ATOL_MAX and err.mean() <= ATOL_MEAN, f"{what}: max {err.max():.4g} mean {err.mean():.4g}"


def base(h, hk, d):
    return SimpleNamespace(config=SimpleNamespace(num_attention_heads=h, num_key_value_heads=hk),
                           layer_idx=0, head_dim=d, scaling=d ** -0.5,
                           q_proj=None, k_proj=None, v_proj=None, o_proj=None)


@pytest.fixture(scope="module", autouse=True)
def _lib_loaded():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from utmist_bigger_bird_b200 import _lib
    _lib.lib()


# ----------------------------------------------------------------------------- router product at d = 128

TC_N, TC_H, TC_HK, TC_D = 2300, 32, 8, 128      # ragged n: the last query and key tiles are partial
TC_KW = dict(sink=64, window=512, vertical=256, n_route=64, scope_chunk=256)


def _tc_inputs(dtype):
    """Post-RoPE-like Gaussian q/k/v [1, heads, n, 128] with 6 salient keys per KV head (2x the
    mean of the group's last 64 query rows), so the routes hold clear winners and near-ties."""
    g = torch.Generator().manual_seed(41)
    q = torch.randn(1, TC_H, TC_N, TC_D, generator=g)
    k = torch.randn(1, TC_HK, TC_N, TC_D, generator=g)
    v = torch.randn(1, TC_HK, TC_N, TC_D, generator=g)
    gq = TC_H // TC_HK
    for h in range(TC_HK):
        pos = torch.randint(TC_KW["sink"], TC_N - TC_KW["window"], (6,), generator=g)
        k[0, h, pos] = 2.0 * q[0, h * gq:(h + 1) * gq, -64:].reshape(-1, TC_D).mean(0)
    return q.to(dtype), k.to(dtype), v.to(dtype)


def _tc_rows():
    n, w, c = TC_N, TC_KW["window"], TC_KW["scope_chunk"]
    edges = [w - 1, w, w + 1, n - 257, n - 256, n - 255, n - 101, n - 100, n - 99]
    groups = [x for g in range(1, n // c + 1) for x in (g * c - 1, g * c)]
    return np.unique(np.clip(np.concatenate([np.arange(0, n, 41), edges, groups, np.arange(n - 3, n)]), 0, n - 1))


def tc_configs():
    import itertools
    for pool, rq, tail, vs in itertools.product(["mean", "max"], ["last", "spread"], [0, 100, 256], [0, 1024]):
        yield f"{pool}_{rq}_t{tail}_s{vs}", dict(TC_KW, route_pool=pool, route_queries=rq, exact_tail=tail,
                                                 vertical_scope=vs)
    yield "f16_mean_last_t256_s0", dict(TC_KW, exact_tail=256, dtype=torch.float16)
    yield "f16_max_spread_t100_s1024", dict(TC_KW, route_pool="max", route_queries="spread", exact_tail=100,
                                            vertical_scope=1024, dtype=torch.float16)
    yield "f16_mean_spread_t0_s1024", dict(TC_KW, route_queries="spread", vertical_scope=1024, dtype=torch.float16)
    yield "sqrt_budget", dict(TC_KW, vertical_sqrt=1.5, exact_tail=256)


@pytest.mark.parametrize("name,kw", list(tc_configs()), ids=lambda x: x if isinstance(x, str) else "")
def test_tc_prefill_matches_oracle(name, kw):
    from utmist_bigger_bird_b200 import RDAttention
    kw = dict(kw)
    dtype = kw.pop("dtype", torch.bfloat16)
    q, k, v = _tc_inputs(dtype)
    attn = RDAttention(base(TC_H, TC_HK, TC_D), **kw)
    with torch.inference_mode():
        out = attn.sparse_prefill(q.to(DEV), k.to(DEV), v.to(DEV))
    torch.cuda.synchronize()
    idx = attn.last_routes.cpu().numpy()
    qn, kn, vn = np32(q[0]), np32(k[0]), np32(v[0])
    want_idx, col = orc.routes(qn, kn, scaling=TC_D ** -0.5, pool=kw.get("route_pool", "mean"),
                               queries=kw.get("route_queries", "last"), dtype=TAG[dtype], return_scores=True,
                               sink=kw["sink"], window=kw["window"], vertical=kw["vertical"],
                               vertical_sqrt=kw.get("vertical_sqrt", 0.0), n_route=kw["n_route"])
    ok, swapped, gap = orc.route_sets_match(idx, want_idx, col, TIE_TOL)
    assert ok, (name, swapped, gap)
    assert (np.diff(idx, axis=-1) > 0).all(), "routes must be sorted and unique"
    rows = _tc_rows()
    want = orc.sparse_prefill_at(qn[:, rows], rows, kn, vn, idx, heads=np.arange(TC_H), scaling=TC_D ** -0.5,
                                 sink=kw["sink"], window=kw["window"], exact_tail=kw.get("exact_tail", 0),
                                 vertical_scope=kw.get("vertical_scope", 0), scope_chunk=kw["scope_chunk"])
    close(np32(out[0][:, rows]), want, name)


# ----------------------------------------------------------------------------- kernel calls with route groups

@pytest.mark.parametrize("h,gq,dtype", [(8, 4, torch.bfloat16), (8, 2, torch.float16), (6, 3, torch.bfloat16),
                                        (4, 1, torch.float16)], ids=["pair_g4", "pair_g2_f16", "single_g3",
                                                                     "single_mha_f16"])
def test_tc_flash_route_groups(h, gq, dtype):
    """bigger_bird_flash at head_dim 128 with 6 route groups of 150 slots (two routed tiles, the
    second partial), empty (-1) slots, routed keys in the sink, inside the window and after the
    query, and 1300 suffix queries over 1500 keys: even groups take the pair kernel, odd groups
    and MHA the single-head kernel."""
    from utmist_bigger_bird_b200 import bigger_bird_flash
    g = torch.Generator().manual_seed(100 + h * gq)
    n, t, d, front, window, chunk, K = 1500, 1300, 128, 40, 200, 256, 150
    q = (torch.randn(h, t, d, generator=g) * 0.4).to(dtype)
    k = torch.randn(h // gq, n, d, generator=g).to(dtype)
    v = torch.randn(h // gq, n, d, generator=g).to(dtype)
    G = -(-n // chunk)
    idx = torch.stack([torch.randperm(n, generator=g)[:K] for _ in range(h * G)]).reshape(h, G, K).int()
    idx[:, :, 7:19] = -1
    idx[0, 2, :4] = torch.tensor([0, 5, 39, 1499], dtype=torch.int32)
    out = bigger_bird_flash(q.to(DEV), k.to(DEV), v.to(DEV), idx.to(DEV), front=front, window=window,
                            num_heads=h, route_chunk=chunk, kv_groups=gq, scale=d ** -0.5)
    rows = np.unique(np.concatenate([np.arange(0, t, 29), np.arange(t - 5, t), [255 - (n - t), 256 - (n - t)]]))
    rows = rows[(rows >= 0) & (rows < t)]
    want = orc.flash(np32(q), np32(k), np32(v), idx.numpy(), front=front, window=window, num_heads=h,
                     route_chunk=chunk, kv_groups=gq, scale=d ** -0.5, rows=rows)
    close(np32(out)[:, rows], want, f"h{h}_g{gq}")


# ----------------------------------------------------------------------------- long layers

def _layer_on_gpu(n, seed, planted, window, heads=32, kv_heads=8, d=128, q_pad_heads=0):
    """Gaussian (x0.5) post-RoPE q [1, H, n, d], k/v [1, Hk, n, d] generated on the device, stored
    as [n, H + q_pad_heads, d] / [n, Hk, d] like a model's projection outputs, with ``planted``
    salient keys per KV head at positions in [64, n - window) (3x the mean of the group's last 64
    query rows)."""
    gen = torch.Generator(device=DEV).manual_seed(seed)
    qs = torch.randn(n, heads + q_pad_heads, d, generator=gen, device=DEV, dtype=torch.bfloat16).mul_(0.5)
    ks = torch.randn(n, kv_heads, d, generator=gen, device=DEV, dtype=torch.bfloat16).mul_(0.5)
    vs = torch.randn(n, kv_heads, d, generator=gen, device=DEV, dtype=torch.bfloat16).mul_(0.5)
    q = qs[:, :heads].permute(1, 0, 2)[None]
    k, v = ks.permute(1, 0, 2)[None], vs.permute(1, 0, 2)[None]
    g = heads // kv_heads
    cpu = torch.Generator().manual_seed(seed)
    for h in range(kv_heads):
        pos = torch.randint(64, n - window, (planted,), generator=cpu).to(DEV)
        target = 3.0 * q[0, h * g:(h + 1) * g, -64:].float().reshape(-1, d).mean(0)
        k[0, h, pos] = target.to(torch.bfloat16)
    return q, k, v


def _long_parity(q, k, v, attn_kw, kv_check, rows, heads_per_kv=(0, 3)):
    """Runs RDAttention.sparse_prefill, then checks the routes of the KV heads ``kv_check`` (every
    query head of the group) and, for query heads ``heads_per_kv`` of each such group, the output
    rows ``rows`` against the oracle computed from that KV head alone."""
    from utmist_bigger_bird_b200 import RDAttention
    H, n, d = q.shape[1], q.shape[2], q.shape[3]
    hk = k.shape[1]
    g = H // hk
    attn = RDAttention(base(H, hk, d), **attn_kw)
    with torch.inference_mode():
        out = attn.sparse_prefill(q, k, v)
    torch.cuda.synchronize()
    idx = attn.last_routes.cpu().numpy()
    assert (np.diff(idx, axis=-1) > 0).all(), "routes must be sorted and unique"
    r = attn_kw["n_route"]
    qpos = np.arange(n - r, n)
    budget = idx.shape[1]
    rows_t = torch.as_tensor(rows, device=DEV)
    q_rows, out_rows = np32(q[0].index_select(1, rows_t)), np32(out[0].index_select(1, rows_t))
    for kvh in kv_check:
        hs = np.arange(kvh * g, (kvh + 1) * g)
        kn = np32(k[0, kvh])[None]
        col = orc.route_scores_at(np32(q[0, kvh * g:(kvh + 1) * g, n - r:]), kn, qpos, scaling=d ** -0.5,
                                  sink=attn_kw["sink"], window=attn_kw["window"], dtype="bf16")
        want_idx = orc.topk_sorted(col, budget)
        ok, swapped, gap = orc.route_sets_match(idx[hs], want_idx, col, TIE_TOL)
        assert ok, (kvh, swapped, gap)
        sel = hs[list(heads_per_kv)]
        want = orc.sparse_prefill_at(q_rows[sel], rows, kn, np32(v[0, kvh])[None], idx[sel],
                                     heads=np.arange(len(sel)), scaling=d ** -0.5, sink=attn_kw["sink"],
                                     window=attn_kw["window"], exact_tail=attn_kw["exact_tail"])
        close(out_rows[sel], want, f"kv{kvh}")
        del kn, col
    return out, idx


def _long_rows(n, window, tail):
    return np.unique(np.concatenate([[0, 63, 64, 127, 128, window - 1, window, window + 1],
                                     np.linspace(window + 2, n - tail - 2, 9).astype(np.int64),
                                     [n - tail - 1, n - tail, n - 2, n - 1]]))


def test_config3_window4096_128k():
    """Config 3's window-4096 arm at 128K (the arm where routed and edge tiles are the largest
    share of the pair kernel's work): routes of every head and sampled rows of two heads per KV
    head."""
    n, w = 131072, 4096
    kw = dict(sink=64, window=w, vertical=512, n_route=64, exact_tail=256)
    q, k, v = _layer_on_gpu(n, seed=31, planted=32, window=w)
    _long_parity(q, k, v, kw, kv_check=range(8), rows=_long_rows(n, w, 256))


def test_layer_512k():
    """Config 3's longest layer (512K, window 16384): routes of every head, sampled rows."""
    n, w = 524288, 16384
    kw = dict(sink=64, window=w, vertical=512, n_route=64, exact_tail=256)
    q, k, v = _layer_on_gpu(n, seed=32, planted=32, window=w)
    _long_parity(q, k, v, kw, kv_check=range(8), rows=_long_rows(n, w, 256))


def test_layer_1m_offsets_beyond_2_32():
    """Config 5's layer (1,048,576 tokens, 64/16384/512/256) with q stored as [n, 33, 128] (one pad
    head), so the last rows' element offsets pass 2^32 (and their byte offsets 2^33): routes of
    KV heads 0 and 7 and sampled rows of query heads 0, 3, 28, 31."""
    n, w = 1 << 20, 16384
    kw = dict(sink=64, window=w, vertical=512, n_route=64, exact_tail=256)
    q, k, v = _layer_on_gpu(n, seed=33, planted=64, window=w, q_pad_heads=1)
    assert (n - 1) * q.stride(2) + 31 * q.stride(1) > 1 << 32
    out, _ = _long_parity(q, k, v, kw, kv_check=(0, 7), rows=_long_rows(n, w, 256))
    assert torch.isfinite(out[0, :, -4:]).all()
