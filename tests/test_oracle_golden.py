"""Pin the numpy oracle to vectors produced by the reference itself (CPU only).

The golden files come from ``tests/golden/make_golden.py``, which runs the reference's
``rope_inplace``, ``RDAttention.routes`` / ``sparse_prefill`` and ``bigger_bird_flash_ref``.
"""
import numpy as np
import pytest
import torch

import cases
from oracle import bigbird_oracle as orc
from utmist_bigger_bird_b200.workload import CONFIGS, make_layer


def np32(t):
    return t.detach().float().cpu().numpy()


def dt_tag(dtype):
    return {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[dtype]


@pytest.mark.parametrize("case", cases.rope_cases(), ids=lambda c: c["name"])
def test_oracle_rope_bit_identical(golden, case):
    g = golden("rope")[case["name"]]
    np.testing.assert_allclose(g["check"], cases.checksum(case["q"], case["k"]), rtol=0, atol=0)
    tag = dt_tag(case["dtype"])
    cos, sin = g["cos"][0], g["sin"][0]
    q_out = orc.rope(np32(case["q"]), cos, sin, tag)
    k_out = orc.rope(np32(case["k"]), cos, sin, tag)
    assert np.array_equal(q_out, g["q_out"])
    assert np.array_equal(k_out, g["k_out"])


@pytest.mark.parametrize("case", cases.flash_cases(), ids=lambda c: c["name"])
def test_oracle_flash_matches_reference(golden, case):
    g = golden("flash")[case["name"]]
    np.testing.assert_allclose(g["check"], cases.checksum(case["q"], case["k"], case["v"]), rtol=0, atol=0)
    kw = dict(case["kw"])
    mask = None if case["token_mask"] is None else case["token_mask"].numpy()
    got = orc.flash(np32(case["q"]), np32(case["k"]), np32(case["v"]), case["idx"].numpy(),
                    token_mask=mask, rows=case["rows"].numpy(), **kw)
    np.testing.assert_allclose(got, g["out_f32"], atol=2e-5, rtol=1e-5)
    # The reference's bf16 run is the fp32 result rounded once to bf16.
    np.testing.assert_allclose(orc.bf16_round(got), g["out_bf16"], atol=1e-6, rtol=2 ** -7)


def test_linspace_restatement_matches_torch():
    for start, end, steps in ((104, 299, 16), (2112, 8191, 64), (16448, 131071, 64), (5, 5, 1),
                              (100, 37, 9), (3, 1000003, 63), (0, 65535, 64)):
        want = torch.linspace(start, end, steps).long().numpy()
        got = orc.route_query_positions(end + 1, steps, "spread", start, 0)
        assert np.array_equal(got, want), (start, end, steps)


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_oracle_routes_and_prefill_match_reference(golden, tag):
    g = golden("prefill")
    s = cases.PREFILL_SHAPE
    dtype = torch.float32 if tag == "f32" else torch.bfloat16
    q, k, v, rows = cases.prefill_inputs(dtype)
    np.testing.assert_allclose(g[f"inputs_{tag}"]["check"], cases.checksum(q, k, v), rtol=0, atol=0)
    q, k, v = np32(q[0]), np32(k[0]), np32(v[0])
    scaling = s["d"] ** -0.5
    for name, kw in cases.prefill_configs():
        rec = g[f"{tag}_{name}"]
        kw = dict(kw)
        pool, queries = kw.pop("route_pool"), kw.pop("route_queries")
        out, idx = orc.sparse_prefill(q, k, v, scaling=scaling, pool=pool, queries=queries, dtype=tag,
                                      rows=rows.numpy(), **kw)
        if tag == "f32":
            assert np.array_equal(idx, rec["idx"]), name          # the reference's CPU contract
        else:
            col = orc.route_scores(q, k, scaling=scaling, sink=kw["sink"], window=kw["window"],
                                   n_route=kw["n_route"], pool=pool, queries=queries, dtype=tag)
            ok, swapped, gap = orc.route_sets_match(idx, rec["idx"], col)
            assert ok, (name, swapped, gap)
        np.testing.assert_allclose(out, rec["out"], atol=2e-5 if tag == "f32" else 1e-2,
                                   rtol=1e-5 if tag == "f32" else 1e-2, err_msg=name)
        if "col" in rec:
            col = orc.route_scores(q, k, scaling=scaling, sink=kw["sink"], window=kw["window"],
                                   n_route=kw["n_route"], pool=pool, queries=queries, dtype=tag)
            np.testing.assert_allclose(col, rec["col"], rtol=2e-5, atol=1e-9, err_msg=name)


@pytest.mark.parametrize("tag", ["f32", "bf16"])
@pytest.mark.parametrize("name", list(cases.EXTRA_ROUTE_CONFIGS))
def test_oracle_route_budget_edges(golden, tag, name):
    rec = golden("prefill")[f"{tag}_{name}"]
    dtype = torch.float32 if tag == "f32" else torch.bfloat16
    q, k, _, _ = cases.prefill_inputs(dtype)
    kw = dict(cases.EXTRA_ROUTE_CONFIGS[name])
    d = cases.PREFILL_SHAPE["d"]
    idx, col = orc.routes(np32(q[0]), np32(k[0]), scaling=d ** -0.5, dtype=tag, return_scores=True, **kw)
    assert idx.shape == rec["idx"].shape
    np.testing.assert_allclose(col, rec["col"], rtol=2e-5, atol=1e-9)
    ok, swapped, gap = orc.route_sets_match(idx, rec["idx"], col)
    assert ok, (swapped, gap)


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_oracle_config1_matches_reference(golden, tag):
    """n=8192, 32/8 heads, d=128, sink 64, window 2048, vertical 128, tail 256."""
    rec = golden("config1")[tag]
    cfg = CONFIGS["config1"]
    q, k, v, cos, sin, planted = make_layer(cfg)
    np.testing.assert_allclose(rec["check"], cases.checksum(q, k, v), rtol=0, atol=0)
    assert np.array_equal(planted.numpy(), rec["planted"])
    dtype = torch.float32 if tag == "f32" else torch.bfloat16
    q, k, v = np32(q[0].to(dtype)), np32(k[0].to(dtype)), np32(v[0].to(dtype))
    c, s_ = np32(cos[0].to(dtype)), np32(sin[0].to(dtype))
    q = orc.rope(q, c, s_, tag)
    k = orc.rope(k, c, s_, tag)
    n = cfg.n
    assert np.array_equal(q[:, n - 2:], rec["q_rot_tail"]) and np.array_equal(k[:, :2], rec["k_rot_head"])
    rows = cases.config1_rows(n).numpy()
    out, idx = orc.sparse_prefill(q, k, v, scaling=cfg.scaling, sink=cfg.sink, window=cfg.window,
                                  vertical=cfg.vertical, n_route=cfg.n_route, exact_tail=cfg.exact_tail,
                                  dtype=tag, rows=rows)
    col = orc.route_scores(q, k, scaling=cfg.scaling, sink=cfg.sink, window=cfg.window,
                           n_route=cfg.n_route, dtype=tag)
    ok, swapped, gap = orc.route_sets_match(idx, rec["idx"], col)
    assert ok, (swapped, gap)
    np.testing.assert_allclose(out, rec["out"], atol=5e-5 if tag == "f32" else 1e-2, rtol=1e-4)


def kept_match(got, want, prio, sink, w, tol=0.0):
    """Same shape; per KV head the kept sets agree except positions whose priority ties (within
    ``tol``) with the lowest kept middle priority (torch.topk's order among ties is unspecified)."""
    if got.shape != want.shape:
        return False
    for h in range(got.shape[0]):
        diff = set(got[h].tolist()) ^ set(want[h].tolist())
        if not diff:
            continue
        cut = prio[h, got[h][sink:got.shape[1] - w]].min()
        if any(abs(float(prio[h, i]) - float(cut)) > tol for i in diff):
            return False
    return True


@pytest.mark.parametrize("tag", ["f32", "bf16"])
@pytest.mark.parametrize("name", list(cases.EVICT_CONFIGS))
def test_oracle_evict_matches_reference(golden, tag, name):
    """RDAttention.evict (modal_rd/attention.py:226-259) through the oracle: kept positions equal
    the reference's up to ties at the cut; the evict_obs scores match evict_scores."""
    g = golden("evict")[f"{tag}_{name}"]
    kw, bkw, s = cases.EVICT_CONFIGS[name], cases.EVICT_BASE_KW, cases.PREFILL_SHAPE
    n, hk, H, d = s["n"], s["hk"], s["H"], s["d"]
    if kw.get("evict_full_layers"):
        assert np.array_equal(g["kept"], np.tile(np.arange(n), (hk, 1)))
        return
    col, tol = g["col"], 0.0
    if kw.get("evict_obs"):
        dtype = torch.float32 if tag == "f32" else torch.bfloat16
        q, k, _, _ = cases.prefill_inputs(dtype)
        col = orc.route_scores(np32(q[0]), np32(k[0]), scaling=d ** -0.5, sink=0, window=0,
                               n_route=kw["evict_obs"], pool="max" if kw.get("evict_obs_max") else "mean",
                               queries="last", dtype=tag)
        obs = col.reshape(hk, H // hk, n).max(1)
        np.testing.assert_allclose(obs, g["obs_scores"], rtol=1e-5, atol=1e-8)
        tol = 1e-6
    pos, prio = orc.evict_positions(g["idx"], col, kv_heads=hk, sink=bkw["sink"], window=bkw["window"],
                                    evict_keep=kw.get("evict_keep", 0), evict_window=kw.get("evict_window", 0),
                                    evict_pool=kw.get("evict_pool", 0), evict_pool_back=kw.get("evict_pool_back", 0))
    w = min(max(bkw["window"], kw.get("evict_window", 0)), n - bkw["sink"])
    assert kept_match(pos, g["kept"], prio, bkw["sink"], w, tol)


def test_oracle_forward_pool_spans():
    """forward_pool (modal_rd/attention.py:70-75) on the span cases of tests/test_kv_evict.py:134-152."""
    score = np.zeros((2, 20), dtype=np.float32)
    score[0, 5], score[1, 18] = 1.0, 0.5
    pooled = orc.forward_pool(score, 4)
    assert (pooled[0, 5:9] == 1).all() and (pooled[0, :5] == 0).all() and (pooled[0, 9:] == 0).all()
    assert (pooled[1, 18:] == 0.5).all() and (pooled[1, :18] == 0).all()
    score = np.zeros((1, 20), dtype=np.float32)
    score[0, 10] = 1.0
    pooled = orc.forward_pool(score, 3, back=4)
    assert (pooled[0, 6:13] == 1).all() and (pooled[0, :6] == 0).all() and (pooled[0, 13:] == 0).all()
    assert (orc.forward_pool(score, 0, back=2)[0, 8:11] == 1).all()


def test_oracle_decode_matches_reference(golden):
    """One-token decode (kernels/bigger_bird_decode.py) through the oracle equals the reference's
    bigger_bird_flash_ref on the last query row with the same (pooled) routes."""
    g = golden("decode")["decode"]
    s = cases.DECODE_SHAPE
    q, k, v, pooled = cases.decode_inputs()
    np.testing.assert_allclose(g["check"], cases.checksum(q, k, v), rtol=0, atol=0)
    n = s["n"]
    got = orc.decode(np32(q[0, :, n - 1]), np32(k[0]), np32(v[0]), pooled.numpy(), front=s["front"],
                     window=s["window"], scale=s["d"] ** -0.5)
    np.testing.assert_allclose(got, g["decode_out"], rtol=1e-5, atol=1e-5)


def test_oracle_pooled_probs_matches_reference(golden):
    """pooled_probs (kernels/bigger_bird_route.py) through the oracle equals the group mean of the
    reference's RDAttention.routes column scores for the last query (fp32, same masks)."""
    g = golden("decode")["decode"]
    s = cases.DECODE_SHAPE
    q, k, _, _ = cases.decode_inputs()
    n, hk = s["n"], s["hk"]
    got = orc.pooled_probs(np32(q[0, :, n - 1]), np32(k[0]), front=s["front"], window=s["window"],
                           scale=s["d"] ** -0.5)
    col = g["route_col"].reshape(hk, -1, n)
    want = col.mean(1)
    want[col[:, 0] == -1] = -1
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-9)
