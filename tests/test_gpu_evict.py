"""KV eviction on the GPU (bb_kv_evict) against the oracle's restatement of RDAttention.evict
(modal_rd/attention.py:226-259), and the reference test suite's eviction invariants
(tests/test_kv_evict.py) on a tiny Llama."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import cases
from oracle import bigbird_oracle as orc
from test_oracle_golden import kept_match

pytestmark = pytest.mark.gpu
DEV = "cuda"


def base(h, hk, d, layer_idx=0):
    return SimpleNamespace(config=SimpleNamespace(num_attention_heads=h, num_key_value_heads=hk),
                           layer_idx=layer_idx, head_dim=d, scaling=d ** -0.5,
                           q_proj=None, k_proj=None, v_proj=None, o_proj=None)


def check_gather(pos, k, v, kk, vv):
    """The kept K/V rows are exactly the rows at the kept positions."""
    gi = pos[:, :, None].expand(-1, -1, k.shape[-1])
    assert torch.equal(kk, k.gather(1, gi))
    assert torch.equal(vv, v.gather(1, gi))


@pytest.mark.parametrize("knobs", [dict(), dict(keep=3000), dict(pool=8), dict(pool_back=8), dict(pool=4, pool_back=3),
                                   dict(unsorted=1), dict(budget=4096)],
                         ids=lambda k: ",".join(f"{a}={b}" for a, b in k.items()) or "default")
def test_kv_evict_kernel_matches_oracle(knobs):
    """Every policy knob against the oracle, plus routes in no particular order and a budget of
    4096 routes per head (16384 per KV-head group)."""
    from utmist_bigger_bird_b200 import _ops
    H, hk, n, d, sink, w = 32, 8, 32768, 128, 64, 4096
    budget = knobs.get("budget", 512)
    g = torch.Generator(device=DEV).manual_seed(7)
    col = torch.rand(H, n, device=DEV, generator=g) * 1e-4
    col[:, :sink] = -1
    col[:, n - w:] = -1
    idx = torch.stack([torch.randperm(n - sink - w, device=DEV, generator=g)[:budget] + sink for _ in range(H)])
    idx = (idx if knobs.get("unsorted") else idx.sort(-1).values).to(torch.int32)
    k = torch.randn(hk, n, d, device=DEV, generator=g).to(torch.bfloat16)
    v = torch.randn(hk, n, d, device=DEV, generator=g).to(torch.bfloat16)
    keep = knobs.get("keep", (H // hk) * budget)
    kk, vv, pos = _ops.kv_evict_(idx, col, k, v, sink=sink, window=w, keep=keep, pool=knobs.get("pool", 0),
                                 pool_back=knobs.get("pool_back", 0))
    torch.cuda.synchronize()
    want, prio = orc.evict_positions(idx.cpu().numpy(), col.cpu().numpy(), kv_heads=hk, sink=sink, window=w,
                                     evict_keep=keep if "keep" in knobs else 0,
                                     evict_pool=knobs.get("pool", 0), evict_pool_back=knobs.get("pool_back", 0))
    got = pos.cpu().numpy()
    assert kept_match(got, want, prio, sink, w)
    assert (got[:, :-1] < got[:, 1:]).all(), "positions sorted and unique"
    check_gather(pos, k, v, kk, vv)


@pytest.mark.parametrize("name", list(cases.EVICT_CONFIGS))
def test_evict_module_on_golden_configs(golden, name):
    """RDAttention.evict on the golden inputs (bf16): kept positions equal the oracle's for the
    GPU's own routes and column scores (up to ties), keep the sink, the window and every route,
    and the cache holds exactly the K/V rows at them. The reference's own kept sets (CPU routes)
    have the same sizes."""
    from utmist_bigger_bird_b200 import RDAttention
    s, bkw, kw = cases.PREFILL_SHAPE, cases.EVICT_BASE_KW, cases.EVICT_CONFIGS[name]
    H, hk, n, d = s["H"], s["hk"], s["n"], s["d"]
    q, k, v, _ = cases.prefill_inputs(torch.bfloat16)
    q, k, v = q.to(DEV), k.to(DEV), v.to(DEV)
    attn = RDAttention(base(H, hk, d), kv_evict=True, block_m=16, block_n=16, **bkw, **kw)
    cache = SimpleNamespace(layers=[SimpleNamespace(keys=None, values=None)])
    with torch.inference_mode():
        attn.sparse_prefill(q, k, v)
        idx, col = attn.last_routes.clone(), attn._col.clone()
        obs = attn._evict_col(q, k) if kw.get("evict_obs") else None
        attn.evict(cache, q, k, v)
    torch.cuda.synchronize()
    ref = golden("evict")[f"bf16_{name}"]["kept"]
    got = attn.kept.cpu().numpy()
    assert got.shape == ref.shape
    if kw.get("evict_full_layers"):
        assert np.array_equal(got, np.tile(np.arange(n), (hk, 1)))
        return
    w = min(max(bkw["window"], kw.get("evict_window", 0)), n - bkw["sink"])
    want, prio = orc.evict_positions(idx.cpu().numpy(), (obs if obs is not None else col).cpu().numpy(),
                                     kv_heads=hk, sink=bkw["sink"], window=bkw["window"],
                                     evict_keep=kw.get("evict_keep", 0), evict_window=kw.get("evict_window", 0),
                                     evict_pool=kw.get("evict_pool", 0), evict_pool_back=kw.get("evict_pool_back", 0))
    assert kept_match(got, want, prio, bkw["sink"], w)
    assert (got[:, :-1] < got[:, 1:]).all()
    assert (got[:, :bkw["sink"]] == np.arange(bkw["sink"])).all()
    assert (got[:, -w:] == np.arange(n - w, n)).all()
    g = H // hk
    for h in range(H):
        assert np.isin(idx[h].cpu().numpy(), got[h // g]).all(), "every routed column survives"
    check_gather(attn.kept, k[0], v[0], cache.layers[0].keys[0], cache.layers[0].values[0])


def test_tiny_llama_evict_keeps_prefill_and_shrinks_cache():
    """tests/test_kv_evict.py:28-64 on the GPU: eviction leaves the prefill logits unchanged; every
    layer's cache shrinks to sink + window + g * vertical rows, holding exactly the full cache's
    rows at sorted, unique kept positions that include the sink, the window and every route."""
    from transformers import DynamicCache, LlamaConfig, LlamaForCausalLM
    from utmist_bigger_bird_b200 import install
    kw = dict(sink=8, window=96, vertical=24, n_route=16, exact_tail=24, block_m=16, block_n=16)
    n = 400
    cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=4096,
                      attn_implementation="sdpa")
    torch.manual_seed(4)
    model = LlamaForCausalLM(cfg).to(DEV, torch.bfloat16).eval()
    ids = torch.randint(0, 512, (1, n), device=DEV)

    def prefill():
        cache = DynamicCache()
        with torch.inference_mode():
            logits = model(ids, past_key_values=cache, use_cache=True).logits
        return logits, cache

    install(model, "vs", **kw)
    want, full = prefill()
    install(model, "vs", kv_evict=True, **kw)
    got, cache = prefill()
    assert torch.equal(got, want), "eviction must not change prefill output"
    g = cfg.num_attention_heads // cfg.num_key_value_heads
    m = kw["sink"] + kw["window"] + g * kw["vertical"]
    for i, layer in enumerate(model.model.layers):
        a, kept = layer.self_attn, layer.self_attn.kept
        assert cache.layers[i].keys.shape == (1, cfg.num_key_value_heads, m, cfg.hidden_size // cfg.num_attention_heads)
        assert (kept[:, :-1] < kept[:, 1:]).all()
        assert (kept[:, :kw["sink"]] == torch.arange(kw["sink"], device=DEV)).all()
        assert (kept[:, -kw["window"]:] == torch.arange(n - kw["window"], n, device=DEV)).all()
        for h in range(cfg.num_attention_heads):
            assert torch.isin(a.last_routes[h].long(), kept[h // g]).all()
        gi = kept[None, :, :, None].expand(1, -1, -1, full.layers[i].keys.shape[-1])
        assert torch.equal(cache.layers[i].keys, full.layers[i].keys.gather(2, gi))
        assert torch.equal(cache.layers[i].values, full.layers[i].values.gather(2, gi))


def test_kv_evict_rejects_bad_arguments():
    from utmist_bigger_bird_b200 import _ops
    k = torch.zeros(2, 64, 32, device=DEV, dtype=torch.bfloat16)
    col = torch.zeros(8, 64, device=DEV)
    idx = torch.zeros(8, 4, device=DEV, dtype=torch.int32)
    with pytest.raises(ValueError):
        _ops.kv_evict_(idx, col, k, k, sink=40, window=40, keep=0)          # sink + window > n
    with pytest.raises(ValueError):
        _ops.kv_evict_(idx, col, k, k, sink=8, window=8, keep=64)           # keep > n - sink - window
    with pytest.raises(ValueError):
        _ops.kv_evict_(idx, col.double(), k, k, sink=8, window=8, keep=4)   # col must be fp32


@pytest.mark.parametrize("n", [32768, 131072])
def test_kv_evict_ties_take_lowest_positions(n):
    """Column scores on four levels only (massive ties at the cut): the kept set equals the
    oracle's exactly, ties resolved towards lower positions (the row-wise top-k runs as a cluster
    of CTAs at these sizes, so this pins its cross-CTA tie order)."""
    from utmist_bigger_bird_b200 import _ops
    H, hk, d, budget, sink, w = 32, 8, 64, 512, 64, 4096
    g = torch.Generator(device=DEV).manual_seed(11)
    col = torch.floor(torch.rand(H, n, device=DEV, generator=g) * 4) * 2.5e-5
    col[:, :sink] = -1
    col[:, n - w:] = -1
    idx = torch.stack([torch.randperm(n - sink - w, device=DEV, generator=g)[:budget] + sink for _ in range(H)])
    idx = idx.sort(-1).values.to(torch.int32)
    k = torch.randn(hk, n, d, device=DEV, generator=g).to(torch.bfloat16)
    keep = 3000
    kk, vv, pos = _ops.kv_evict_(idx, col, k, k, sink=sink, window=w, keep=keep)
    torch.cuda.synchronize()
    want, _ = orc.evict_positions(idx.cpu().numpy(), col.cpu().numpy(), kv_heads=hk, sink=sink, window=w,
                                  evict_keep=keep)
    assert np.array_equal(pos.cpu().numpy(), want)
