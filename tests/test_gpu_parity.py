"""CUDA path vs the numpy oracle (needs an sm_100a GPU).

Tolerances (from the north star): attention output within max-abs 2e-2 and mean-abs 2e-3 of the
fp32 oracle computed with the SAME routes; route sets identical except where the oracle's scores
of the swapped keys lie within 1e-6 of the budget-th score; RoPE bit-identical.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import cases
from oracle import bigbird_oracle as orc

pytestmark = pytest.mark.gpu

ATOL_MAX, ATOL_MEAN, TIE_TOL = 2e-2, 2e-3, 1e-6
DEV = "cuda"


def np32(t):
    return t.detach().float().cpu().numpy()


def close(got, want, what=""):
    err = np.abs(np.asarray(got, dtype=np.float32) - np.asarray(want, dtype=np.float32))
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    assert err.max() <= ATOL_MAX and err.mean() <= ATOL_MEAN, f"{what}: max {err.max():.4g} mean {err.mean():.4g}"
    return err


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


# ----------------------------------------------------------------------------- RoPE

@pytest.mark.parametrize("case", cases.rope_cases(), ids=lambda c: c["name"])
def test_rope_bit_identical(case):
    from utmist_bigger_bird_b200 import rope_inplace
    from utmist_bigger_bird_b200.workload import rope_tables
    tag = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[case["dtype"]]
    cos, sin = rope_tables(case["n"], case["d"], case["theta"], case["dtype"])
    q = case["q"].to(DEV)
    k = case["k"].to(DEV).transpose(1, 2).contiguous().transpose(1, 2)        # strided view
    rope_inplace(q, cos[None].to(DEV), sin[None].to(DEV))
    rope_inplace(k, cos[None].to(DEV), sin[None].to(DEV))
    c, s = np32(cos), np32(sin)
    assert np.array_equal(np32(q), orc.rope(np32(case["q"]), c, s, tag))
    assert np.array_equal(np32(k), orc.rope(np32(case["k"]), c, s, tag))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
def test_rope_heads_d128_projection_views(dtype):
    """head_dim 128 with many heads: q and k as head views of `[1, n, H*d]` projection outputs (the
    model path's layout), rotated by `rope_inplace` and by `bb_sparse_prefill`'s single q+k launch;
    both bit-identical to the oracle."""
    from utmist_bigger_bird_b200 import _ops, rope_inplace
    from utmist_bigger_bird_b200.attention import route_query_positions
    from utmist_bigger_bird_b200.workload import rope_tables
    tag = {torch.bfloat16: "bf16", torch.float16: "f16"}[dtype]
    n, hq, hk, d = 1000, 32, 8, 128
    cos, sin = rope_tables(n, d, 500000.0, dtype)
    g = torch.Generator().manual_seed(12)
    q0 = torch.randn(1, n, hq * d, generator=g).to(dtype)
    k0 = torch.randn(1, n, hk * d, generator=g).to(dtype)
    v0 = torch.randn(1, n, hk * d, generator=g).to(dtype)
    c, s = np32(cos), np32(sin)
    want_q = orc.rope(np32(q0.view(1, n, hq, d).transpose(1, 2)), c, s, tag)
    want_k = orc.rope(np32(k0.view(1, n, hk, d).transpose(1, 2)), c, s, tag)
    heads = lambda t, h: t.to(DEV).view(1, n, h, d).transpose(1, 2)  # noqa: E731
    q, k = heads(q0, hq), heads(k0, hk)
    rope_inplace(q, cos[None].to(DEV), sin[None].to(DEV))
    rope_inplace(k, cos[None].to(DEV), sin[None].to(DEV))
    assert np.array_equal(np32(q), want_q) and np.array_equal(np32(k), want_k)
    q, k, v = heads(q0, hq), heads(k0, hk), heads(v0, hk)
    out = torch.empty((n, hq, d), device=DEV, dtype=dtype).permute(1, 0, 2)
    idx = torch.empty((hq, 64), device=DEV, dtype=torch.int32)
    qpos = route_query_positions(n, 64, "last", 16, 256, DEV)
    with torch.inference_mode():
        _ops.sparse_prefill_(q[0], k[0], v[0], qpos, out, idx, sink=16, window=256, budget=64, exact_tail=64,
                             scaling=d ** -0.5, cos=cos.to(DEV), sin=sin.to(DEV))
    assert np.array_equal(np32(q), want_q) and np.array_equal(np32(k), want_k)


# ----------------------------------------------------------------------------- kernel cases

@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("case", cases.flash_cases(), ids=lambda c: c["name"])
def test_flash_matches_oracle(case, dtype):
    from utmist_bigger_bird_b200 import bigger_bird_flash
    q, k, v = (case[x].to(DEV, dtype) for x in "qkv")
    mask = case["token_mask"]
    out = bigger_bird_flash(q, k, v, case["idx"].to(DEV), token_mask=None if mask is None else mask.to(DEV),
                            **case["kw"])
    assert out.shape == q.shape and out.stride() == (q.shape[2], q.shape[0] * q.shape[2], 1)
    want = orc.flash(np32(q), np32(k), np32(v), case["idx"].numpy(),
                     token_mask=None if mask is None else mask.numpy(), **case["kw"])
    close(np32(out), want, case["name"])


def test_grouped_equals_repeated():
    """tests/test_rd_attention_gqa.py:63-73: GQA in-kernel == repeat_interleave'd K/V."""
    from utmist_bigger_bird_b200 import bigger_bird_flash
    g = torch.Generator().manual_seed(1)
    h, gq, n, d = 8, 4, 384, 32
    q = torch.randn(h, n, d, generator=g).to(DEV, torch.bfloat16)
    k = torch.randn(h // gq, n, d, generator=g).to(DEV, torch.bfloat16)
    v = torch.randn(h // gq, n, d, generator=g).to(DEV, torch.bfloat16)
    idx = torch.stack([torch.randperm(n - 160, generator=g)[:24] + 16 for _ in range(h)]).sort(-1).values.int().to(DEV)
    grouped = bigger_bird_flash(q, k, v, idx[:, None], front=16, window=64, num_heads=h, kv_groups=gq, scale=0.2)
    repeated = bigger_bird_flash(q, k.repeat_interleave(gq, 0), v.repeat_interleave(gq, 0), idx[:, None],
                                 front=16, window=64, num_heads=h, scale=0.2)
    assert torch.equal(grouped, repeated)


@pytest.mark.parametrize("n,t,window,front,h,gq", [(4096, 64, 4096, 0, 8, 4), (20000, 256, 20000, 0, 4, 2),
                                                   (9000, 200, 1000, 32, 4, 4)])
def test_long_rows_split_over_keys(n, t, window, front, h, gq):
    """Few query rows over many keys (the exact tail shape): the kernel splits the key range."""
    from utmist_bigger_bird_b200 import bigger_bird_flash
    g = torch.Generator().manual_seed(n)
    d = 128
    q = (torch.randn(h, t, d, generator=g) * 0.3).to(DEV, torch.bfloat16)
    k = torch.randn(h // gq, n, d, generator=g).to(DEV, torch.bfloat16)
    v = torch.randn(h // gq, n, d, generator=g).to(DEV, torch.bfloat16)
    idx = torch.stack([torch.randperm(n, generator=g)[:40] for _ in range(h)]).int()
    out = bigger_bird_flash(q, k, v, idx.to(DEV)[:, None], front=front, window=window, num_heads=h,
                            kv_groups=gq, scale=d ** -0.5)
    want = orc.flash(np32(q), np32(k), np32(v), idx.numpy()[:, None], front=front, window=window,
                     num_heads=h, kv_groups=gq, scale=d ** -0.5)
    close(np32(out), want, "split")


def test_tail_equals_dense_causal_rows():
    """tests/test_rd_attention_gqa.py:90-102: window=n == SDPA causal rows."""
    import torch.nn.functional as F
    from utmist_bigger_bird_b200 import bigger_bird_flash
    g = torch.Generator().manual_seed(3)
    h, gq, n, d, r = 8, 4, 3000, 64, 300
    q = torch.randn(h, n, d, generator=g).to(DEV, torch.bfloat16)
    k = torch.randn(h // gq, n, d, generator=g).to(DEV, torch.bfloat16)
    v = torch.randn(h // gq, n, d, generator=g).to(DEV, torch.bfloat16)
    none = torch.full((h, 1, 1), -1, dtype=torch.int32, device=DEV)
    tail = bigger_bird_flash(q[:, n - r:], k, v, none, front=0, window=n, num_heads=h, kv_groups=gq, scale=0.3)
    qp = torch.arange(n - r, n, device=DEV)[:, None]
    mask = torch.arange(n, device=DEV)[None] <= qp
    want = F.scaled_dot_product_attention(q[None, :, n - r:].float(), k[None].float(), v[None].float(),
                                          attn_mask=mask, scale=0.3, enable_gqa=True)[0]
    close(np32(tail), np32(want), "tail")


def test_full_budget_equals_sdpa():
    """modal_rd/selfcheck.py:37-41: routes covering every key => exact causal attention."""
    import torch.nn.functional as F
    from utmist_bigger_bird_b200 import bigger_bird_flash
    torch.manual_seed(0)
    h, n, d, sink, window = 32, 4096, 128, 64, 512
    Q, K, V = (torch.randn(h, n, d, device=DEV, dtype=torch.bfloat16) for _ in range(3))
    Q = Q * d ** -0.5
    full = torch.arange(sink, n - window, device=DEV, dtype=torch.int32).expand(h, -1).contiguous()
    out = bigger_bird_flash(Q, K, V, full.view(h, 1, -1), front=sink, window=window, num_heads=h, scale=1.0)
    dense = F.scaled_dot_product_attention(Q[None], K[None], V[None], is_causal=True, scale=1.0)[0]
    close(np32(out), np32(dense), "full budget")


@pytest.mark.parametrize("n", [524224, 524288, 524352, 995993])
def test_long_index_identity(n):
    """modal_rd/check_long_indexing.py:32,40-55 (the reference's four lengths): window=1, no routes
    => out[h] == v[h // 4] exactly, with [n, H, d] strided views (element offsets beyond 2^31)."""
    from utmist_bigger_bird_b200 import bigger_bird_flash
    h, hk, d = 32, 8, 128
    q = torch.zeros((n, h, d), device=DEV, dtype=torch.bfloat16).permute(1, 0, 2)
    k = torch.zeros((n, hk, d), device=DEV, dtype=torch.bfloat16).permute(1, 0, 2)
    v = torch.empty_like(k)
    for head in range(hk):
        v[head].copy_(((torch.arange(n, device=DEV) % 97).float() + head * .25)[:, None].expand(n, d))
    idx = torch.empty((h, 1, 0), device=DEV, dtype=torch.int32)
    out = bigger_bird_flash(q, k, v, idx, front=0, window=1, num_heads=h, kv_groups=4)
    torch.cuda.synchronize()
    for head in range(h):
        assert torch.equal(out[head], v[head // 4]), head


def test_validation_errors_match_reference():
    """kernels/bigger_bird_flash.py:110-130 error behaviour."""
    from utmist_bigger_bird_b200 import bigger_bird_flash
    q = torch.randn(4, 16, 32, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(2, 16, 32, device=DEV, dtype=torch.bfloat16)
    idx = torch.full((4, 1, 3), -1, dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError):
        bigger_bird_flash(q.float(), k.float(), k.float(), idx, num_heads=4, kv_groups=2)
    with pytest.raises(ValueError):
        bigger_bird_flash(q, k, k[:, :8], idx, num_heads=4, kv_groups=2)
    with pytest.raises(ValueError):
        bigger_bird_flash(q, k, k, idx, num_heads=4, kv_groups=2, window=0)
    with pytest.raises(ValueError):
        bigger_bird_flash(q, k[:, :8], k[:, :8], idx, num_heads=4, kv_groups=2)
    with pytest.raises(ValueError):
        bigger_bird_flash(q, k, k, idx, num_heads=4, kv_groups=2, route_chunk=32, block_m=64)
    with pytest.raises(ValueError):
        bigger_bird_flash(q, k, k, idx, num_heads=4, kv_groups=2, token_mask=torch.ones(1, 16, device=DEV))
    out = bigger_bird_flash(q, k, k, idx, num_heads=4, kv_groups=2, front=4, window=5)
    assert torch.isfinite(out).all()


# ----------------------------------------------------------------------------- routes + prefill

@pytest.mark.parametrize("name,kw", list(cases.prefill_configs()) + [(f"extra_{a}", b) for a, b in cases.EXTRA_ROUTE_CONFIGS.items()],
                         ids=lambda x: x if isinstance(x, str) else "")
def test_prefill_matches_oracle(name, kw):
    from utmist_bigger_bird_b200 import RDAttention
    s = cases.PREFILL_SHAPE
    q, k, v, rows = cases.prefill_inputs(torch.bfloat16)
    kw = dict(kw)
    attn = RDAttention(base(s["H"], s["hk"], s["d"]), block_m=16, block_n=16, **kw)
    with torch.inference_mode():
        out = attn.sparse_prefill(q.to(DEV), k.to(DEV), v.to(DEV))
    idx = attn.last_routes.cpu().numpy()
    pool, queries = kw.pop("route_pool", "mean"), kw.pop("route_queries", "last")
    kw.pop("scope_chunk", None)
    qn, kn, vn = np32(q[0]), np32(k[0]), np32(v[0])
    want_idx, col = orc.routes(qn, kn, scaling=s["d"] ** -0.5, pool=pool, queries=queries, dtype="bf16",
                               return_scores=True, sink=kw["sink"], window=kw["window"],
                               vertical=kw["vertical"], vertical_sqrt=kw.get("vertical_sqrt", 0.0),
                               n_route=kw["n_route"])
    ok, swapped, gap = orc.route_sets_match(idx, want_idx, col, TIE_TOL)
    assert ok, (name, swapped, gap)
    assert (np.diff(idx, axis=-1) > 0).all(), "routes must be sorted and unique"
    n = s["n"]
    if attn.route_budget(n) == 0 or n <= kw["sink"] + kw["window"]:
        return
    okw = {a: b for a, b in kw.items() if a in ("sink", "window", "vertical", "exact_tail", "vertical_scope")}
    want, _ = orc.sparse_prefill(qn, kn, vn, scaling=s["d"] ** -0.5, dtype="bf16", idx=idx,
                                 scope_chunk=64, **okw)
    close(np32(out[0]), want, name)


def _layer_parity(cfg, rows, check_rope=True):
    from utmist_bigger_bird_b200 import RDAttention, rope_inplace
    from utmist_bigger_bird_b200.workload import make_layer
    q, k, v, cos, sin, planted = make_layer(cfg)
    q, k, v, cos, sin = (t.to(torch.bfloat16) for t in (q, k, v, cos, sin))
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    attn = RDAttention(base(cfg.heads, cfg.kv_heads, cfg.head_dim), **cfg.attn_kwargs())
    with torch.inference_mode():
        rope_inplace(qd, cos.to(DEV), sin.to(DEV))
        rope_inplace(kd, cos.to(DEV), sin.to(DEV))
        out = attn.sparse_prefill(qd, kd, vd)
    torch.cuda.synchronize()
    c, s_ = np32(cos[0]), np32(sin[0])
    kn = orc.rope(np32(k[0]), c, s_, "bf16")
    assert np.array_equal(np32(kd[0]), kn)
    qn = np32(qd[0])
    if check_rope:
        assert np.array_equal(qn, orc.rope(np32(q[0]), c, s_, "bf16"))
    idx = attn.last_routes.cpu().numpy()
    want_idx, col = orc.routes(qn, kn, scaling=cfg.scaling, sink=cfg.sink, window=cfg.window,
                               vertical=cfg.vertical, n_route=cfg.n_route, dtype="bf16", return_scores=True)
    ok, swapped, gap = orc.route_sets_match(idx, want_idx, col, TIE_TOL)
    assert ok, (swapped, gap)
    want, _ = orc.sparse_prefill(qn, kn, np32(v[0]), scaling=cfg.scaling, sink=cfg.sink, window=cfg.window,
                                 vertical=cfg.vertical, exact_tail=cfg.exact_tail, n_route=cfg.n_route,
                                 dtype="bf16", rows=rows, idx=idx)
    return close(np32(out[0][:, rows]), want, cfg.name), swapped


def test_config1_layer_bf16():
    """BASELINE config 1 shape (n=8192, 32/8 heads, d=128, 64/2048/128/256) in bf16."""
    from utmist_bigger_bird_b200.workload import CONFIGS
    cfg = CONFIGS["config1"]
    rows = np.unique(np.concatenate([np.arange(0, cfg.n, 61), np.arange(cfg.n - 300, cfg.n)]))
    _layer_parity(cfg, rows)


def test_config2_layer_128k():
    """BASELINE config 2 (n=131072, bf16, 64/16384/512/256): full-size route parity and sampled
    attention rows (every tail row class, window edges, spread rows)."""
    from utmist_bigger_bird_b200.workload import CONFIGS
    cfg = CONFIGS["config2"]
    n = cfg.n
    rows = np.unique(np.concatenate([np.arange(0, n, 4099), [cfg.window - 1, cfg.window, cfg.window + 1],
                                     np.arange(n - 260, n - 250), np.arange(n - 6, n)]))
    _layer_parity(cfg, rows, check_rope=False)


def test_sparse_prefill_single_c_call_matches_module():
    """bb_sparse_prefill (RoPE + routes + main + tail in one C call) == the module path."""
    from utmist_bigger_bird_b200 import RDAttention, _ops, rope_inplace
    from utmist_bigger_bird_b200.attention import route_query_positions
    from utmist_bigger_bird_b200.workload import LayerConfig, make_layer
    cfg = LayerConfig("c", 4096, torch.bfloat16, 9, 1.0, 4, 64, None, 64, 1024, 128, 200)
    q, k, v, cos, sin, _ = make_layer(cfg)
    q, k, v, cos, sin = (t.to(DEV) for t in (q, k, v, cos, sin))
    attn = RDAttention(base(cfg.heads, cfg.kv_heads, cfg.head_dim), **cfg.attn_kwargs())
    q1, k1 = q.clone(), k.clone()
    with torch.inference_mode():
        rope_inplace(q1, cos, sin)
        rope_inplace(k1, cos, sin)
        want = attn.sparse_prefill(q1, k1, v)
        q2, k2 = q.clone(), k.clone()
        budget = attn.route_budget(cfg.n)
        out = torch.empty((cfg.n, cfg.heads, cfg.head_dim), device=DEV, dtype=q.dtype).permute(1, 0, 2)
        idx = torch.empty((cfg.heads, budget), device=DEV, dtype=torch.int32)
        qpos = route_query_positions(cfg.n, cfg.n_route, "last", cfg.sink, cfg.window, DEV)
        _ops.sparse_prefill_(q2[0], k2[0], v[0], qpos, out, idx, sink=cfg.sink, window=cfg.window,
                             budget=budget, exact_tail=cfg.exact_tail, scaling=cfg.scaling,
                             cos=cos[0], sin=sin[0])
    assert torch.equal(q2, q1) and torch.equal(k2, k1)
    assert torch.equal(idx, attn.last_routes)
    assert torch.equal(out, want[0])


def test_model_full_budget_matches_native_hf():
    """A tiny random Llama with every layer on the sparse path and a budget that covers every key
    (so the union is all causal keys) reproduces the native HF (SDPA) prefill logits."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from utmist_bigger_bird_b200 import install
    cfg = LlamaConfig(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=16, num_key_value_heads=4, max_position_embeddings=8192,
                      attn_implementation="sdpa")
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).to(DEV, torch.bfloat16).eval()
    ids = torch.randint(0, 512, (1, 700), device=DEV)
    with torch.inference_mode():
        want = model(ids, use_cache=True).logits.float()
        install(model, "vs", sink=8, window=96, vertical=10 ** 6, n_route=16, exact_tail=32)
        got = model(ids, use_cache=True).logits.float()
    routes = model.model.layers[0].self_attn.last_routes
    assert routes is not None and routes.shape[-1] == 700 - 8 - 96
    err = (got - want).abs()
    assert err.max() < 0.1 and err.mean() < 1e-2, (err.max().item(), err.mean().item())


def test_no_kv_sized_copies():
    """tests/test_rd_attention_gqa.py:131-187: sparse_prefill makes no K/V-sized copies."""
    from torch.utils._python_dispatch import TorchDispatchMode
    from utmist_bigger_bird_b200 import RDAttention

    class AllocLog(TorchDispatchMode):
        def __init__(self):
            super().__init__()
            self.records = []

        def __torch_dispatch__(self, func, types, args=(), kwargs=None):
            out = func(*args, **(kwargs or {}))
            for t in torch.utils._pytree.tree_leaves(out):
                if isinstance(t, torch.Tensor) and t.numel() * t.element_size() >= 1 << 16:
                    self.records.append((t.numel() * t.element_size(), str(func)))
            return out

    n, H, hk, d = 2048, 16, 4, 32
    attn = RDAttention(base(H, hk, d), sink=16, window=256, vertical=64, n_route=32, exact_tail=64)
    q = torch.randn(1, H, n, d, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(1, hk, n, d, device=DEV, dtype=torch.bfloat16)
    v = torch.randn_like(k)
    with torch.inference_mode(), AllocLog() as log:
        attn.sparse_prefill(q, k, v)
    h_wide = H * n * d * 2
    copies = [(b, f) for b, f in log.records if b >= h_wide // 4 and any(
        c in f for c in ("repeat_interleave", "index_select", "clone", "contiguous", "_to_copy"))]
    assert not copies, copies


def test_no_device_fault_recorded():
    """No kernel gave up a bounded wait during the tests above (the fault word stays 0)."""
    import ctypes as C
    from utmist_bigger_bird_b200 import _lib
    torch.cuda.synchronize()
    code = C.c_int(-1)
    _lib.check(_lib.lib().bb_device_fault(C.byref(code)), "device_fault")
    assert code.value == 0, f"a kernel recorded fault code {code.value}"
