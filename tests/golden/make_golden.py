"""Generate the golden vectors in this folder by running the REFERENCE implementation itself.

Run once where a checkout of the reference is available (read-only), naming it with
``BB_REFERENCE`` or as the first argument::

    PYTHONDONTWRITEBYTECODE=1 BB_REFERENCE=<reference checkout> python tests/golden/make_golden.py

It imports ``modal_rd.attention`` (``RDAttention``, ``rope_inplace``) and
``kernels.bigger_bird_flash_ref`` from the reference and runs them on the CPU (the reference's
dispatcher at ``modal_rd/attention.py:41-45`` picks the pure-PyTorch kernel for CPU tensors).
Inputs come from the seeded generators in ``cases.py``; only outputs (row-subsampled where
large) and input checksums are stored. bf16 outputs are stored as float32 (exact).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
_ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("BB_REFERENCE")
if not _ref:
    raise SystemExit("make_golden.py: name the reference checkout with BB_REFERENCE=<path> or as the first argument")
REF = Path(_ref)
sys.dont_write_bytecode = True
sys.path.insert(0, str(REF))
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

from kernels.bigger_bird_flash_ref import bigger_bird_flash_ref  # noqa: E402  (reference)
from modal_rd import attention as ref_attn  # noqa: E402  (reference)
from transformers import LlamaConfig  # noqa: E402
from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding  # noqa: E402

import cases  # noqa: E402
from utmist_bigger_bird_b200.workload import CONFIGS, make_layer, rope_tables  # noqa: E402

torch.set_num_threads(os.cpu_count())


def f32(t):
    return t.detach().float().cpu().numpy()


def base(h, hk, d):
    return SimpleNamespace(config=SimpleNamespace(num_attention_heads=h, num_key_value_heads=hk),
                           layer_idx=0, head_dim=d, scaling=d ** -0.5,
                           q_proj=None, k_proj=None, v_proj=None, o_proj=None)


def gen_rope():
    out = {}
    for c in cases.rope_cases():
        q, k, d, n = c["q"], c["k"], c["d"], c["n"]
        check = cases.checksum(q, k)
        cfg = LlamaConfig(hidden_size=q.shape[1] * d, num_attention_heads=q.shape[1],
                          num_key_value_heads=k.shape[1], head_dim=d, rope_theta=c["theta"],
                          max_position_embeddings=8192)
        cos, sin = LlamaRotaryEmbedding(cfg)(q, torch.arange(n)[None])
        # The workload's own table builder must agree bit-for-bit with HF's.
        c2, s2 = rope_tables(n, d, c["theta"], q.dtype)
        assert torch.equal(c2, cos[0]) and torch.equal(s2, sin[0]), c["name"]
        k_strided = k.clone().transpose(1, 2).contiguous().transpose(1, 2)
        got_q = ref_attn.rope_inplace(q.clone(), cos, sin, 64)
        got_k = ref_attn.rope_inplace(k_strided, cos, sin, 64)
        out[c["name"]] = dict(q_out=f32(got_q), k_out=f32(got_k), cos=f32(cos), sin=f32(sin),
                              check=check)
    return out


def gen_flash():
    out = {}
    for c in cases.flash_cases():
        rows = c["rows"]
        rec = dict(check=cases.checksum(c["q"], c["k"], c["v"]))
        for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
            o = bigger_bird_flash_ref(c["q"].to(dt), c["k"].to(dt), c["v"].to(dt), c["idx"],
                                      token_mask=c["token_mask"], **c["kw"])
            rec[f"out_{tag}"] = f32(o[:, rows])
        out[c["name"]] = rec
    return out


def gen_prefill():
    s = cases.PREFILL_SHAPE
    out = {}
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        q, k, v, rows = cases.prefill_inputs(dt)
        out[f"inputs_{tag}"] = dict(check=cases.checksum(q, k, v))
        for name, kw in cases.prefill_configs():
            attn = ref_attn.RDAttention(base(s["H"], s["hk"], s["d"]), kv_evict=True, block_m=16, block_n=16, **kw)
            with torch.inference_mode():
                o = attn.sparse_prefill(q, k, v)
            rec = dict(idx=attn.last_routes.numpy(), out=f32(o[0][:, rows]))
            if kw["exact_tail"] == 0 and kw["vertical_scope"] == 0:
                rec["col"] = attn._col.numpy()
            out[f"{tag}_{name}"] = rec
        for name, kw in cases.EXTRA_ROUTE_CONFIGS.items():
            attn = ref_attn.RDAttention(base(s["H"], s["hk"], s["d"]), kv_evict=True, **kw)
            with torch.inference_mode():
                idx = attn.routes(q, k)
            out[f"{tag}_{name}"] = dict(idx=idx.numpy(), col=attn._col.numpy())
    return out


def gen_config1():
    """BASELINE config 1 (n=8192) through the reference: RoPE, routes, sparse prefill. Stores the
    routes, the per-head boundary scores (budget-th and next) and sampled output rows."""
    cfg = CONFIGS["config1"]
    q, k, v, cos, sin, planted = make_layer(cfg)
    n = cfg.n
    rows = cases.config1_rows(n)
    check = cases.checksum(q, k, v)
    out = {}
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        qq, kk, vv = q.to(dt).clone(), k.to(dt).clone(), v.to(dt).clone()
        cc, ss = cos.to(dt), sin.to(dt)
        ref_attn.rope_inplace(qq, cc, ss)
        ref_attn.rope_inplace(kk, cc, ss)
        attn = ref_attn.RDAttention(base(cfg.heads, cfg.kv_heads, cfg.head_dim), kv_evict=True,
                                    **cfg.attn_kwargs())
        with torch.inference_mode():
            o = attn.sparse_prefill(qq, kk, vv)
        col = attn._col
        budget = attn.last_routes.shape[-1]
        top = col.topk(budget + 1, dim=-1).values
        out[tag] = dict(idx=attn.last_routes.numpy(), kth=top[:, budget - 1].numpy(),
                        next=top[:, budget].numpy(), out=f32(o[0][:, rows]),
                        planted=planted.numpy(), check=check,
                        q_rot_tail=f32(qq[0, :, n - 2:]), k_rot_head=f32(kk[0, :, :2]))
    return out


def gen_evict():
    """KV eviction through the reference: routes of the prefill, then RDAttention.evict on a
    one-layer cache. Stores the routes, the routing column scores and the kept positions."""
    s = cases.PREFILL_SHAPE
    out = {}
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        q, k, v, _ = cases.prefill_inputs(dt)
        for name, kw in cases.EVICT_CONFIGS.items():
            attn = ref_attn.RDAttention(base(s["H"], s["hk"], s["d"]), kv_evict=True, **cases.EVICT_BASE_KW, **kw)
            cache = SimpleNamespace(layers=[SimpleNamespace(keys=None, values=None)])
            with torch.inference_mode():
                attn.sparse_prefill(q, k, v)
                idx, col = attn.last_routes.clone(), attn._col.clone()
                attn.evict(cache, q, k, v)
            rec = dict(idx=idx.numpy(), col=col.numpy(), kept=attn.kept.numpy())
            if kw.get("evict_obs"):
                with torch.inference_mode():
                    rec["obs_scores"] = attn.evict_scores(q, k).numpy()
            out[f"{tag}_{name}"] = rec
    return out


def gen_decode():
    """One-token decode and decode routing through the reference's CPU functions (fp32)."""
    s = cases.DECODE_SHAPE
    q, k, v, pooled = cases.decode_inputs()
    n, H, hk, d = s["n"], s["H"], s["hk"], s["d"]
    g = H // hk
    per_head = pooled.repeat_interleave(g, 0)[:, None, :]       # [H, 1, R]
    o = bigger_bird_flash_ref(q[0, :, n - 1:], k[0], v[0], per_head, front=s["front"], window=s["window"],
                              num_heads=H, kv_groups=g, scale=d ** -0.5)
    out = dict(check=cases.checksum(q, k, v), pooled=pooled.numpy(), decode_out=f32(o[:, 0]))
    attn = ref_attn.RDAttention(base(H, hk, d), kv_evict=True, sink=s["front"], window=s["window"],
                                vertical=s["R"], n_route=1)
    with torch.inference_mode():
        attn.routes(q, k)
    out["route_col"] = attn._col.numpy()                          # [H, n], sink/window columns -1
    return {"decode": out}


def save(name, groups):
    flat = {}
    for key, rec in groups.items():
        for field_, val in rec.items():
            flat[f"{key}/{field_}"] = np.asarray(val)
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, **flat)
    print(f"{path.name}: {len(groups)} records, {path.stat().st_size / 1e3:.0f} KB")


if __name__ == "__main__":
    save("rope", gen_rope())
    save("flash", gen_flash())
    save("prefill", gen_prefill())
    save("config1", gen_config1())
    save("evict", gen_evict())
    save("decode", gen_decode())
