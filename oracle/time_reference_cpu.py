"""Times the reference's own CPU path against this repository's two CPU restatements (the numpy
parity oracle ``bigbird_oracle`` and the torch ``torch_port`` that ``bench.py`` times as its CPU
leg) on the same bounded sample of config 2, so that the CPU baseline ``bench.py`` reports (run on
the GPU box's host cores, where the reference does not travel) can be related to the reference's own
CPU speed.

Test infrastructure, like ``tests/golden/make_golden.py``: it imports the reference checkout named by
``BB_REFERENCE`` (or the first argument) read-only and runs on the CPU only::

    PYTHONDONTWRITEBYTECODE=1 BB_REFERENCE=<reference checkout> python oracle/time_reference_cpu.py

Sample (one KV head of config 2, 131072 tokens, fp32 math on bf16-valued inputs):
  * RoPE of its 4 query heads and its K (``modal_rd/attention.py:51-60``);
  * ``RDAttention.routes`` for those 4 heads over all keys (``modal_rd/attention.py:143-174``);
  * the attention of the last 48 query rows of 2 of those heads with the routes
    (``kernels/bigger_bird_flash_ref.py:10-52``; the reference's kernel takes a query suffix).
Prints one JSON line: seconds per part for each side, the thread count, and whether each
restatement's routes equal the reference's (as sets) and how far its attention values lie from them.
"""
from __future__ import annotations

import json
import os
import sys
import time
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
_ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("BB_REFERENCE")
if not _ref:
    raise SystemExit("time_reference_cpu.py: name the reference checkout with BB_REFERENCE=<path> or as the first argument")
sys.dont_write_bytecode = True
sys.path.insert(0, str(Path(_ref)))
sys.path.insert(0, str(REPO))

from kernels.bigger_bird_flash_ref import bigger_bird_flash_ref  # noqa: E402  (reference)
from modal_rd import attention as ref_attn  # noqa: E402  (reference)

from oracle import bigbird_oracle as orc  # noqa: E402
from oracle import torch_port as tp  # noqa: E402
from utmist_bigger_bird_b200.workload import CONFIGS, make_layer  # noqa: E402


def timed(fn):
    t0 = time.perf_counter()
    out = fn()
    return out, time.perf_counter() - t0


def main():
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = CONFIGS["config2"]
    q, k, v, cos, sin, _ = make_layer(cfg, kv_heads=[0])          # q [1, 4, n, d], k/v [1, 1, n, d]
    q, k, v, cos, sin = (t.float() for t in (q, k, v, cos, sin))   # bf16 values, fp32 math on both sides
    n, d, rows, heads = cfg.n, cfg.head_dim, 48, 2
    g = cfg.heads // cfg.kv_heads
    res = {"sample": f"config2 KV head 0: RoPE of 4 query heads + K, routes of 4 heads over {n} keys, "
                     f"attention of the last {rows} rows of {heads} heads", "threads": threads}

    # reference
    qr, kr = q.clone(), k.clone()
    _, t_rope = timed(lambda: (ref_attn.rope_inplace(qr, cos, sin), ref_attn.rope_inplace(kr, cos, sin)))
    base = SimpleNamespace(config=SimpleNamespace(num_attention_heads=g, num_key_value_heads=1), layer_idx=0,
                           head_dim=d, scaling=cfg.scaling, q_proj=None, k_proj=None, v_proj=None, o_proj=None)
    attn = ref_attn.RDAttention(base, **cfg.attn_kwargs())
    with torch.inference_mode():
        idx_ref, t_routes = timed(lambda: attn.routes(qr, kr))
        o_ref, t_attn = timed(lambda: bigger_bird_flash_ref(
            qr[0, :heads, n - rows:], kr[0], v[0], idx_ref[:heads], front=cfg.sink, window=cfg.window,
            num_heads=heads, kv_groups=heads, scale=cfg.scaling, head_chunk=1))
    res["reference_s"] = {"rope": t_rope, "routes": t_routes, "attention": t_attn,
                          "total": t_rope + t_routes + t_attn}

    # numpy restatement (the parity oracle)
    f = lambda t: t.numpy()  # noqa: E731
    c, s = f(cos[0]), f(sin[0])
    (qn, kn), t_rope = timed(lambda: (orc.rope(f(q[0]), c, s, "f32"), orc.rope(f(k[0]), c, s, "f32")))
    idx_port, t_routes = timed(lambda: orc.routes(qn, kn, scaling=cfg.scaling, sink=cfg.sink, window=cfg.window,
                                                  vertical=cfg.vertical, n_route=cfg.n_route, dtype="f32"))
    o_port, t_attn = timed(lambda: orc.flash(qn[:heads, n - rows:], kn, f(v[0]), idx_port[:heads],
                                             front=cfg.sink, window=cfg.window, num_heads=heads, kv_groups=heads,
                                             scale=cfg.scaling))
    res["numpy_port_s"] = {"rope": t_rope, "routes": t_routes, "attention": t_attn,
                           "total": t_rope + t_routes + t_attn}
    # torch restatement (what bench.py times)
    qt, t_rope = timed(lambda: (tp.rope(q[0], cos[0], sin[0]), tp.rope(k[0], cos[0], sin[0])))
    qt, kt = qt
    idx_t, t_routes = timed(lambda: tp.routes(qt, kt, scaling=cfg.scaling, sink=cfg.sink, window=cfg.window,
                                              vertical=cfg.vertical, n_route=cfg.n_route))
    qs = torch.arange(n - rows, n)
    o_t, t_attn = timed(lambda: tp.attend_rows(qt[:heads][:, qs], qs, kt, v[0], idx_t, heads=list(range(heads)),
                                               kv_groups=g, scaling=cfg.scaling, sink=cfg.sink,
                                               window=cfg.window, exact_tail=0))
    res["torch_port_s"] = {"rope": t_rope, "routes": t_routes, "attention": t_attn,
                           "total": t_rope + t_routes + t_attn}
    res["reference_s_over_torch_port_s"] = res["reference_s"]["total"] / res["torch_port_s"]["total"]
    res["reference_s_over_numpy_port_s"] = res["reference_s"]["total"] / res["numpy_port_s"]["total"]
    res["torch_port_routes_identical"] = all(set(idx_t[h].tolist()) == set(np.asarray(idx_ref[h]).tolist())
                                             for h in range(g))
    res["torch_port_attention_max_abs_diff"] = float(np.abs(o_ref.numpy() - o_t.numpy()).max())
    same_routes = all(set(np.asarray(idx_ref[h]).tolist()) == set(np.asarray(idx_port[h]).tolist())
                      for h in range(g))
    res["numpy_port_routes_identical"] = bool(same_routes)
    res["numpy_port_attention_max_abs_diff"] = float(np.abs(o_ref.numpy() - o_port).max())
    res["cpu"] = next((line.split(":", 1)[1].strip() for line in open("/proc/cpuinfo")
                       if line.startswith("model name")), "unknown")
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
