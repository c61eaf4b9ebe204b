#!/usr/bin/env python
"""Benchmark of one Bigger Bird v3 sparse-prefill attention layer on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config config2] [--impl ours|reference]

A step is one sparse-prefill layer: in-place RoPE on Q/K, routing (last 64 queries score every
key, top-512 per query head), the sink + window + routed main pass, and the exact causal tail,
all through the one-call C entry point ``bb_sparse_prefill``. The default workload is BASELINE
config 2 (n = 131072, bf16, 32 Q / 8 KV heads, d = 128, sink 64, window 16384, vertical 512,
tail 256). ``value`` is effective TFLOP/s: algorithmic FLOPs (4 * d * attended query-key pairs,
counted exactly from the step's routes) over the max-over-ranks device time. With N > 1 the layer's
KV heads are split across ranks (rank p owns KV heads [p*8/N, (p+1)*8/N) and their query heads);
the single-layer path has no cross-rank data exchange, so the timing reductions are the only
collectives.

``--impl reference`` times the reference algorithm's CPU path (the numpy restatement under
``oracle/``; the reference itself is Python and does not travel) on the host cores over a bounded
sample of the same workload, and prints the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from utmist_bigger_bird_b200.workload import CONFIGS, make_layer  # noqa: E402

PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
KERNEL_SOURCES = [ROOT / "utmist_bigger_bird_b200" / "csrc" / f for f in ("flash_tc.cu", "tc_common.cuh", "bb_common.cuh")]
# DRAM traffic of the main-pass kernel, from one ncu capture (dram__bytes_read.sum +
# dram__bytes_write.sum) of config 2's main pass, and the hash of the kernel sources it was taken
# on. When the sources change the figure no longer describes the kernel and the bench reports null.
MAIN_TRAFFIC = {"sources_sha256": "21f28c8d45ed1775", "bytes_per_launch": 644.84e6 * (131072 - 256) / (32768 - 256),
                "capture": "dram__bytes_read.sum + dram__bytes_write.sum of the main pass of "
                           "`bench.py --config sweep_n32768_w16384 --part layer` (644.8 MB), scaled by main-pass "
                           "query rows x4.024"}


def sources_sha256():
    import hashlib
    h = hashlib.sha256()
    for f in KERNEL_SOURCES:
        h.update(f.read_bytes())
    return h.hexdigest()[:16]


def peaks():
    if PEAKS_FILE.exists():
        return json.loads(PEAKS_FILE.read_text()), "measured"
    return FALLBACK, "fallback"


def parse_kv_shard(spec, rank, world):
    """(rank, ranks) of the KV-head split whose share this process times: the launch's own
    (RANK, WORLD_SIZE), or R/N from --kv-shard, one rank's share of an N-GPU run alone on this GPU
    (no process group, so it cannot be combined with torchrun)."""
    if not spec:
        return rank, world
    if world > 1:
        raise SystemExit("--kv-shard times one rank's share on one GPU: launch it without torchrun")
    try:
        r, n = (int(x) for x in spec.split("/"))
    except ValueError:
        raise SystemExit(f"--kv-shard wants R/N, got {spec!r}") from None
    if not 0 <= r < n:
        raise SystemExit("--kv-shard R/N needs 0 <= R < N")
    return r, n


def main_traffic(cfg, kv_heads_here, sha=None):
    """(DRAM bytes per main-pass launch, where the figure comes from), or (None, why not). The
    committed ncu figure is for config 2's full launch on the kernel sources whose hash it carries; a
    launch over some of its KV heads moves that share of it (each KV head's K/V and its query heads'
    Q and output); other configs, and changed sources, have no capture."""
    if cfg.name != "config2":
        return None, f"no ncu capture of {cfg.name}"
    sha = sha or sources_sha256()
    if MAIN_TRAFFIC["bytes_per_launch"] is None or MAIN_TRAFFIC["sources_sha256"] != sha:
        return None, f"no ncu capture of the current kernel sources ({sha})"
    src = f"ncu dram bytes of the config2 main-pass launch ({MAIN_TRAFFIC['capture']}; sources {sha})"
    if kv_heads_here != cfg.kv_heads:
        src += f", scaled to {kv_heads_here} of {cfg.kv_heads} KV heads"
    return MAIN_TRAFFIC["bytes_per_launch"] * kv_heads_here / cfg.kv_heads, src


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


# ----------------------------------------------------------------------------- FLOP counting

def attended_pairs(n, sink, window, exact_tail, idx):
    """Query-key pairs the layer attends (BASELINE section 2 formula), per query head, exact:
    sink and window keys of the main rows, routed keys beyond each query's window, and the dense
    causal tail rows. ``idx`` [heads, budget] are the step's routes."""
    r = min(exact_tail, n)
    m = n - r
    q = np.arange(m, dtype=np.int64)
    sink_p = np.minimum(sink, q + 1).sum()
    lo = np.maximum(sink, q - window + 1)
    win_p = np.maximum(0, q - lo + 1).sum()
    tail_p = (np.arange(m, n, dtype=np.int64) + 1).sum()
    idx = np.asarray(idx, dtype=np.int64)
    routed = np.where(idx >= sink, np.maximum(0, m - (idx + window)), 0).sum(axis=-1)
    return (sink_p + win_p + tail_p) * idx.shape[0] + routed.sum(), (sink_p + win_p, routed, tail_p)


def main_pass_pairs(n, sink, window, exact_tail, idx):
    r = min(exact_tail, n)
    m = n - r
    q = np.arange(m, dtype=np.int64)
    base = np.minimum(sink, q + 1).sum() + np.maximum(0, q - np.maximum(sink, q - window + 1) + 1).sum()
    idx = np.asarray(idx, dtype=np.int64)
    routed = np.where(idx >= sink, np.maximum(0, m - (idx + window)), 0).sum()
    return base * idx.shape[0] + routed


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.proc = None
        self.path = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.gpu = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            self.gpu = str(device.index or 0)

    def __enter__(self):
        try:
            import tempfile
            self.path = tempfile.NamedTemporaryFile(prefix="bb_clocks_", suffix=".csv", delete=False).name
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), float(parts[2]), parts[3:]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3][1:5]) if v.lower() == "active"})
        loaded = [r for r in rows if r[2] > 200.0] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": reasons}


# ----------------------------------------------------------------------------- reference arm

def cpu_sample(cfg, kv_head=0, heads=2, rows_per_head=48):
    """One bounded CPU sample of the workload with the torch restatement of the reference's CPU path
    (``oracle/torch_port.py``: fp32, all host threads, the reference's own CPU contract): RoPE of one
    KV head's query heads and K, their routes over all n keys, and ``rows_per_head`` spread query rows
    (incl. tail rows) of ``heads`` query heads. Returns (seconds, algorithmic FLOPs of the sample)."""
    from oracle import torch_port as tp
    q, k, v, cos, sin, _ = make_layer(cfg, kv_heads=[kv_head])
    q, k, v, cos, sin = (t[0].float() for t in (q, k, v, cos, sin))
    g = cfg.heads // cfg.kv_heads
    n = cfg.n
    rows = np.unique(np.concatenate([np.linspace(0, n - 1 - cfg.exact_tail, rows_per_head - 8).astype(np.int64),
                                     np.arange(n - 8, n)]))
    t0 = time.perf_counter()
    qr, kr = tp.rope(q, cos, sin), tp.rope(k, cos, sin)
    idx_t = tp.routes(qr, kr, scaling=cfg.scaling, sink=cfg.sink, window=cfg.window, vertical=cfg.vertical,
                      n_route=cfg.n_route)
    tp.attend_rows(qr[:heads][:, rows], torch.from_numpy(rows), kr, v, idx_t, heads=np.arange(heads), kv_groups=g,
                   scaling=cfg.scaling, sink=cfg.sink, window=cfg.window, exact_tail=cfg.exact_tail)
    dt = time.perf_counter() - t0
    idx = idx_t.numpy()
    # FLOPs of the sample: routing (2 QK^T passes of g*r rows over n keys) + attended pairs of the rows
    route_flops = 2 * 2 * g * cfg.n_route * n * cfg.head_dim
    r = min(cfg.exact_tail, n)
    pairs = 0
    for h in range(heads):
        for qp in rows:
            if qp >= n - r:
                pairs += qp + 1
            else:
                lo = max(cfg.sink, qp - cfg.window + 1)
                pairs += min(cfg.sink, qp + 1) + max(0, qp - lo + 1)
                pairs += int(((idx[h] >= cfg.sink) & (idx[h] <= qp - cfg.window)).sum())
    return dt, 4.0 * cfg.head_dim * pairs + route_flops


# The reference's own CPU path measured against this CPU leg (oracle/torch_port.py) on one bounded
# config-2 sample in the build container (8 threads, Intel Xeon): `oracle/time_reference_cpu.py`
# (it imports the reference, which does not travel to the GPU box). Routes identical, attention
# identical (max |diff| 0); the reference took 0.360 s, the torch restatement 0.393 s (the numpy
# parity oracle 1.91 s).
REFERENCE_CPU_CALIBRATION = {"reference_s_over_port_s": 0.915, "measured_by": "oracle/time_reference_cpu.py",
                             "note": "the reference's own CPU path ran the same sample in 0.92x this leg's time"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    for _ in range(args.warmup):
        cpu_sample(cfg, rows_per_head=16)
    times, flops = [], 0.0
    for i in range(args.steps):
        dt, fl = cpu_sample(cfg, kv_head=i % cfg.kv_heads)
        times.append(dt)
        flops += fl
    total = sum(times)
    value = flops / total / 1e12
    sample = (f"per step: RoPE + routes of 1 KV head over all {cfg.n} keys + 48 query rows x 2 query heads of "
              f"{cfg.name} (torch restatement of the reference's CPU path, fp32 on bf16-valued inputs)")
    line = {"impl": "reference", "metric": "eff_tflops_sparse_prefill_layer", "value": value, "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": cfg.name, "n": cfg.n, "sample": "bounded CPU sample (see cpu_baseline)"},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "cpu": cpu_model(), "kind": "port",
                             "dtype": "fp32", "sample": sample, "calibration": REFERENCE_CPU_CALIBRATION},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- our arm

def event_time(fn, reps, stream):
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(reps):
        fn()
    e.record(stream)
    e.synchronize()
    return s.elapsed_time(e) / reps


def flushed_time(fn, reps, stream, scrub):
    """Mean device time of fn over reps calls, each after a read of ``scrub`` (larger than L2) so
    that a working set smaller than L2 is read from HBM every call; the scrub is outside the timing.
    A read, not a write: a written scrub would leave L2 full of dirty lines whose write-back the
    timed call would pay for.
    fn is captured once into a CUDA graph and replayed, the way a serving loop runs these short
    calls, so that the host's Python time does not open gaps inside the timed region."""
    side = torch.cuda.Stream(stream.device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        fn()
        fn()
    stream.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        fn()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for s, e in ev:
        scrub.sum()
        s.record(stream)
        graph.replay()
        e.record(stream)
    ev[-1][1].synchronize()
    del graph
    return sum(s.elapsed_time(e) for s, e in ev) / reps


def side_paths(cfg, qr, kr, v, idx, qpos, budget, dev, stream, reps, pk, parts=("evict", "decode")):
    """KV eviction and decode on this rank's post-RoPE cache (kr, v) and prefill routes (idx);
    returns their JSON objects (None for a part not asked for)."""
    from utmist_bigger_bird_b200 import _ops
    per, H, n, d = kr.shape[1], qr.shape[1], kr.shape[2], kr.shape[3]
    g = H // per
    scrub = torch.ones(64 << 20, device=dev, dtype=torch.float32)  # 256 MB, twice L2
    evict_line = decode_line = None
    w = min(cfg.window, n - cfg.sink)  # the window the module uses when it covers the whole prompt
    if "evict" in parts:
        # ---- KV eviction after the prefill (RDAttention.evict, default policy): priorities from the
        # step's routes and routing column scores, the g*budget best middle keys, K/V gather. HBM-bound;
        # algorithmic bytes = the column scores read + the kept K and V rows read and written. Its working
        # set (and the sparse decode's) fits in L2, so these are timed with L2 scrubbed before each call.
        col_buf = torch.empty(H, n, device=dev, dtype=torch.float32)
        _ops.routes_(qr[0], kr[0], qpos, sink=cfg.sink, window=cfg.window, budget=budget, scaling=cfg.scaling,
                     out_col=col_buf)
        keep = min(g * budget, n - cfg.sink - w)

        def evict():
            _ops.kv_evict_(idx, col_buf, kr[0], v[0], sink=cfg.sink, window=w, keep=keep)

        evict()
        torch.cuda.synchronize(dev)
        evict_ms = flushed_time(evict, reps, stream, scrub)
        kept_rows = cfg.sink + keep + w
        evict_bytes = H * n * 4 + 2 * 2 * per * kept_rows * d * 2
        evict_gbs = evict_bytes / (evict_ms * 1e-3) / 1e9
        evict_line = {"bound": "hbm", "ms": evict_ms, "kept_rows_per_kv_head": kept_rows, "achieved_gbs": evict_gbs,
                      "peak_gbs": pk["hbm_gbs"], "frac": evict_gbs / pk["hbm_gbs"], "algorithmic_bytes": evict_bytes}

    if "decode" in parts:
        # ---- decode of one new token per head over this rank's cache (n keys): decode routing
        # (pooled probabilities + top-budget per KV head), sparse split-K decoding over front | window |
        # pooled routes, and dense flash-decoding over all n keys. HBM-bound; algorithmic bytes = the
        # K (and V) rows each one must read.
        from utmist_bigger_bird_b200 import bigger_bird_decode, bigger_bird_route
        qd = qr[0, :, n - 1].contiguous()
        droute = lambda: bigger_bird_route(qd, kr[0], budget, front=cfg.sink, window=w,  # noqa: E731
                                           scale=cfg.scaling)
        no_routes = torch.empty(per, 0, dtype=torch.int64, device=dev)
        didx = droute() if budget > 0 else no_routes
        dsparse = lambda: bigger_bird_decode(qd, kr[0], v[0], didx, front=cfg.sink, window=w,  # noqa: E731
                                             scale=cfg.scaling)
        ddense = lambda: bigger_bird_decode(qd, kr[0], v[0], no_routes, front=0, window=n,  # noqa: E731
                                            scale=cfg.scaling)
        for fn in (dsparse, ddense):
            fn()
        torch.cuda.synchronize(dev)
        dec = {}
        for name, fn, nbytes in (("route", droute, per * n * d * 2),
                                 ("sparse", dsparse, 2 * per * (cfg.sink + w + budget) * d * 2),
                                 ("dense", ddense, 2 * per * n * d * 2)):
            if name == "route" and budget == 0:
                continue  # nothing to route: front and window cover the cache
            t = flushed_time(fn, reps * 3, stream, scrub)
            gbs = nbytes / (t * 1e-3) / 1e9
            dec[name] = {"ms": t, "algorithmic_bytes": nbytes, "achieved_gbs": gbs, "frac": gbs / pk["hbm_gbs"]}
        decode_line = dict(dec, bound="hbm", peak_gbs=pk["hbm_gbs"],
                           config=f"one token per head over the rank's {n}-key cache: route = pooled probabilities + "
                                  f"top-{budget} per KV head; sparse = front {cfg.sink} | window {w} | "
                                  f"{budget} pooled routes; dense = all keys")
    return evict_line, decode_line


def host_link(q_h, k_h, v_h, cos_h, sin_h, out_h, buf, s_in, s_out, steps, dev, world, local):
    """The host link alone: the e2e step's H2D copies (pinned q/k/v/cos/sin) on one stream and its
    D2H copy of the output on another, concurrently, with no compute, on every rank at once (the
    ranks share the host's links). Returns the per-step time (max over ranks) and rates; the e2e
    step cannot be faster than this."""
    import torch.distributed as dist
    from utmist_bigger_bird_b200.sharding import reduce_step
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize(dev)
    t0 = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    t1 = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    start = torch.cuda.Event()
    start.record(s_in)
    s_out.wait_event(start)
    t0[0].record(s_in)
    t0[1].record(s_out)
    for _ in range(steps):
        with torch.cuda.stream(s_in):
            for name, src in (("q", q_h), ("k", k_h), ("v", v_h), ("cos", cos_h), ("sin", sin_h)):
                buf[name].copy_(src, non_blocking=True)
        with torch.cuda.stream(s_out):
            out_h.copy_(buf["out"].permute(1, 0, 2), non_blocking=True)
    t1[0].record(s_in)
    t1[1].record(s_out)
    torch.cuda.synchronize(dev)
    h2d_ms = t0[0].elapsed_time(t1[0]) / steps
    d2h_ms = t0[1].elapsed_time(t1[1]) / steps
    ms, _ = reduce_step(max(h2d_ms, d2h_ms), 0.0, dev)
    h2d = sum(t.numel() * t.element_size() for t in (q_h, k_h, v_h, cos_h, sin_h))
    d2h = out_h.numel() * out_h.element_size()
    return {"ms_per_step": ms, "h2d_gbs": h2d / (h2d_ms * 1e-3) / 1e9, "d2h_gbs": d2h / (d2h_ms * 1e-3) / 1e9,
            "note": "H2D and D2H of one e2e step's bytes concurrently on this rank, no compute, all ranks at once; "
                    "ms_per_step = max over ranks of the slower direction"}


def collectives(n, w_local, hidden, dev, stream, world, local, reps=5):
    """The whole-model step's exchanges for one layer at this layer's size (n tokens), on the
    launch's process group: the all-gather of the ranks' head outputs [n, w_local] bf16 before a
    replicated o_proj (``sharding.GatheredOProj``, with its projection), and the all-reduce of
    [n, hidden] bf16 after the row-parallel o_proj or MLP down projection
    (``sharding.RowParallelLinear``). Device time with CUDA events, max over ranks; bus rates
    use NCCL's conventions ((P-1)/P of the gathered bytes; 2(P-1)/P of the reduced bytes)."""
    import torch.distributed as dist
    from utmist_bigger_bird_b200.sharding import GatheredOProj, reduce_step
    x = torch.randn(n, w_local, device=dev, dtype=torch.bfloat16)
    gathered = torch.empty(world * n, w_local, device=dev, dtype=torch.bfloat16)
    red = torch.randn(n, hidden, device=dev, dtype=torch.bfloat16)
    o_proj = torch.nn.Linear(world * w_local, hidden, bias=False, device=dev, dtype=torch.bfloat16)
    gproj = GatheredOProj(o_proj, world)
    ops = {"all_gather": lambda: dist.all_gather_into_tensor(gathered, x),
           "all_reduce": lambda: dist.all_reduce(red),
           "gathered_o_proj": lambda: gproj(x)}
    out = {}
    for name, fn in ops.items():
        fn()
        dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)
        ms, _ = reduce_step(event_time(fn, reps, stream), 0.0, dev)
        out[name] = {"ms": ms}
    frac = (world - 1) / world
    ag_bytes = world * n * w_local * 2
    ar_bytes = n * hidden * 2
    out["all_gather"].update(bytes=ag_bytes, bus_gbs=ag_bytes * frac / (out["all_gather"]["ms"] * 1e-3) / 1e9)
    out["all_reduce"].update(bytes=ar_bytes, bus_gbs=2 * ar_bytes * frac / (out["all_reduce"]["ms"] * 1e-3) / 1e9)
    out["gathered_o_proj"].update(flops=2.0 * n * world * w_local * hidden)
    out["note"] = (f"one layer's exchange at n={n}: all-gather of [n, {w_local}] bf16 per rank (before the replicated "
                   f"o_proj), all-reduce of [n, {hidden}] bf16 (after a row-parallel o_proj or MLP); NCCL over NVLink")
    del x, gathered, red, o_proj, gproj
    torch.cuda.empty_cache()
    return out


def run_ours(args):
    import torch.distributed as dist

    from utmist_bigger_bird_b200 import _lib, _ops
    from utmist_bigger_bird_b200.sharding import kv_head_shard, reduce_step
    from utmist_bigger_bird_b200.attention import route_query_positions, vertical_budget

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    cfg = CONFIGS[args.config]
    shard_r, shard_n = parse_kv_shard(args.kv_shard, rank, world)
    kv_heads = kv_head_shard(shard_r, shard_n, cfg.kv_heads)
    per = len(kv_heads)
    g = cfg.heads // cfg.kv_heads
    H = per * g
    n, d = cfg.n, cfg.head_dim
    q_h, k_h, v_h, cos_h, sin_h, _ = make_layer(cfg, kv_heads=kv_heads)
    q_h, k_h, v_h, cos_h, sin_h = (t.pin_memory() for t in (q_h, k_h, v_h, cos_h, sin_h))
    q0, k0, v, cos, sin = (t.to(dev) for t in (q_h, k_h, v_h, cos_h, sin_h))
    q, k = q0.clone(), k0.clone()
    budget = min(vertical_budget(n, cfg.vertical, 0.0), max(0, n - cfg.sink - cfg.window))
    qpos = route_query_positions(n, min(cfg.n_route, n), "last", cfg.sink, cfg.window, dev)
    out = torch.empty((n, H, d), device=dev, dtype=q.dtype).permute(1, 0, 2)
    idx = torch.empty((H, budget), device=dev, dtype=torch.int32)
    stream = torch.cuda.current_stream(dev)
    L = _lib.lib()

    def step():
        _ops.sparse_prefill_(q[0], k[0], v[0], qpos, out, idx, sink=cfg.sink, window=cfg.window, budget=budget,
                             exact_tail=cfg.exact_tail, scaling=cfg.scaling, cos=cos[0], sin=sin[0])

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def restore():
        # The step applies RoPE to q/k in place: give every step the stated (pre-RoPE) inputs.
        q.copy_(q0)
        k.copy_(k0)

    def timed_steps(steps):
        """Mean device time of ``step`` over ``steps`` steps, each on freshly restored inputs; the
        restoring copies sit between the timed events."""
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for s_ev, e_ev in evs:
            restore()
            s_ev.record(stream)
            step()
            e_ev.record(stream)
        evs[-1][1].synchronize()
        return sum(s_ev.elapsed_time(e_ev) for s_ev, e_ev in evs) / steps

    for _ in range(max(args.warmup, 3)):
        restore()
        step()
    barrier()
    launches0 = L.bb_kernel_launches()
    with ClockSampler(dev) as clocks:
        barrier()
        ms = timed_steps(args.steps)
        barrier()
    launches = L.bb_kernel_launches() - launches0
    clock = clocks.summary()

    # exact FLOPs of this rank's step from its routes (routes are input-determined: identical every step)
    pairs, _ = attended_pairs(n, cfg.sink, cfg.window, cfg.exact_tail, idx.cpu().numpy())
    flops = 4.0 * d * float(pairs)
    ms_max, flops_all = reduce_step(ms, flops, dev)
    value = flops_all / (ms_max * 1e-3) / 1e12

    # ---- dominant kernel (main sparse pass) and routing, timed alone on this rank
    qr, kr = q0.clone(), k0.clone()
    _ops.rope_inplace_(qr, cos, sin)
    _ops.rope_inplace_(kr, cos, sin)
    r_tail = min(cfg.exact_tail, n)
    routed = idx.view(H, 1, -1)
    chunk = 1 << (n - 1).bit_length()

    def main_pass():
        _ops.flash_(qr[0], kr[0], v[0], routed, out, front=cfg.sink, window=cfg.window, num_heads=H,
                    kv_groups=g, route_chunk=chunk, scale=cfg.scaling, row_begin=0, row_end=n - r_tail)

    def routing():
        _ops.routes_(qr[0], kr[0], qpos, sink=cfg.sink, window=cfg.window, budget=budget, scaling=cfg.scaling)

    def tail():
        none = idx.view(H, 1, -1)[:, :, :0]
        _ops.flash_(qr[0][:, n - r_tail:], kr[0], v[0], none, out[:, n - r_tail:], front=0, window=n,
                    num_heads=H, kv_groups=g, route_chunk=chunk, scale=cfg.scaling)

    for fn in (main_pass, routing, tail):
        fn()
    torch.cuda.synchronize(dev)
    reps = max(3, min(args.steps, 10))
    main_ms = event_time(main_pass, reps, stream)
    route_ms = event_time(routing, reps * 3, stream)
    tail_ms = event_time(tail, reps, stream)
    main_flops = 4.0 * d * float(main_pass_pairs(n, cfg.sink, cfg.window, cfg.exact_tail, idx.cpu().numpy()))
    pk, pk_kind = peaks()
    achieved = main_flops / (main_ms * 1e-3) / 1e12
    traffic, traffic_src = main_traffic(cfg, per)
    route_bytes = per * n * d * 2 + H * min(cfg.n_route, n) * d * 2 + H * budget * 4
    route_gbs = route_bytes / (route_ms * 1e-3) / 1e9
    if args.part == "layer":
        # The layer and its kernels only (no side paths, comparators, e2e or CPU sample): the
        # committed command the ncu captures of these kernels run.
        main_max, _ = reduce_step(main_ms, 0.0, dev)
        if world > 1:
            dist.barrier(device_ids=[local])
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"part": "layer", "workload": cfg.name, "n_gpus": world, "ms_per_step": ms_max,
                              "eff_tflops": value, "main_ms": main_max, "main_tflops": achieved,
                              "main_frac": achieved / pk["bf16_tflops"], "routing_ms": route_ms,
                              "exact_tail_ms": tail_ms, "gpu_launches": int(launches), "clocks": clock}),
                  flush=True)
        return

    evict_line, decode_line = side_paths(cfg, qr, kr, v, idx, qpos, budget, dev, stream, reps, pk)

    # ---- dense causal SDPA on the same inputs (the reference's comparator, attn_bench.py:47)
    import torch.nn.functional as F
    dense = lambda: F.scaled_dot_product_attention(qr, kr, v, is_causal=True, scale=cfg.scaling,  # noqa: E731
                                                   enable_gqa=True)
    dense()
    torch.cuda.synchronize(dev)
    dense_ms = event_time(dense, max(2, reps // 2), stream)

    # ---- end to end through the C entry point with host buffers: every step copies its q/k/v/cos/sin
    # from pinned host memory and its output back. Steps are pipelined the way a serving loop runs
    # them: two device buffer sets; H2D of step i+1 and D2H of step i-1 overlap the compute of step i
    # (copy-in stream, compute stream, copy-out stream, ordered by events).
    del qr, kr
    torch.cuda.empty_cache()
    h2d = sum(t.numel() * t.element_size() for t in (q_h, k_h, v_h, cos_h, sin_h))
    out_h = [torch.empty((n, H, d), dtype=q.dtype).pin_memory() for _ in range(2)]
    d2h = out_h[0].numel() * out_h[0].element_size()
    bufs = [dict(q=torch.empty_like(q0), k=torch.empty_like(k0), v=torch.empty_like(v),
                 cos=torch.empty_like(cos), sin=torch.empty_like(sin),
                 out=torch.empty((n, H, d), device=dev, dtype=q.dtype).permute(1, 0, 2),
                 idx=torch.empty((H, budget), device=dev, dtype=torch.int32)) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready = [ev() for _ in range(2)]
    computed = [ev() for _ in range(2)]
    drained = [ev() for _ in range(2)]
    inputs_free = [ev() for _ in range(2)]
    for e in drained + inputs_free:
        e.record(stream)

    def e2e_run(steps):
        for i in range(steps):
            b = bufs[i % 2]
            with torch.cuda.stream(s_in):
                s_in.wait_event(inputs_free[i % 2])
                for name, src in (("q", q_h), ("k", k_h), ("v", v_h), ("cos", cos_h), ("sin", sin_h)):
                    b[name].copy_(src, non_blocking=True)
                in_ready[i % 2].record(s_in)
            stream.wait_event(in_ready[i % 2])
            stream.wait_event(drained[i % 2])
            _ops.sparse_prefill_(b["q"][0], b["k"][0], b["v"][0], qpos, b["out"], b["idx"], sink=cfg.sink,
                                 window=cfg.window, budget=budget, exact_tail=cfg.exact_tail, scaling=cfg.scaling,
                                 cos=b["cos"][0], sin=b["sin"][0])
            computed[i % 2].record(stream)
            inputs_free[i % 2].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(computed[i % 2])
                out_h[i % 2].copy_(b["out"].permute(1, 0, 2), non_blocking=True)
                drained[i % 2].record(s_out)

    e2e_run(2)
    torch.cuda.synchronize(dev)
    barrier()
    # The pipeline's first H2D and last D2H are not overlapped with compute; over K steps they cost
    # (H2D + D2H) / K per step, so the run uses the same K as the timed device steps (at least 5).
    e2e_steps = max(5, args.steps)
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record(s_in)
    e2e_run(e2e_steps)
    s_in.wait_stream(s_out)
    t_end.record(s_in)
    t_end.synchronize()
    e2e_ms = t_start.elapsed_time(t_end) / e2e_steps
    e2e_max, _ = reduce_step(e2e_ms, 0.0, dev)
    e2e_value = flops_all / (e2e_max * 1e-3) / 1e12
    link = host_link(q_h, k_h, v_h, cos_h, sin_h, out_h[0], bufs[0], s_in, s_out, e2e_steps, dev, world, local)
    link["e2e_frac"] = link["ms_per_step"] / e2e_max
    del bufs, out_h
    torch.cuda.empty_cache()
    coll = collectives(n, H * d, cfg.heads * d, dev, stream, world, local) if world > 1 else None

    # ---- CPU baseline (rank 0, N = 1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        dt, fl = cpu_sample(cfg)
        cpu = {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "cpu": cpu_model(), "kind": "port",
               "dtype": "fp32", "calibration": REFERENCE_CPU_CALIBRATION,
               "sample": f"RoPE + routes of KV head 0 over all {n} keys + 48 spread/tail query rows x 2 query "
                         f"heads, torch restatement of the reference's CPU path ({dt:.2f} s)"}

    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return
    metric = "eff_tflops_sparse_prefill_layer" + ("_rank_share" if args.kv_shard else "")
    line = {
        "metric": metric, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "kv_shard": args.kv_shard,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms_max, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{cfg.name}: one sparse-prefill attention layer (RoPE + routes + main + exact tail)",
                   "n": n, "q_heads": cfg.heads, "kv_heads": cfg.kv_heads, "head_dim": d, "sink": cfg.sink,
                   "window": cfg.window, "vertical": cfg.vertical, "exact_tail": cfg.exact_tail,
                   "n_route": cfg.n_route,
                   "parallelism": (f"kv-head shards x{world}" if not args.kv_shard else
                                   f"kv-head shard {shard_r} of {shard_n} alone on 1 GPU (the per-rank step of "
                                   f"a {shard_n}-GPU run)"),
                   "l2": "inputs (%.2f GB per rank) exceed L2; no flush" % ((q.numel() + k.numel() + v.numel()) * 2 / 1e9),
                   "flops_per_step": flops_all},
        "roofline": {"bound": "tensor", "kernel": "flash main pass (sink+window+routed)", "achieved": achieved,
                     "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": achieved / pk["bf16_tflops"],
                     "peak_kind": f"{pk_kind} bf16 burst", "traffic": traffic, "traffic_source": traffic_src,
                     "launch_ms": main_ms,
                     "flops_per_launch": main_flops},
        "routing": {"bound": "hbm", "ms": route_ms, "achieved_gbs": route_gbs, "peak_gbs": pk["hbm_gbs"],
                    "frac": route_gbs / pk["hbm_gbs"], "algorithmic_bytes": route_bytes},
        "exact_tail_ms": tail_ms,
        "kv_evict": evict_line,
        "decode": decode_line,
        "dense_sdpa": {"ms": dense_ms, "speedup_sparse_vs_dense": dense_ms / ms},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "ms": e2e_max, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "note": "pipelined serving loop: H2D of step i+1 and D2H of step i-1 overlap step i; "
                        "the first H2D and last D2H are inside the timed region",
                "host_link": link},
        "collectives": coll,
        "gpu_launches": int(launches),
        "clocks": clock,
        "gpu": torch.cuda.get_device_name(dev),
    }
    print(json.dumps(line), flush=True)


def run_part(args):
    """One side path alone on one GPU (``--part decode`` or ``--part evict``), at the config's full
    size: the layer's post-RoPE cache and prefill routes, then that part's timing as one JSON line.
    Used for focused profiling of those kernels."""
    from utmist_bigger_bird_b200 import _ops
    from utmist_bigger_bird_b200.attention import route_query_positions, vertical_budget
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    n = cfg.n
    q, k, v, cos, sin, _ = (t.to(dev) for t in make_layer(cfg, kv_heads=list(range(cfg.kv_heads))))
    _ops.rope_inplace_(q, cos, sin)
    _ops.rope_inplace_(k, cos, sin)
    budget = min(vertical_budget(n, cfg.vertical, 0.0), max(0, n - cfg.sink - cfg.window))
    qpos = route_query_positions(n, min(cfg.n_route, n), "last", cfg.sink, cfg.window, dev)
    idx = _ops.routes_(q[0], k[0], qpos, sink=cfg.sink, window=cfg.window, budget=budget, scaling=cfg.scaling)
    pk, _ = peaks()
    stream = torch.cuda.current_stream(dev)
    reps = max(3, min(args.steps, 10))
    evict_line, decode_line = side_paths(cfg, q, k, v, idx, qpos, budget, dev, stream, reps, pk, parts=(args.part,))
    print(json.dumps({"part": args.part, "workload": cfg.name, "kv_evict": evict_line, "decode": decode_line}),
          flush=True)


def run_model(args):
    """Whole-model prefill (config 4): a random-init 32-layer Llama-3-8B over ``--model-tokens``
    token ids, KV cache kept, logits of the last position only. On one GPU: the stock Hugging Face
    model (dense SDPA, no memory savers), then the same weights with the sparse attention and the
    memory savers installed. Under torchrun (N GPUs): every rank holds the weights, attention is
    head-sharded (``shard_llama``: the rank's KV heads and their query heads) and either
    ``--model-shard gather`` (one NCCL all-gather a layer before a replicated o_proj, MLP replicated)
    or ``tensor`` (row-parallel o_proj, tensor-parallel MLP, two all-reduces a layer); norms
    replicated; the step time is the max over ranks.
    Prints one JSON line (rank 0)."""
    import torch.distributed as dist
    from transformers import DynamicCache
    from utmist_bigger_bird_b200 import (install, install_chunked_mlp, install_cpu_embedding, install_fused_rmsnorm,
                                         install_inplace_residual)
    from utmist_bigger_bird_b200.sharding import reduce_step, shard_llama
    from utmist_bigger_bird_b200.workload import make_llama
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    n = args.model_tokens
    model = make_llama(n_layers=args.model_layers, seed=2, device=dev)
    g = torch.Generator(device="cpu").manual_seed(2)
    ids = torch.randint(0, model.config.vocab_size, (1, n), generator=g).to(dev)
    stream = torch.cuda.current_stream(dev)
    attn = dict(sink=64, window=16384, vertical=512, exact_tail=256)

    def measure():
        def fwd():
            with torch.inference_mode():
                cache = DynamicCache(config=model.config)
                out = model(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1)
                return out.logits, cache

        logits, cache = fwd()  # warm-up
        del cache
        torch.cuda.synchronize(dev)
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats(dev)
        base = torch.cuda.memory_allocated(dev)
        times = []
        for _ in range(max(1, args.steps)):
            if world > 1:
                dist.barrier(device_ids=[local])
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            logits, cache = fwd()
            e.record(stream)
            e.synchronize()
            times.append(s.elapsed_time(e))
            del cache
        peak = torch.cuda.max_memory_allocated(dev) - base
        ms, _ = reduce_step(min(times), 0.0, dev)
        pk, _ = reduce_step(peak / 1e9, 0.0, dev)
        return {"ms": ms, "tokens_per_s": n / (ms * 1e-3), "peak_extra_gb_max_rank": pk,
                "weights_gb": base / 1e9}, logits.float()

    line = {"part": "model", "n_gpus": world,
            "workload": f"config4 model: random-init Llama-3-8B x{args.model_layers} layers, {n} tokens, KV cache "
                        f"kept, last-position logits" + (
                            f"; attention head-sharded over {world} GPUs, " + (
                                "all-gather before a replicated o_proj, MLP replicated" if args.model_shard == "gather"
                                else "row-parallel o_proj and tensor-parallel MLP (two all-reduces a layer)")
                            if world > 1 else "") + f"; RMSNorm {args.model_norm}",
            "gpu": torch.cuda.get_device_name(dev)}
    if world == 1:
        stock, lg_dense = measure()
        install(model, "vs", **attn)
        line["stock_hf_dense"] = stock
    else:
        shard_llama(model, rank, world, mode=args.model_shard, **attn)
    install_chunked_mlp(model, 8192)
    install_cpu_embedding(model)
    install_inplace_residual(model)
    if args.model_norm == "fused":
        install_fused_rmsnorm(model)
    ours, lg_sparse = measure()
    line["ours_sparse_savers"] = ours
    if world == 1:
        line["speedup"] = stock["ms"] / ours["ms"]
        line["peak_ratio"] = ours["peak_extra_gb_max_rank"] / max(stock["peak_extra_gb_max_rank"], 1e-9)
        line["next_token_dense"] = int(lg_dense[0, -1].argmax())
    line["next_token_sparse"] = int(lg_sparse[0, -1].argmax())
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--config", default="config2", choices=sorted(CONFIGS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    p.add_argument("--kv-shard", default=None, metavar="R/N",
                   help="time rank R's share of an N-way KV-head split alone on this one GPU (no process "
                        "group): the per-rank step of --gpus N, for a config whose whole layer needs more "
                        "GPUs (or memory) than one")
    p.add_argument("--part", default="all", choices=["all", "layer", "decode", "evict", "model"],
                   help="time one side path alone (1 GPU) instead of the full benchmark; 'layer' = the layer "
                        "steps and its kernels timed alone, nothing else; 'model' = the whole-model prefill "
                        "with and without the sparse path and memory savers")
    p.add_argument("--model-tokens", type=int, default=131072, help="--part model: prompt length")
    p.add_argument("--model-layers", type=int, default=32, help="--part model: decoder layers")
    p.add_argument("--model-norm", default="fused", choices=["fused", "chunked"],
                   help="--part model: fused RMSNorm kernel (within 2 ulp of HF) or HF's norm in chunks (exact)")
    p.add_argument("--model-shard", default="tensor", choices=["gather", "tensor"],
                   help="--part model under torchrun: all-gather before a replicated o_proj and MLP, or "
                        "row-parallel o_proj + tensor-parallel MLP")
    args = p.parse_args()
    if args.part == "model":
        run_model(args)
    elif args.part not in ("all", "layer"):
        run_part(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
