"""Host logic of bench.py that runs without a GPU: the per-rank share option, the scope of the main
kernel's DRAM-traffic figure, the CPU description and the CPU leg."""
import pytest

import bench
from utmist_bigger_bird_b200.workload import CONFIGS


def test_kv_shard_defaults_to_the_launch():
    assert bench.parse_kv_shard(None, 3, 8) == (3, 8)
    assert bench.parse_kv_shard("", 0, 1) == (0, 1)


def test_kv_shard_parses_one_ranks_share():
    assert bench.parse_kv_shard("7/8", 0, 1) == (7, 8)
    assert bench.parse_kv_shard("0/2", 0, 1) == (0, 2)


@pytest.mark.parametrize("spec,world", [("8/8", 1), ("-1/8", 1), ("a/b", 1), ("3", 1), ("1/2", 2)])
def test_kv_shard_rejects_bad_specs(spec, world):
    with pytest.raises(SystemExit):
        bench.parse_kv_shard(spec, 0, world)


def test_traffic_only_for_the_captured_kernel_and_config(monkeypatch):
    """The committed ncu figure applies only to config 2 and only to the kernel sources it was
    captured on; a rank's share is scaled by its KV heads."""
    cfg2 = CONFIGS["config2"]
    monkeypatch.setitem(bench.MAIN_TRAFFIC, "sources_sha256", "abc")
    monkeypatch.setitem(bench.MAIN_TRAFFIC, "bytes_per_launch", 8.0e9)
    monkeypatch.setitem(bench.MAIN_TRAFFIC, "capture", "test")
    t, src = bench.main_traffic(cfg2, cfg2.kv_heads, sha="abc")
    assert t == 8.0e9 and "config2" in src
    t, src = bench.main_traffic(cfg2, 1, sha="abc")
    assert t == pytest.approx(1.0e9) and "scaled to 1 of 8" in src
    t, src = bench.main_traffic(cfg2, 8, sha="other")
    assert t is None and "current kernel sources" in src
    assert bench.main_traffic(CONFIGS["config5"], 1, sha="abc")[0] is None
    assert bench.main_traffic(CONFIGS["sweep_n65536_w16384"], 8, sha="abc")[0] is None


def test_sources_hash_is_stable():
    assert bench.sources_sha256() == bench.sources_sha256() and len(bench.sources_sha256()) == 16


def test_cpu_model_is_named():
    assert isinstance(bench.cpu_model(), str) and bench.cpu_model()


def test_cpu_leg_runs_and_counts_flops():
    """The CPU leg (the torch restatement that --impl reference and cpu_baseline time) on config 1:
    it runs on the CPU and reports positive seconds and FLOPs."""
    dt, flops = bench.cpu_sample(CONFIGS["config1"], rows_per_head=12)
    assert dt > 0 and flops > 0
