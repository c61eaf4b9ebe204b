"""Host logic of bench.py that runs without a GPU: the per-rank share option and the scope of the
main kernel's DRAM-traffic figure."""
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


def test_traffic_only_for_the_captured_config():
    full = bench.measured_traffic()
    assert full is not None and full > 0, "profiles/flash_main_config2.md carries the ncu figure"
    cfg2 = CONFIGS["config2"]
    assert bench.main_traffic(cfg2, cfg2.kv_heads) == (full, "ncu dram bytes of the config2 main-pass launch")
    t, src = bench.main_traffic(cfg2, 1)
    assert t == pytest.approx(full / cfg2.kv_heads) and "scaled to 1 of 8" in src
    assert bench.main_traffic(CONFIGS["config5"], 1) == (None, None)
    assert bench.main_traffic(CONFIGS["sweep_n65536_w16384"], 8) == (None, None)
