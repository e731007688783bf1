"""bench.py's TP partition (the multi-GPU sharding of the reload path):
every rank owns heads / TP KV heads of every layer, TP from --tp, the
config's own TP or the number of GPUs, and the scaling kind follows from it.
Pure host logic, no GPU."""
from __future__ import annotations

import pytest

import bench


@pytest.mark.parametrize("world,heads", [(1, 8), (2, 4), (4, 2), (8, 1)])
def test_c2_splits_its_heads_over_the_gpus(world, heads):
    cfg = bench.shard_config(bench.CONFIGS["c2"], world, None)
    assert (cfg["heads"], cfg["heads_total"], cfg["tp"]) == (heads, 8, world)
    assert cfg["tp_from_gpus"]
    # One model's heads split over the GPUs: the job's work is fixed.
    assert bench.scaling_kind(cfg, world) == "strong"


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_c5_keeps_its_own_tp8_shard(world):
    """C5 is Llama-3-70B at TP = 8: one KV head per GPU whatever the GPU count,
    so N GPUs run N fixed shards."""
    cfg = bench.shard_config(bench.CONFIGS["c5"], world, None)
    assert (cfg["heads"], cfg["tp"]) == (1, 8)
    assert not cfg["tp_from_gpus"]
    assert bench.scaling_kind(cfg, world) == "weak"


def test_more_gpus_than_heads_repeat_the_shards():
    cfg = bench.shard_config(bench.CONFIGS["c3"], 8, None)   # 4 KV heads
    assert (cfg["heads"], cfg["tp"]) == (1, 4)
    assert bench.scaling_kind(cfg, 8) == "weak"


def test_explicit_tp():
    cfg = bench.shard_config(bench.CONFIGS["c2"], 8, 2)
    assert (cfg["heads"], cfg["tp"]) == (4, 2)
    assert bench.scaling_kind(cfg, 8) == "weak"
    with pytest.raises(SystemExit):
        bench.shard_config(bench.CONFIGS["c2"], 1, 3)


def test_host_bound_ceilings_scale_by_algorithmic_bytes_per_wire_byte():
    host = {"gbs": 100.0, "threads": 16}
    out = bench.host_bound(host, encrypt_gbs=50.0, algo=200, wire=100, link_all_gbs=40.0, link_bytes=100)
    assert out["host_copy_gbs"] == 100.0
    assert out["e2e_bound_gbs"] == 100.0          # 50 GB/s of wire x 2 algorithmic bytes per wire byte
    assert out["e2e_link_bound_gbs"] == 80.0      # 40 GB/s crossing x 200 / 100
