"""bench.py's host logic without a GPU: per-rank inputs, config descriptions, traffic records."""
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from aihost_b200.configs import CONFIGS  # noqa: E402


def test_every_rank_gets_the_global_lengths_and_capacity():
    """Ranks reseed the data but not the lengths: each rank's cache must hold the longest
    sequence of the shared length list (a rank-reseeded length draw once overflowed it)."""
    cfg = CONFIGS[3].scaled(batch=4, n_q_heads=8, n_kv_heads=2, head_dim=64)
    base = bench.device_inputs(cfg, torch.device("cpu"), 0)
    for rank in range(1, 8):
        inp = bench.device_inputs(cfg, torch.device("cpu"), rank)
        assert inp["lengths"] == base["lengths"] == cfg.lengths()
        assert inp["capacity"] == cfg.capacity()
        assert not torch.equal(inp["q"], base["q"])  # but different data


def test_head_shard_inputs_keep_global_lengths():
    cfg = CONFIGS[5].scaled(batch=2, cached=None, cached_list=[100, 300])
    for rank in range(4):
        inp, spec, shard, local = bench.shard_inputs(cfg, torch.device("cpu"), rank, 4)
        assert inp["lengths"] == [100, 300] and inp["capacity"] == cfg.capacity()
        assert spec.kv_token_stride % 16 == 0 and local.n_kv_heads == 2


def test_reference_arm_prints_the_same_config_as_ours():
    for n in range(1, 6):
        for world in (1, 2, 8):
            a = bench.cfg_desc(CONFIGS[n], "seq", world)
            assert a == bench.cfg_desc(CONFIGS[n], "seq", world)
            assert "parallelism" in a and "l2" in a


def test_stale_traffic_records_are_not_reported(tmp_path, monkeypatch):
    src = bench.KERNEL_SOURCE[2]
    good = bench.source_sha16(src)
    prof = tmp_path / "profiles"
    prof.mkdir()
    (prof / "traffic.txt").write_text(f"# header\nconfig2 123 {src} {good}\nconfig3 456 {bench.KERNEL_SOURCE[3]} "
                                      f"0000000000000000\n")
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    (tmp_path / "aihost_b200" / "csrc").mkdir(parents=True)
    for f in set(bench.KERNEL_SOURCE.values()):
        (tmp_path / "aihost_b200" / "csrc" / f).write_bytes((ROOT / "aihost_b200" / "csrc" / f).read_bytes())
    assert bench.read_traffic(2)[0] == 123.0
    assert bench.read_traffic(3)[0] is None and "stale" in bench.read_traffic(3)[1]
    assert bench.read_traffic(4)[0] is None
