"""bench.py's CPU-side contract (no GPU): the reference arm prints one JSON
line with the keys the driver reads, and the synthetic inputs follow the
reference generator."""

import json
import os
import subprocess
import sys

import torch

from conftest import REPO
from oracle import layer as O


def test_reference_arm_json_line():
    proc = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                           "--config", "1", "--steps", "2", "--warmup", "3"],
                          capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] == "port"
    assert "workload" in d["config"] and "model" not in d["config"]
    # the GPU arm prints the same workload description (bench._config_dict)
    sys.path.insert(0, REPO)
    import bench

    assert d["config"] == bench._config_dict(1, 1, 1)


def test_traffic_table_parses_the_committed_summary():
    sys.path.insert(0, REPO)
    import bench

    table = bench._traffic_table()
    assert table[(3, "attention")] == 104_517_376 + 24_575_488
    assert table[(5, "gemm_ffn_in_gelu")] == 102_283_264 + 241_223_680
    assert all(v > 0 for v in table.values())


def test_reference_arm_other_ranks_exit_quietly():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    proc = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "3"], capture_output=True, text=True,
                          timeout=300, env=env)
    assert proc.returncode == 0 and proc.stdout.strip() == ""


def test_synthetic_case_matches_reference_generator():
    sys.path.insert(0, REPO)
    import bench

    cfg = bench._Cfg(1, 1)
    x, mask = bench._synthetic_case(cfg, 1234, cfg.batch_size)
    ocfg, pad = O.BASELINE_CONFIGS[1]
    ox, om = O.generate_random_case(ocfg, 1234, pad, 1.0)
    assert torch.equal(x, ox) and torch.equal(mask, om)


def test_attention_pairs_counts():
    import bench

    cfg = bench._Cfg(2, 1)   # causal, no mask
    assert bench._attention_pairs(cfg, None) == 4 * 512 * 513 // 2
    assert bench._attention_pairs(cfg, None, batch=1) == 512 * 513 // 2   # one shard's rows
    cfg1 = bench._Cfg(1, 1)  # key padding
    mask = torch.zeros(2, 128, dtype=torch.bool)
    mask[0, :100] = True
    mask[1, :70] = True
    assert bench._attention_pairs(cfg1, mask) == 128 * 100 + 128 * 70
