"""bench.py's CPU-side contract: the reference arm prints one JSON line with
the driver's keys (run on a small sequence so that it takes seconds), and
the FLOP counts and profile lookups the GPU arm reports are consistent."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--workload", "mha", "--seq-len", "512", "--steps", "1", "--warmup", "3"],
                         capture_output=True, text=True, check=True, cwd=ROOT).stdout
    lines = [l for l in out.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] == "port"


def test_flop_counts_and_profiles():
    # causal pairs N(N+1)/2, 4*d each
    assert bench.attn_flops(1, 1, 4, 4, 8, True) == 4 * 8 * 10
    assert bench.attn_flops(2, 3, 4, 5, 8, False) == 4 * 8 * 20 * 6
    assert bench.symphony_flops(4, 8) == bench.attn_flops(1, 1, 4, 4, 8, True) + 16 * 4 * 64 + 8 * 32
    # the default workload's DRAM traffic comes from the committed ncu summary
    assert bench.profile_traffic("mha") is not None and bench.profile_traffic("mha") > 4e8
    assert bench.profile_traffic("ring") is not None and bench.profile_traffic("ring") > 8e9  # the default
    for name, w in bench.WORKLOADS.items():
        assert w["cfg"] and w["D"] in (64, 128, 256), name
