"""bench.py's reference arm (the CPU implementation of the path, no GPU): one JSON line
with the contract's keys, for both workloads, and the same workload string as the
engine's arm."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("workload,unit", [("c2", "GFLOP/s"), ("lloyd", "iter/s")])
def test_reference_arm_line(workload, unit):
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--workload",
                          workload, "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=300,
                         cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == unit and line["value"] > 0
    assert line["higher_is_better"] is True and line["warmup"] >= 3
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    sys.path.insert(0, REPO)
    import bench
    assert line["config"] == bench.workload_config(workload, line["config"]["n"], 1)
    assert line["metric"] == bench.METRIC
