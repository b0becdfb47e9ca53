"""``bench.py`` end to end on a 2-head layer: the process exits 0 and prints one
JSON line carrying the keys of the bench contract."""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.gpu
def test_bench_prints_one_contract_line(cuda):
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--heads", "2", "--steps", "1", "--warmup", "3",
           "--no-cpu-baseline"]
    res = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout[-3000:]
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "config", "e2e", "roofline", "clocks", "gpu_launches"):
        assert key in line, key
    assert line["value"] > 0 and line["e2e"]["value"] > 0 and line["gpu_launches"] > 0
    assert line["config"]["heads"] == 2
