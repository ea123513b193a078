"""The JSON line of `bench.py --impl reference` (the reference algorithm timed on the host cores),
checked on the CPU-sized workload: the keys the bench contract asks for, the warm-up and step
counts it really used, and that ranks other than 0 exit without work."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(extra_env=None, *args):
    env = dict(os.environ, **(extra_env or {}))
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "cpu", *args]
    return subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_line():
    res = _run(None, "--steps", "2", "--warmup", "3")
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["warmup"] == 3 and line["steps"] == 2
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert abs(line["value"] - line["cpu_baseline"]["value"]) < 1e-9
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert "3 warm-up drafts" in line["cpu_baseline"]["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"] == "cfg1-cpu-plumbing"


def test_reference_arm_other_ranks_exit_quietly():
    res = _run({"RANK": "1", "WORLD_SIZE": "2"}, "--steps", "1", "--warmup", "3")
    assert res.returncode == 0, res.stderr[-2000:]
    assert res.stdout.strip() == ""
