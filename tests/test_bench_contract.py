"""bench.py's reference arm (the reference's CPU step, no GPU) prints one
JSON line with the keys of the benchmark contract; ranks other than 0 print
nothing and exit 0."""

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                           *args], capture_output=True, text=True, env=env, timeout=600)


@pytest.mark.parametrize("world", [1, 2])
def test_reference_arm_line(world):
    env = {"WORLD_SIZE": str(world), "RANK": "0", "LOCAL_RANK": "0"}
    p = _run(env, "--gpus", str(world), "--steps", "2", "--warmup", "1")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == world and d["steps"] == 2
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_do_no_work():
    p = _run({"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"}, "--gpus", "2", "--steps", "2",
             "--warmup", "1")
    assert p.returncode == 0, p.stderr[-2000:]
    assert p.stdout.strip() == ""
