"""The bench's reference arm on the host cores (no GPU).

`bench.py --impl reference` times the CPU implementation of the per-die
timing path (the oracle port: the reference's per-die model lives in the
absent MQSim submodule) on a prefix of the config-1 trace and prints one
JSON line with the same metric, unit and config as the GPU arm, plus its
`cpu_baseline` and a zero-copy `e2e`.  Under torchrun only rank 0 runs it.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def _run(extra_env):
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    env.update(extra_env)
    return subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "3"],
                          cwd=REPO, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_line():
    p = _run({})
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "simulated HBF accesses/sec" and d["unit"] == "accesses/s"
    assert d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 3
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert "prefix" in d["config"]["sample"] and d["config"]["workload"].startswith("c1")
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert "prefix" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"],
                        "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_do_nothing():
    p = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [l for l in p.stdout.splitlines() if l.startswith("{")]
