"""bench.py's reference arm (the oracle port timed on the host cores) keeps the JSON-line
contract the driver reads, on CPU: one line from rank 0 with the metric, config, e2e and
cpu_baseline keys; other ranks print nothing."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_ref(extra_env):
    env = dict(os.environ, BBH_REF_STEP_SECONDS="0.3", **extra_env)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3", "--workload", "cfg2"], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [l for l in r.stdout.splitlines() if l.strip()]


def test_reference_arm_line():
    lines = run_ref({"RANK": "0"})
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["metric"] == "sentences/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["workload"].startswith("cfg2")
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]


def test_reference_arm_other_ranks_silent():
    assert run_ref({"RANK": "1"}) == []
