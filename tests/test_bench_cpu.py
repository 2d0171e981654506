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


def test_roofline_traffic_is_per_launch():
    """roofline.traffic = ncu DRAM bytes per token x the tokens ONE launch processes: a layer
    kernel runs once per layer of each forward, so a pass of F forwards over T tokens has
    F x layers launches of T / F tokens each."""
    sys.path.insert(0, ROOT)
    import bench

    T, layers, forwards, bpt = 8_900_000, 6, 128, 4390.5
    per_launch = bench.traffic_per_launch("ffn2_gemm_ln", bpt, T, layers, forwards * layers)
    assert abs(per_launch - bpt * T / forwards) <= 0.1 * bpt * T / forwards
    # once-per-forward kernels
    assert bench.traffic_per_launch("pool_l2", 769.4, T, layers, forwards) == 769.4 * T / forwards


def test_kernel_entry_rooflines():
    """A GEMM's roofline is the larger of its tensor time and its HBM time at the measured
    peaks; the O projection (K = 384) is HBM-bound, FFN2 (K = 1536) tensor-bound."""
    sys.path.insert(0, ROOT)
    import bench

    peaks = (6451.2, 1686.2, 1426.8)
    T, layers, launches = 70_000 * 128, 6, 128 * 6
    o = bench.kernel_entry("o_gemm_ln", 50e-3 * launches, launches, T, layers, 0.0, peaks)
    f = bench.kernel_entry("ffn2_gemm_ln", 100e-3 * launches, launches, T, layers, 0.0, peaks)
    assert o["bound"] == "hbm" and f["bound"] == "tensor"
    assert abs(f["tflops"] - 2 * 70_000 * 384 * 1536 / 100e-6 / 1e12) < 1.0
    assert f["roofline_frac"] == f["tensor_frac"] and o["roofline_frac"] == o["hbm_frac"]
