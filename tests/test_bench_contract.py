"""bench.py's reference arm on CPU: one JSON line with the fields the
benchmark contract requires (the GPU arm's line is checked on the GPU box)."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_line():
    proc = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "cfg1",
         "--steps", "1", "--warmup", "3"],
        capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["config"]["workload"] == "cfg1"
    assert d["steps"] == 1 and d["warmup"] == 3 and d["value"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_warmup_below_three_is_rejected():
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--warmup", "2"],
                          capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert proc.returncode != 0 and "--warmup must be >= 3" in proc.stderr


def test_roofline_bound_follows_arithmetic_intensity():
    """Below the ridge (measured bf16 peak / measured HBM bandwidth) the line
    reports HBM GB/s against the measured copy bandwidth; above it, TFLOP/s
    against the measured bf16 peak.  Both fractions are always present."""
    import bench

    peaks = {"bf16_tflops": 1658.6, "hbm_gbs": 6553.9}
    cfg1 = bench.WORKLOADS["cfg1"]
    flop = bench.flops_for(cfg1, 2, 8, None)
    nbytes = bench.algorithmic_bytes(cfg1, 2, 8, None)
    assert nbytes == 4 * 2 * 8 * 512 * 64 * 2  # Q, K, V read and O written, bf16
    r = bench.roofline(flop, nbytes, 0.0118, peaks, "measured", None, None)
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and r["peak"] == peaks["hbm_gbs"]
    assert abs(r["achieved"] - nbytes / 0.0118e-3 / 1e9) < 1e-6
    assert abs(r["frac"] - r["achieved"] / peaks["hbm_gbs"]) < 1e-12
    assert r["tensor"]["unit"] == "TFLOP/s" and r["arithmetic_intensity"] < r["ridge"]

    cfg4 = bench.WORKLOADS["cfg4"]
    flop = bench.flops_for(cfg4, 1, 32, None)
    nbytes = bench.algorithmic_bytes(cfg4, 1, 32, None)
    r = bench.roofline(flop, nbytes, 7.0, peaks, "measured", 1.2e9, {"file": "x"})
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s" and r["peak"] == peaks["bf16_tflops"]
    assert r["hbm"]["unit"] == "GB/s" and r["traffic"] == 1.2e9


def test_key_padded_bytes_count_valid_rows_only():
    import bench

    cfg3 = bench.WORKLOADS["cfg3"]
    lengths = [1024] * 16
    got = bench.algorithmic_bytes(cfg3, 16, 32, lengths)
    # Q, K, V valid rows read, the whole output written, plus the bool mask
    want = 2 * 128 * (32 * 3 * 1024 * 16 + 16 * 32 * 4096) + 16 * 4096
    assert got == want


def test_default_workload_is_the_largest_single_gpu_config():
    import bench

    args = bench.argparse.ArgumentParser()
    src = (ROOT / "bench.py").read_text()
    assert 'ap.add_argument("--workload", default="cfg4"' in src
    assert bench.WORKLOADS["cfg4"]["shard"] == "heads"
    del args


def test_reference_arm_of_the_softmax_workload_times_the_softmax():
    proc = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "sm2",
         "--steps", "1", "--warmup", "3", "--heads", "1"],
        capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-2000:]
    d = json.loads([l for l in proc.stdout.splitlines() if l.startswith("{")][-1])
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["value"] > 0
    assert "reference_softmax" in d["cpu_baseline"]["sample"]
