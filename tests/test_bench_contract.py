"""bench.py's reference arm on the CPU: one JSON line with the keys the
benchmark contract requires (impl, metric/value/unit, steps/warmup,
higher_is_better, cpu_baseline with kind/cores/sample, e2e with zero host
copies), on the cheapest workload (the config-0 GEMV)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--workload", "gemv", "--steps", "1", "--warmup", "3"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better",
                "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["steps"] == 1 and d["warmup"] == 3
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] == "gemv"


def test_reference_arm_times_the_int8_head_port():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--workload", "int8-head", "--steps", "1", "--warmup", "3"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["config"]["workload"] == "int8-head"
    assert d["unit"] == "GB/s" and d["value"] > 0
    assert d["metric"] == "int8 affine head GEMV HBM GB/s"


def test_both_arms_share_the_workload_config():
    """The reference arm and the GPU arm describe a workload with the same
    config object (workload_config), so the two lines compare like for like."""
    sys.path.insert(0, ROOT)
    import bench
    for w in ("oss120-decode64", "oss20-decode1", "qwen3-decode32", "gemv", "int8-head"):
        a, b = bench.workload_config(w, 1), bench.workload_config(w, 1)
        assert a == b and a["workload"] == w
    at2 = bench.workload_config("oss120-decode64", 2)
    assert at2["parallelism"].startswith("ep2 (all-to-all") and at2["layers"] == 36
    assert bench.workload_config("gemv")["copies"] == bench.GEMV_COPIES
