"""bench.py's CPU legs run here: the reference arm (the reference's own CPU
GEMM compiled from its sources) and the cpu_baseline port, on tiny shapes,
printing the contract's JSON line."""
import json
import os
import subprocess
import sys

import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(O.ref() is None, reason="oracle/_ref not built")
def test_reference_arm_json():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
                        "--warmup", "1", "--m", "64", "--n", "256", "--k", "256"], capture_output=True, text=True,
                       timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    assert d["higher_is_better"] is True


def test_reference_arm_other_ranks_exit_quietly():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1"],
                       capture_output=True, text=True, timeout=120, cwd=ROOT, env=env)
    assert r.returncode == 0 and r.stdout.strip() == ""


def test_cpu_baseline_port():
    sys.path.insert(0, ROOT)
    import bench
    d = bench.cpu_baseline_port(64, 256, 256, 0.2)
    assert d["kind"] == "port" and d["value"] > 0 and d["cores"] >= 1 and "rows" in d["sample"]


def test_cpu_reference_1core():
    sys.path.insert(0, ROOT)
    import bench
    d = bench.cpu_reference_1core(8192, 8192, 8192, n=64)
    assert d["cores"] == 1 and d["gflops"] > 0 and d["kind"] in ("reference", "port")
    assert abs(d["extrapolated_s_full_workload"] - 2.0 * 8192 ** 3 / (d["gflops"] * 1e9)) < 1e-6 * d[
        "extrapolated_s_full_workload"]
    m = bench.cpu_model()
    assert m is None or isinstance(m, str)
