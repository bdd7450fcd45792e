"""C++ harness (kebab_b200/bin/bench_gemm, runonce_gemm): the YAML-subset
config reader keeps the reference ConfigParser's keys and defaults
(kebab/lib/common/config_parser.cpp:184-392) — checked on CPU through
--dump-config — and the config-driven benchmark runs, verifies and writes the
reference's CSV columns on the GPU."""
import csv
import json
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "kebab_b200", "bin")


def dump(tmp_path, text):
    p = tmp_path / "c.yaml"
    p.write_text(text)
    r = subprocess.run([os.path.join(BIN, "bench_gemm"), "--config", str(p), "--dump-config"], capture_output=True,
                       text=True)
    return r


def test_dump_full_schema(tmp_path):
    r = dump(tmp_path, """
# comment line
build:
  mode: debug   # trailing comment
benchmark:
  warmup_runs: 7
  measurement_runs: 33
operators:
  gemm:
    enabled: true
    gpu_id: 3
    impl:
      - cuda
      - "cute"
    versions: [104, 105]
    init_method: 'one-rand'
    verbose: yes
    seed: 9
    matrix_sizes:
    - 512
    - 1024
    shapes: [[64, 8192, 8192], [16384, 28672, 8192]]
    modes: [RC, rr]
    precisions: [float16]
""")
    assert r.returncode == 0, r.stderr
    d = json.loads(r.stdout)
    assert d["warmup_runs"] == 7 and d["measurement_runs"] == 33
    assert d["impls"] == ["cuda", "cute"] and d["versions"] == [104, 105]
    assert d["matrix_sizes"] == [512, 1024] and d["modes"] == ["RC", "rr"]
    assert d["init_method"] == "one-rand" and d["gpu_id"] == 3 and d["verbose"] is True and d["seed"] == 9
    assert d["shapes"] == [[64, 8192, 8192], [16384, 28672, 8192]]
    assert d["build_mode"] == "debug"


def test_reference_defaults(tmp_path):
    # Missing keys fall back to the reference's defaults.
    r = dump(tmp_path, "operators:\n  gemm:\n    version: 5\n    impl: cuda\n")
    assert r.returncode == 0, r.stderr
    d = json.loads(r.stdout)
    assert d["warmup_runs"] == 10 and d["measurement_runs"] == 100
    assert d["versions"] == [5] and d["impls"] == ["cuda"]
    assert d["modes"] == ["NT"] and d["precisions"] == ["float16"] and d["init_method"] == "rand-rand"
    assert d["gpu_id"] == 0 and d["verbose"] is False and d["seed"] == 42 and d["enabled"] is True
    r = dump(tmp_path, "operators:\n  gemm:\n    enabled: false\n")
    d = json.loads(r.stdout)
    assert d["impls"] == ["cute"] and d["versions"] == [1] and d["enabled"] is False


def test_repo_config_parses(tmp_path):
    r = subprocess.run([os.path.join(BIN, "bench_gemm"), "--config", os.path.join(ROOT, "config.yaml"),
                        "--dump-config"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    d = json.loads(r.stdout)
    assert 105 in d["versions"] and d["modes"] == ["RC"]


def test_bad_yaml_is_an_error(tmp_path):
    r = dump(tmp_path, "operators:\n\tgemm:\n    versions: [1]\n")
    assert r.returncode == 1 and "tabs" in r.stderr
    r = dump(tmp_path, "operators:\n  gemm:\n    versions: [1, 2\n")
    assert r.returncode == 1 and "unterminated" in r.stderr
    r = subprocess.run([os.path.join(BIN, "bench_gemm"), "--config", str(tmp_path / "missing.yaml")],
                       capture_output=True, text=True)
    assert r.returncode == 1 and "cannot open" in r.stderr


@pytest.mark.gpu
def test_bench_gemm_runs_and_writes_csv(cuda, tmp_path):
    cfg = tmp_path / "c.yaml"
    cfg.write_text("""
benchmark: {}
operators:
  gemm:
    impl: [cuda, cute]
    versions: [1, 101, 102, 103, 104, 105, 120, 10]
    matrix_sizes: [512, 1024]
    shapes: [[64, 1024, 512], [264, 520, 136]]
    modes: [RC]
    precisions: [float16, bfloat16, float32]
""".replace("benchmark: {}", "benchmark:\n  warmup_runs: 2\n  measurement_runs: 5"))
    r = subprocess.run([os.path.join(BIN, "bench_gemm"), "--config", str(cfg), "--out-dir", str(tmp_path / "out")],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "FAIL" not in r.stdout and "ERROR" not in r.stdout
    for t in ("float16", "bfloat16"):
        rows = list(csv.DictReader(open(tmp_path / "out" / ("gemm_results_%s_cuda_cute.csv" % t))))
        assert list(rows[0].keys()) == ["Operator", "Variant", "BatchSize", "Latency(ms)", "Throughput(GFLOPS)",
                                        "Speedup"]
        assert len(rows) == 4 * 8  # 4 problems x 8 versions, all verified
        assert all(float(x["Throughput(GFLOPS)"]) > 0 for x in rows)


@pytest.mark.gpu
def test_runonce(cuda):
    r = subprocess.run([os.path.join(BIN, "runonce_gemm"), "--config", os.path.join(ROOT, "config.yaml"),
                        "--version", "105", "--m", "2048", "--n", "1024", "--k", "4096"], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout + r.stderr
