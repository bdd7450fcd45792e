"""CPU tests of the autotune driver and the report generator.

The autotune driver is exercised end to end against a stand-in bench_gemm
(a small script that reads the trial config and writes the reference's CSV
columns), so its grid, config emission, CSV parsing, ranking, reports and
--apply-best are covered without a GPU.
"""
import json
import os
import stat
import sys
import textwrap
from pathlib import Path

import pytest

from kebab_b200 import autotune, report

FAKE_BENCH = textwrap.dedent(
    """\
    #!{python}
    # Stand-in for bench_gemm: TFLOP/s = version / 10, halved for "dp".
    import os, re, sys
    args = sys.argv[1:]
    cfg = open(args[args.index("--config") + 1]).read()
    out = args[args.index("--out-dir") + 1]
    versions = [int(v) for v in re.search(r"versions: \\[([^\\]]*)\\]", cfg).group(1).split(",")]
    prec = re.search(r"precisions: \\[(\\w+)\\]", cfg).group(1)
    m = re.search(r"matrix_sizes: \\[(\\d+)\\]", cfg)
    M = int(m.group(1)) if m else int(re.search(r"shapes: \\[\\[(\\d+),", cfg).group(1))
    mode = os.environ.get("KEBAB_V120_MODE", "")
    with open(os.path.join(out, "gemm_results_%s_cuda.csv" % prec), "w") as f:
        f.write("Operator,Variant,BatchSize,Latency(ms),Throughput(GFLOPS),Speedup\\n")
        for v in versions:
            if v == 999:
                continue  # a version that failed verification is not written
            tf = v / 10.0 * (0.5 if mode == "dp" else 1.0)
            f.write("GEMM,cuda_v%d_name,%d,%.4f,%.1f,%.4f\\n" % (v, M, 1.0 / tf, tf * 1000.0, tf / 20.0))
    sys.exit(2 if 999 in versions else 0)
    """
)


@pytest.fixture
def fake_bench(tmp_path):
    p = tmp_path / "bench_gemm"
    p.write_text(FAKE_BENCH.format(python=sys.executable))
    p.chmod(p.stat().st_mode | stat.S_IXUSR)
    return p


@pytest.fixture
def cfg(tmp_path):
    p = tmp_path / "config.yaml"
    p.write_text("# keep me\noperators:\n  gemm:\n    versions: [104, 105, 120]  # order\n    seed: 7\n"
                 "    init_method: rand-rand\n")
    return p


def test_grid_groups_plain_versions_and_splits_v120_modes():
    runs = autotune.build_grid([105, 107, 120], ["RC"], ["float16"], [(4096, 4096, 4096)], ["heuristic", "dp"])
    assert runs == [((105, 107), "RC", "float16", (4096, 4096, 4096), None),
                    ((120,), "RC", "float16", (4096, 4096, 4096), "heuristic"),
                    ((120,), "RC", "float16", (4096, 4096, 4096), "dp")]


def test_trial_config_is_readable_by_the_harness_subset():
    base = {"gpu_id": 0, "init_method": "rand-rand", "seed": 42}
    sq = autotune.trial_config_text(base, [105, 107], "RC", "float16", (2048, 2048, 2048), 3, 5)
    assert "matrix_sizes: [2048]" in sq and "shapes" not in sq and "versions: [105, 107]" in sq
    rect = autotune.trial_config_text(base, [120], "RR", "bfloat16", (64, 8192, 4096), 3, 5)
    assert "shapes: [[64, 8192, 4096]]" in rect and "matrix_sizes" not in rect
    import yaml

    d = yaml.safe_load(rect)
    assert d["benchmark"] == {"warmup_runs": 3, "measurement_runs": 5}
    assert d["operators"]["gemm"]["shapes"] == [[64, 8192, 4096]]


def test_parse_shapes():
    assert autotune.parse_shapes("16384x28672x8192, 64X8192X8192") == [(16384, 28672, 8192), (64, 8192, 8192)]
    with pytest.raises(ValueError):
        autotune.parse_shapes("1x2")


def test_autotune_end_to_end_with_stand_in_bench(tmp_path, fake_bench, cfg):
    out = tmp_path / "results"
    rc = autotune.main(["--config", str(cfg), "--bench-bin", str(fake_bench), "--versions", "104,105,120,999",
                        "--sizes", "2048", "--shapes", "64x8192x8192", "--v120-modes", "heuristic,dp",
                        "--out-dir", str(out), "--apply-best"])
    assert rc == 0
    data = json.loads(next(out.glob("autotune_gemm_*.json")).read_text())
    # 2 problems x (3 versions that report + v120 twice) ... 999 is dropped.
    assert data["num_trials"] == 2 * (2 + 2)
    assert data["best"]["version"] == 120 and data["best"]["v120_mode"] == "heuristic"
    assert {(t["M"], t["version"]) for t in data["best_per_problem"]} == {(2048, 120), (64, 120)}
    dp = [t for t in data["trials"] if t["v120_mode"] == "dp"]
    assert dp and all(abs(t["tflops"] - 6.0) < 1e-9 for t in dp)
    assert "Best per problem" in next(out.glob("autotune_gemm_*.md")).read_text()
    text = cfg.read_text()
    assert "versions: [120, 104, 105]  # order" in text and text.startswith("# keep me")


def test_autotune_rejects_unknown_v120_mode(cfg, fake_bench):
    assert autotune.main(["--config", str(cfg), "--bench-bin", str(fake_bench), "--v120-modes", "bogus",
                          "--dry-run"]) == 2


def test_autotune_dry_run_needs_no_binary(cfg, capsys):
    assert autotune.main(["--config", str(cfg), "--bench-bin", "/nonexistent", "--dry-run", "--sizes", "8192"]) == 0
    assert "bench_gemm runs" in capsys.readouterr().out


LAUNCH_CSV = """==PROF== Connected to process 1
"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"
"0","1","p","h","void kb::gemm_kernel<__half, 512>(CUtensorMap_st, UmmaArgs)","1","7","(320, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","us","750.00"
"1","1","p","h","void kb::gemm_kernel<__half, 512>(CUtensorMap_st, UmmaArgs)","1","7","(320, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","ms","0.75"
"2","1","p","h","void at::fill_kernel(float*)","1","7","(128, 1, 1)","(8, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","ns","500000"
"""

RAW_CSV = """"ID","Kernel Name","gpu__time_duration.sum","dram__bytes_read.sum","dram__bytes_write.sum","sm__cycles_elapsed.avg.per_second","launch__shared_mem_per_block_dynamic","sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed"
"","","us","Mbyte","Kbyte","Ghz","Kbyte/block","%"
"0","void kb::gemm_kernel<__half, 512>(CUtensorMap_st)","800","900","134217.728","1.4","200","90.5"
"""


def test_launch_list_shares():
    agg = report.launch_list(LAUNCH_CSV)
    name = "void kb::gemm_kernel<__half, 512>(CUtensorMap_st, UmmaArgs)"
    assert agg[name]["launches"] == 2 and agg[name]["total_s"] == pytest.approx(1.5e-3)
    md = report.launch_list_markdown(agg, "t", "python bench.py")
    assert "`kb::gemm_kernel<__half, 512>`" in md and "75.0 %" in md and "25.0 %" in md


def test_ncu_raw_figures_and_roofline():
    rows = report.raw_rows(RAW_CSV)
    f = report.launch_figures(rows[0], flops=1.0995e12, alg_bytes=402653184)
    assert f["duration"] == "800.0 us"
    assert f["SM clock"] == "1400 MHz"
    assert f["dynamic smem/block"] == "200.000 KB"
    assert f["DRAM traffic (read+write)"] == "1034217728 B"
    assert float(f["achieved TFLOP/s (under ncu)"]) == pytest.approx(1374.4, abs=0.1)
    assert float(f["traffic / algorithmic bytes"]) == pytest.approx(1034217728 / 402653184, abs=1e-3)


def test_bench_csv_markdown(tmp_path):
    p = tmp_path / "gemm_results_float16_cuda.csv"
    p.write_text("Operator,Variant,BatchSize,Latency(ms),Throughput(GFLOPS),Speedup\n"
                 "GEMM,cuda_v105_pair,8192,0.9,1200000,0.95\nGEMM,cuda_v107_wide,8192,0.85,1290000,1.01\n")
    md = report.bench_csv_markdown(report.read_bench_rows([p]))
    lines = [l for l in md.splitlines() if l.startswith("| 8192")]
    assert "cuda_v107_wide`**" not in lines[0] and "**best**" in lines[0] and "1290.0" in lines[0]


def test_report_cli_launches(tmp_path):
    p = tmp_path / "l.csv"
    p.write_text(LAUNCH_CSV)
    o = tmp_path / "o.md"
    assert report.main(["launches", str(p), "-o", str(o)]) == 0
    assert "gemm_kernel" in o.read_text()


def test_profile_commands_are_safe():
    from kebab_b200 import profile
    plain, cap = profile.commands(107, 4096, 4096, 4096, "float16", "RC", Path("x/y"), "full", 1, "gemm_umma")
    assert plain[0].endswith("runonce_gemm") and "--version" in plain
    assert cap[:2] == ["ncu", "--set"] and "--clock-control" in cap and cap[cap.index("--clock-control") + 1] == "none"
    assert cap[cap.index("-c") + 1] == "1" and cap[cap.index("-k") + 1] == "regex:gemm_umma"
    assert cap[-len(plain):] == plain  # ncu profiles exactly the command that ran plainly
    with pytest.raises(ValueError):
        profile.commands(107, 64, 64, 64, "float16", "RC", Path("x"), "full", 5, "gemm")


def test_profile_refuses_large_problems(capsys):
    from kebab_b200 import profile
    assert profile.main(["--m", "32768", "--n", "32768", "--k", "32768", "--dry-run"]) == 2
    assert profile.main(["--m", "1024", "--n", "1024", "--k", "1024", "--dry-run"]) == 0
    out = capsys.readouterr().out
    assert "--clock-control none" in out


def test_autotune_modes_match_the_v120_parser():
    """Every KEBAB_V120_MODE value the C++ dispatcher accepts (its primary
    spelling) is a mode autotune can sweep, and no other."""
    import re

    src = (Path(__file__).resolve().parents[1] / "kebab_b200" / "csrc" / "gemm_api.cu").read_text()
    body = src[src.index("int choose_v120("):]
    body = body[:body.index("// Decode-like shapes")]
    parsed = {m.group(1).lower() for m in re.finditer(r'if \(\(?m == "(\w+)"', body)}
    assert parsed | {"heuristic"} == set(autotune.V120_MODES)
