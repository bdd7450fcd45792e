"""Autotune over the B200 ladder: the role of the reference's
``scripts/autotune_gemm.py`` (``:84-178`` trial loop, ``:181-231`` reports,
``:234-250`` apply-best), driven through ``kebab_b200/bin/bench_gemm``.

Search space: versions x modes x precisions x problems, and for version 120
(the decomposition heuristic, reference v20) every ``KEBAB_V120_MODE`` listed
(the reference's ``KEBAB_V20_MODE`` sweep, ``autotune_gemm.py:300-305``).
Each trial writes its own config file into a scratch directory and runs
``bench_gemm --config <it> --out-dir <scratch>``; the user's config.yaml is
never edited unless ``--apply-best`` is given (the reference edits it in
place and restores it). Results are read back from the CSV columns the
reference's scripts read (``Variant``, ``Latency(ms)``,
``Throughput(GFLOPS)``, ``Speedup``), ranked by (speedup vs cuBLAS, TFLOP/s,
-latency) like ``trial_sort_key`` (``:176-177``).

Extensions over the reference: non-square problems (``--shapes MxNxK,...``)
and a per-problem winner table, which is what a dispatcher needs (the
reference only reports the global best).

Usage::

    python -m kebab_b200.autotune --sizes 2048,4096,8192 --versions 105,107,109,120
"""
from __future__ import annotations

import argparse
import csv
import itertools
import json
import os
import re
import subprocess
import sys
import tempfile
import time
from dataclasses import asdict, dataclass
from datetime import datetime
from pathlib import Path
from typing import Dict, List, Optional, Sequence, Tuple

REPO = Path(__file__).resolve().parents[1]
DEFAULT_BENCH = REPO / "kebab_b200" / "bin" / "bench_gemm"
V120_MODES = ("heuristic", "dp", "persistent", "pair", "wide", "pair384", "streamk", "streamk1", "skinny", "n128", "n64")

Problem = Tuple[int, int, int]


@dataclass
class Trial:
    version: int
    mode: str
    precision: str
    M: int
    N: int
    K: int
    v120_mode: Optional[str]
    variant: str
    latency_ms: float
    tflops: float
    speedup: float
    est_cublas_tflops: float

    @property
    def problem(self) -> Problem:
        return (self.M, self.N, self.K)


def parse_list_int(raw: str) -> List[int]:
    return [int(x) for x in raw.split(",") if x.strip()]


def parse_list_str(raw: str) -> List[str]:
    return [x.strip() for x in raw.split(",") if x.strip()]


def parse_shapes(raw: str) -> List[Problem]:
    out = []
    for s in parse_list_str(raw):
        parts = re.split(r"[xX*]", s)
        if len(parts) != 3:
            raise ValueError(f"shape {s!r} is not MxNxK")
        out.append(tuple(int(p) for p in parts))
    return out


def load_base(path: Path) -> dict:
    """The keys of the user's config that a trial keeps (warm-up and
    measurement counts are overridden per run)."""
    import yaml

    with path.open(encoding="utf-8") as f:
        data = yaml.safe_load(f) or {}
    gemm = ((data.get("operators") or {}).get("gemm")) or {}
    return {
        "gpu_id": int(gemm.get("gpu_id", 0)),
        "init_method": str(gemm.get("init_method", "rand-rand")),
        "seed": int(gemm.get("seed", 42)),
    }


def trial_config_text(base: dict, versions: Sequence[int], mode: str, precision: str, problem: Problem,
                      warmup: int, measurement: int) -> str:
    """A config in the YAML subset bench_gemm reads (flow lists, one level of
    nesting for shapes). Square problems go to matrix_sizes, the rest to
    shapes, so the CSV's variant names match the reference's."""
    M, N, K = problem
    lines = [
        "benchmark:",
        f"  warmup_runs: {int(warmup)}",
        f"  measurement_runs: {int(measurement)}",
        "operators:",
        "  gemm:",
        "    enabled: true",
        f"    gpu_id: {base['gpu_id']}",
        "    impl: [cuda]",
        f"    versions: [{', '.join(str(int(v)) for v in versions)}]",
        f"    init_method: {base['init_method']}",
        f"    seed: {base['seed']}",
    ]
    if M == N == K:
        lines.append(f"    matrix_sizes: [{M}]")
    else:
        lines.append(f"    shapes: [[{M}, {N}, {K}]]")
    lines += [f"    modes: [{mode}]", f"    precisions: [{precision}]", ""]
    return "\n".join(lines)


def read_csv_rows(path: Path) -> List[Dict[str, str]]:
    with path.open(encoding="utf-8", newline="") as f:
        return list(csv.DictReader(f))


def trials_from_rows(rows: List[Dict[str, str]], versions: Sequence[int], mode: str, precision: str,
                     problem: Problem, v120_mode: Optional[str]) -> List[Trial]:
    """One Trial per requested version: its best CSV row (variant prefix
    ``cuda_v<id>_``, as ``autotune_gemm.py:146-156`` matches them)."""
    out = []
    for v in versions:
        tag = f"cuda_v{v}_"
        best = None
        for r in rows:
            if not r.get("Variant", "").startswith(tag):
                continue
            if best is None or float(r["Throughput(GFLOPS)"]) > float(best["Throughput(GFLOPS)"]):
                best = r
        if best is None:
            continue
        tflops = float(best["Throughput(GFLOPS)"]) / 1000.0
        speedup = float(best["Speedup"])
        out.append(Trial(version=v, mode=mode, precision=precision, M=problem[0], N=problem[1], K=problem[2],
                         v120_mode=v120_mode, variant=best["Variant"], latency_ms=float(best["Latency(ms)"]),
                         tflops=tflops, speedup=speedup,
                         est_cublas_tflops=tflops / speedup if speedup > 0 else 0.0))
    return out


def trial_sort_key(t: Trial):
    return (t.speedup, t.tflops, -t.latency_ms)


def build_grid(versions, modes, precisions, problems, v120_modes):
    """Runs of bench_gemm: (versions, mode, precision, problem, v120_mode).
    Plain versions of one (problem, mode, precision) share a run (one cuBLAS
    timing, one input upload); each v120 mode is its own run, since it is an
    environment variable of the process."""
    plain = [v for v in versions if v != 120]
    runs = []
    for problem, mode, precision in itertools.product(problems, modes, precisions):
        if plain:
            runs.append((tuple(plain), mode, precision, problem, None))
        if 120 in versions:
            for vm in v120_modes:
                runs.append(((120,), mode, precision, problem, vm))
    return runs


def run_one(bench_bin: Path, base: dict, run, warmup: int, measurement: int, timeout_s: int,
            scratch: Path) -> List[Trial]:
    versions, mode, precision, problem, v120_mode = run
    cfg = scratch / "trial.yaml"
    cfg.write_text(trial_config_text(base, versions, mode, precision, problem, warmup, measurement))
    out_dir = scratch / "results"
    out_dir.mkdir(exist_ok=True)
    csv_path = out_dir / f"gemm_results_{precision}_cuda.csv"
    if csv_path.exists():
        csv_path.unlink()
    env = os.environ.copy()
    if v120_mode:
        env["KEBAB_V120_MODE"] = v120_mode
    else:
        env.pop("KEBAB_V120_MODE", None)
    proc = subprocess.run([str(bench_bin), "--config", str(cfg), "--out-dir", str(out_dir)], env=env,
                          capture_output=True, text=True, timeout=timeout_s, check=False)
    # bench_gemm exits 2 when a version fails verification; the passing ones
    # are still in the CSV (a failing version is dropped, as in the reference).
    if proc.returncode not in (0, 2) or not csv_path.exists():
        raise RuntimeError(f"bench_gemm failed (rc={proc.returncode}) for {run}:\n"
                           f"stdout:\n{proc.stdout[-2000:]}\nstderr:\n{proc.stderr[-2000:]}")
    return trials_from_rows(read_csv_rows(csv_path), versions, mode, precision, problem, v120_mode)


def best_per_problem(trials: List[Trial]) -> Dict[Tuple[Problem, str, str], Trial]:
    best: Dict[Tuple[Problem, str, str], Trial] = {}
    for t in trials:
        k = (t.problem, t.mode, t.precision)
        if k not in best or trial_sort_key(t) > trial_sort_key(best[k]):
            best[k] = t
    return best


def write_reports(out_dir: Path, trials: List[Trial], top_k: int, stamp: Optional[str] = None) -> Dict[str, Path]:
    out_dir.mkdir(parents=True, exist_ok=True)
    stamp = stamp or datetime.now().strftime("%Y%m%d_%H%M%S")
    ranked = sorted(trials, key=trial_sort_key, reverse=True)
    winners = best_per_problem(trials)
    jpath = out_dir / f"autotune_gemm_{stamp}.json"
    with jpath.open("w", encoding="utf-8") as f:
        json.dump({"generated_at": datetime.now().isoformat(), "num_trials": len(trials), "top_k": top_k,
                   "best": asdict(ranked[0]) if ranked else None,
                   "best_per_problem": [asdict(t) for t in winners.values()],
                   "trials": [asdict(t) for t in ranked]}, f, indent=2)
    mpath = out_dir / f"autotune_gemm_{stamp}.md"
    with mpath.open("w", encoding="utf-8") as f:
        f.write("# GEMM autotune report\n\n")
        f.write(f"Trials: {len(trials)}\n\n")
        f.write("| Rank | Version | v120 mode | Mode | Precision | M | N | K | TFLOP/s | vs cuBLAS | Latency (ms) | Variant |\n")
        f.write("|---:|---:|---|---|---|---:|---:|---:|---:|---:|---:|---|\n")
        for i, t in enumerate(ranked[:top_k], 1):
            f.write(f"| {i} | {t.version} | {t.v120_mode or '-'} | {t.mode} | {t.precision} | {t.M} | {t.N} | {t.K} "
                    f"| {t.tflops:.1f} | {t.speedup:.3f} | {t.latency_ms:.4f} | {t.variant} |\n")
        f.write("\n## Best per problem\n\n")
        f.write("| M | N | K | Mode | Precision | Version | v120 mode | TFLOP/s | vs cuBLAS |\n")
        f.write("|---:|---:|---:|---|---|---:|---|---:|---:|\n")
        for (p, mode, prec), t in sorted(winners.items()):
            f.write(f"| {p[0]} | {p[1]} | {p[2]} | {mode} | {prec} | {t.version} | {t.v120_mode or '-'} "
                    f"| {t.tflops:.1f} | {t.speedup:.3f} |\n")
        if ranked:
            b = ranked[0]
            f.write("\n## Recommended\n\n")
            f.write(f"- versions priority: [{b.version}]\n")
            if b.version == 120:
                f.write(f"- export KEBAB_V120_MODE={b.v120_mode or 'heuristic'}\n")
    return {"json": jpath, "md": mpath}


def apply_best(cfg_path: Path, best: Trial) -> None:
    """Move the winning version to the front of operators.gemm.versions,
    editing only that line (comments and the rest of the file are kept)."""
    text = cfg_path.read_text(encoding="utf-8")
    m = re.search(r"^(\s*versions:\s*)\[([^\]]*)\](.*)$", text, flags=re.M)
    if not m:
        raise RuntimeError(f"no flow-style 'versions: [...]' line in {cfg_path}")
    current = [int(x) for x in m.group(2).split(",") if x.strip()]
    new = [best.version] + [v for v in current if v != best.version]
    line = f"{m.group(1)}[{', '.join(str(v) for v in new)}]{m.group(3)}"
    cfg_path.write_text(text[:m.start()] + line + text[m.end():], encoding="utf-8")


def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(description="Autotune the B200 GEMM ladder through bench_gemm")
    ap.add_argument("--config", default=str(REPO / "config.yaml"))
    ap.add_argument("--bench-bin", default=str(DEFAULT_BENCH))
    ap.add_argument("--versions", default="104,105,107,108,109,120")
    ap.add_argument("--modes", default="RC")
    ap.add_argument("--precisions", default="float16")
    ap.add_argument("--sizes", default="2048,4096,8192")
    ap.add_argument("--shapes", default="", help="extra problems, MxNxK comma separated")
    ap.add_argument("--v120-modes", default="heuristic,pair,wide,pair384,streamk")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--measurement", type=int, default=40)
    ap.add_argument("--top-k", type=int, default=10)
    ap.add_argument("--timeout", type=int, default=1800, help="seconds per bench_gemm run")
    ap.add_argument("--out-dir", default="bench_results")
    ap.add_argument("--apply-best", action="store_true", help="put the best version first in config.yaml")
    ap.add_argument("--dry-run", action="store_true")
    args = ap.parse_args(argv)

    cfg_path = Path(args.config).resolve()
    bench_bin = Path(args.bench_bin).resolve()
    versions = parse_list_int(args.versions)
    modes = parse_list_str(args.modes)
    precisions = parse_list_str(args.precisions)
    problems = [(s, s, s) for s in parse_list_int(args.sizes)] + parse_shapes(args.shapes)
    v120_modes = parse_list_str(args.v120_modes)
    bad = [m for m in v120_modes if m.lower() not in V120_MODES]
    if bad:
        print(f"ERROR: unknown v120 mode(s) {bad}; known: {', '.join(V120_MODES)}", file=sys.stderr)
        return 2
    if not (versions and modes and precisions and problems):
        print("ERROR: empty search space.", file=sys.stderr)
        return 2
    runs = build_grid(versions, modes, precisions, problems, v120_modes)
    print(f"[autotune] {len(runs)} bench_gemm runs")
    if args.dry_run:
        for i, r in enumerate(runs, 1):
            print(f"  {i:03d}: versions={list(r[0])} mode={r[1]} precision={r[2]} problem={r[3]} "
                  f"v120_mode={r[4] or '-'}")
        return 0
    if not cfg_path.exists():
        print(f"ERROR: config file not found: {cfg_path}", file=sys.stderr)
        return 2
    if not bench_bin.exists():
        print(f"ERROR: bench binary not found: {bench_bin} (python -m kebab_b200.build)", file=sys.stderr)
        return 2
    base = load_base(cfg_path)
    trials: List[Trial] = []
    t0 = time.time()
    with tempfile.TemporaryDirectory(prefix="kebab_autotune_") as scratch:
        for i, r in enumerate(runs, 1):
            print(f"[autotune] ({i}/{len(runs)}) versions={list(r[0])} mode={r[1]} precision={r[2]} "
                  f"problem={'x'.join(map(str, r[3]))} v120_mode={r[4] or '-'}", flush=True)
            got = run_one(bench_bin, base, r, args.warmup, args.measurement, args.timeout, Path(scratch))
            for t in got:
                print(f"          v{t.version}: {t.tflops:.1f} TFLOP/s, {t.speedup:.3f}x cuBLAS, "
                      f"{t.latency_ms:.4f} ms", flush=True)
            trials.extend(got)
    if not trials:
        print("ERROR: no successful trials.", file=sys.stderr)
        return 3
    best = max(trials, key=trial_sort_key)
    paths = write_reports(Path(args.out_dir), trials, args.top_k)
    print(f"[autotune] done in {time.time() - t0:.1f}s")
    print(f"[autotune] best: v{best.version} (v120 mode {best.v120_mode or '-'}) {best.mode} {best.precision} "
          f"{best.M}x{best.N}x{best.K}: {best.tflops:.1f} TFLOP/s, {best.speedup:.3f}x cuBLAS")
    print(f"[autotune] report json: {paths['json']}\n[autotune] report md:   {paths['md']}")
    if args.apply_best:
        apply_best(cfg_path, best)
        print(f"[autotune] moved v{best.version} to the front of versions in {cfg_path}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
