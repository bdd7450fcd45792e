"""Text summaries of benchmark and profiler output: the role of the
reference's ``scripts/generate_report.py`` (bench CSV -> Markdown),
``make report`` (``Makefile:1347-1411``, ncu report -> text) and
``scripts/profile_gemm.sh:52-68`` (the metric list it asks ncu for).

Three inputs, one Markdown table each, small enough to commit:

``csv``
    bench_gemm CSVs (columns Operator, Variant, BatchSize, Latency(ms),
    Throughput(GFLOPS) or Throughput(GB/s), Speedup): a table per operator and
    problem size, best variant marked.
``launches``
    an ncu launch list (``ncu --metrics gpu__time_duration.sum --csv
    --log-file F``, one metric per row): per kernel its launches, total time
    and share of the total. Per-launch times under ncu are cold-cache and
    serialised, so the share is the comparable figure.
``ncu``
    an ncu report (``.ncu-rep``, exported with ``ncu -i R --page raw --csv``)
    or that CSV: per captured launch the figures a roofline needs (duration,
    SM clock, tensor-pipe %, DRAM bytes and throughput, L2 hit rate, registers,
    launch shape), plus achieved TFLOP/s and DRAM traffic over algorithmic
    bytes when ``--flops`` / ``--bytes`` are given.

No SASS or PTX is read or printed.

Usage::

    python -m kebab_b200.report csv bench_results/*.csv
    python -m kebab_b200.report launches launches.csv --title "bench 8192^3"
    python -m kebab_b200.report ncu prof.ncu-rep --flops 1.0995e12 --bytes 402653184
"""
from __future__ import annotations

import argparse
import csv
import io
import re
import subprocess
import sys
from collections import OrderedDict
from pathlib import Path
from typing import Dict, Iterable, List, Optional, Sequence

# Metric names asked for by the profiling recipe and shown by the ncu table,
# in display order: (metric, label, scale, unit shown).
NCU_FIELDS = [
    ("gpu__time_duration.sum", "duration", 1.0, None),
    ("sm__cycles_elapsed.avg.per_second", "SM clock", 1.0, None),
    ("sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed", "tensor pipe % (elapsed)", 1.0, "%"),
    ("sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active", "tensor pipe % (active)", 1.0, "%"),
    ("dram__bytes_read.sum", "DRAM read", 1.0, None),
    ("dram__bytes_write.sum", "DRAM write", 1.0, None),
    ("gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed", "DRAM throughput %", 1.0, "%"),
    ("lts__t_sector_hit_rate.pct", "L2 hit rate %", 1.0, "%"),
    ("sm__throughput.avg.pct_of_peak_sustained_elapsed", "SM throughput %", 1.0, "%"),
    ("sm__warps_active.avg.pct_of_peak_sustained_active", "warps active %", 1.0, "%"),
    ("launch__registers_per_thread", "registers/thread", 1.0, ""),
    ("launch__grid_size", "grid", 1.0, ""),
    ("launch__block_size", "block", 1.0, ""),
    ("launch__cluster_dim_x", "cluster x", 1.0, ""),
    ("launch__shared_mem_per_block_dynamic", "dynamic smem/block", 1.0, None),
    ("smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio", "stall long scoreboard", 1.0, ""),
    ("smsp__average_warps_issue_stalled_barrier_per_issue_active.ratio", "stall barrier", 1.0, ""),
    ("smsp__average_warps_issue_stalled_wait_per_issue_active.ratio", "stall wait", 1.0, ""),
]

_TIME_SCALE = {"ns": 1e-9, "nsecond": 1e-9, "us": 1e-6, "usecond": 1e-6, "ms": 1e-3, "msecond": 1e-3,
               "s": 1.0, "second": 1.0}
_BYTE_SCALE = {"byte": 1.0, "kbyte": 1e3, "mbyte": 1e6, "gbyte": 1e9, "tbyte": 1e12,
               "kib": 1024.0, "mib": 1024.0 ** 2, "gib": 1024.0 ** 3}
_FREQ_SCALE = {"hz": 1.0, "khz": 1e3, "mhz": 1e6, "ghz": 1e9, "cycle/nsecond": 1e9, "cycle/usecond": 1e6,
               "cycle/second": 1.0}


def _num(s: str) -> Optional[float]:
    s = (s or "").strip().replace(",", "")
    try:
        return float(s)
    except ValueError:
        return None


def to_seconds(value: float, unit: str) -> float:
    return value * _TIME_SCALE.get(unit.strip().lower(), 1.0)


def to_bytes(value: float, unit: str) -> float:
    # "Kbyte/block" and the like: the scale is the part before the slash.
    return value * _BYTE_SCALE.get(unit.strip().lower().split("/")[0], 1.0)


def to_hz(value: float, unit: str) -> float:
    return value * _FREQ_SCALE.get(unit.strip().lower(), 1.0)


def _fmt_time(sec: float) -> str:
    if sec >= 1e-3:
        return f"{sec * 1e3:.3f} ms"
    return f"{sec * 1e6:.1f} us"


def _fmt_bytes(b: float) -> str:
    for unit, scale in (("GB", 1e9), ("MB", 1e6), ("KB", 1e3)):
        if b >= scale:
            return f"{b / scale:.3f} {unit}"
    return f"{b:.0f} B"


def short_kernel_name(name: str, width: int = 90) -> str:
    """Drop the parameter list and shorten namespaces; keep template args."""
    n = name.strip()
    if n.startswith("void "):
        n = n[5:]
    depth, cut = 0, None
    for i, ch in enumerate(n):
        if ch == "<":
            depth += 1
        elif ch == ">":
            depth -= 1
        elif ch == "(" and depth == 0:
            cut = i
            break
    if cut is not None:
        n = n[:cut]
    # Anonymous namespaces, as ncu prints them ("<unnamed>::", and a
    # truncated "unnamed>::" for nested ones).
    n = n.replace("(anonymous namespace)::", "").replace("<unnamed>::", "")
    if n.startswith("unnamed>::"):
        n = n[len("unnamed>::"):]
    return n if len(n) <= width else n[: width - 1] + "…"


def _strip_ncu_noise(text: str) -> str:
    """ncu's --log-file keeps its ==PROF== / ==WARNING== lines ahead of the CSV."""
    return "\n".join(l for l in text.splitlines() if not l.startswith("==") and l.strip())


# --------------------------------------------------------------------------
# bench CSV
# --------------------------------------------------------------------------
def read_bench_rows(paths: Iterable[Path]) -> List[Dict[str, str]]:
    rows = []
    for p in paths:
        with Path(p).open(newline="", encoding="utf-8") as f:
            for r in csv.DictReader(f):
                r = {k.strip(): (v or "").strip() for k, v in r.items() if k}
                r["_file"] = str(p)
                rows.append(r)
    return rows


def bench_csv_markdown(rows: List[Dict[str, str]], title: str = "Benchmark summary") -> str:
    out = io.StringIO()
    out.write(f"# {title}\n\n")
    by_op: "OrderedDict[str, OrderedDict[str, List[Dict[str, str]]]]" = OrderedDict()
    for r in rows:
        by_op.setdefault(r.get("Operator", "?"), OrderedDict()).setdefault(r.get("BatchSize", "?"), []).append(r)
    for op, sizes in by_op.items():
        gb = any("Throughput(GB/s)" in r for s in sizes.values() for r in s)
        tp_key, tp_label = ("Throughput(GB/s)", "GB/s") if gb else ("Throughput(GFLOPS)", "TFLOP/s")
        scale = 1.0 if gb else 1e-3
        out.write(f"## {op}\n\n")
        out.write(f"| size | variant | latency (ms) | {tp_label} | vs comparator | source |\n")
        out.write("|---:|---|---:|---:|---:|---|\n")
        for size, rs in sizes.items():
            best = max(rs, key=lambda r: _num(r.get(tp_key, "0")) or 0.0)
            for r in sorted(rs, key=lambda r: -(_num(r.get(tp_key, "0")) or 0.0)):
                tp = (_num(r.get(tp_key, "0")) or 0.0) * scale
                mark = " **best**" if r is best else ""
                out.write(f"| {size} | `{r.get('Variant', '?')}`{mark} | {_num(r.get('Latency(ms)', '0')) or 0:.4f} "
                          f"| {tp:.1f} | {_num(r.get('Speedup', '0')) or 0:.3f} | {Path(r['_file']).name} |\n")
        out.write("\n")
    return out.getvalue()


# --------------------------------------------------------------------------
# ncu launch list (one metric per row)
# --------------------------------------------------------------------------
def launch_list(text: str) -> "OrderedDict[str, Dict[str, float]]":
    """kernel name -> {launches, total_s}; reads the gpu__time_duration.sum rows."""
    rdr = csv.DictReader(io.StringIO(_strip_ncu_noise(text)))
    agg: "OrderedDict[str, Dict[str, float]]" = OrderedDict()
    for r in rdr:
        if r.get("Metric Name") != "gpu__time_duration.sum":
            continue
        v = _num(r.get("Metric Value", ""))
        if v is None:
            continue
        name = r.get("Kernel Name", "?")
        d = agg.setdefault(name, {"launches": 0, "total_s": 0.0})
        d["launches"] += 1
        d["total_s"] += to_seconds(v, r.get("Metric Unit", "ns"))
    return agg


def launch_list_markdown(agg, title: str = "Launch list", command: Optional[str] = None) -> str:
    total = sum(d["total_s"] for d in agg.values()) or 1.0
    out = io.StringIO()
    out.write(f"# {title}\n\n")
    if command:
        out.write(f"Command:\n\n```\n{command}\n```\n\n")
    out.write("Per kernel: launches, total device time (cold-cache, serialised: compare shares, "
              "not absolutes), share.\n\n")
    out.write("| kernel | launches | total time | per launch | share |\n|---|---:|---:|---:|---:|\n")
    for name, d in sorted(agg.items(), key=lambda kv: -kv[1]["total_s"]):
        out.write(f"| `{short_kernel_name(name)}` | {int(d['launches'])} | {_fmt_time(d['total_s'])} "
                  f"| {_fmt_time(d['total_s'] / max(1, d['launches']))} | {100.0 * d['total_s'] / total:.1f} % |\n")
    return out.getvalue()


# --------------------------------------------------------------------------
# ncu raw page (one launch per row, units in the second row)
# --------------------------------------------------------------------------
def raw_rows(text: str) -> List[Dict[str, tuple]]:
    """Rows of `ncu -i R --page raw --csv`: metric -> (value string, unit)."""
    rows = list(csv.reader(io.StringIO(_strip_ncu_noise(text))))
    if len(rows) < 2:
        return []
    hdr, units = rows[0], rows[1]
    return [{h: (v, u) for h, v, u in zip(hdr, r, units)} for r in rows[2:]]


def raw_from_report(path: Path, ncu: str = "ncu") -> str:
    if path.suffix == ".ncu-rep":
        proc = subprocess.run([ncu, "-i", str(path), "--page", "raw", "--csv"], capture_output=True, text=True,
                              check=False)
        if proc.returncode != 0:
            raise RuntimeError(f"ncu -i {path} failed: {proc.stderr.strip()[:500]}")
        return proc.stdout
    return path.read_text(encoding="utf-8", errors="replace")


def launch_figures(row: Dict[str, tuple], flops: Optional[float] = None,
                   alg_bytes: Optional[float] = None) -> "OrderedDict[str, str]":
    """Display values for one captured launch, plus the derived roofline figures."""
    f: "OrderedDict[str, str]" = OrderedDict()
    dur = None
    if "gpu__time_duration.sum" in row:
        v, u = row["gpu__time_duration.sum"]
        if _num(v) is not None:
            dur = to_seconds(_num(v), u or "ns")
    rd = wr = None
    for metric, label, _, unit in NCU_FIELDS:
        if metric not in row:
            continue
        v, u = row[metric]
        x = _num(v)
        if x is None:
            continue
        if metric == "gpu__time_duration.sum":
            f[label] = _fmt_time(dur)
        elif metric == "sm__cycles_elapsed.avg.per_second":
            f[label] = f"{to_hz(x, u or 'hz') / 1e6:.0f} MHz"
        elif metric.startswith("dram__bytes") or metric.startswith("launch__shared_mem"):
            b = to_bytes(x, u or "byte")
            f[label] = _fmt_bytes(b)
            if metric == "dram__bytes_read.sum":
                rd = b
            elif metric == "dram__bytes_write.sum":
                wr = b
        else:
            f[label] = f"{x:g}{unit if unit else ''}"
    if rd is not None and wr is not None:
        f["DRAM traffic (read+write)"] = f"{rd + wr:.0f} B"
        if alg_bytes:
            f["traffic / algorithmic bytes"] = f"{(rd + wr) / alg_bytes:.3f}"
        if dur:
            f["DRAM GB/s"] = f"{(rd + wr) / dur / 1e9:.0f}"
    if flops and dur:
        f["achieved TFLOP/s (under ncu)"] = f"{flops / dur / 1e12:.1f}"
    if alg_bytes and dur:
        f["achieved algorithmic GB/s (under ncu)"] = f"{alg_bytes / dur / 1e9:.0f}"
    return f


def ncu_markdown(rows: List[Dict[str, tuple]], title: str = "ncu summary", command: Optional[str] = None,
                 flops: Optional[float] = None, alg_bytes: Optional[float] = None) -> str:
    out = io.StringIO()
    out.write(f"# {title}\n\n")
    if command:
        out.write(f"Command:\n\n```\n{command}\n```\n\n")
    if flops:
        out.write(f"Algorithmic FLOPs per launch: {flops:.6g}.\n")
    if alg_bytes:
        out.write(f"Algorithmic DRAM bytes per launch: {alg_bytes:.6g}.\n")
    if flops or alg_bytes:
        out.write("\n")
    for i, row in enumerate(rows):
        name = row.get("Kernel Name", ("?", ""))[0]
        out.write(f"## launch {i}: `{short_kernel_name(name)}`\n\n| figure | value |\n|---|---:|\n")
        for k, v in launch_figures(row, flops, alg_bytes).items():
            out.write(f"| {k} | {v} |\n")
        out.write("\n")
    return out.getvalue()


def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(description="Markdown summaries of bench CSVs and ncu output")
    sub = ap.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("csv", help="bench_gemm CSV files -> Markdown")
    a.add_argument("files", nargs="+")
    a.add_argument("--title", default="Benchmark summary")
    b = sub.add_parser("launches", help="ncu launch-list CSV -> per-kernel shares")
    b.add_argument("file")
    b.add_argument("--title", default="Launch list")
    b.add_argument("--command", default=None, help="the command the list was captured from")
    c = sub.add_parser("ncu", help=".ncu-rep or its raw CSV -> per-launch roofline figures")
    c.add_argument("file")
    c.add_argument("--title", default="ncu summary")
    c.add_argument("--command", default=None)
    c.add_argument("--flops", type=float, default=None, help="algorithmic FLOPs per launch")
    c.add_argument("--bytes", type=float, default=None, help="algorithmic DRAM bytes per launch")
    c.add_argument("--kernel", default=None, help="regex: keep launches whose kernel name matches")
    c.add_argument("--ncu", default="ncu")
    for p in (a, b, c):
        p.add_argument("-o", "--output", default=None)
    args = ap.parse_args(argv)

    if args.cmd == "csv":
        text = bench_csv_markdown(read_bench_rows([Path(f) for f in args.files]), args.title)
    elif args.cmd == "launches":
        agg = launch_list(Path(args.file).read_text(encoding="utf-8", errors="replace"))
        if not agg:
            print("ERROR: no gpu__time_duration.sum rows found", file=sys.stderr)
            return 2
        text = launch_list_markdown(agg, args.title, args.command)
    else:
        rows = raw_rows(raw_from_report(Path(args.file), args.ncu))
        if args.kernel:
            rows = [r for r in rows if re.search(args.kernel, r.get("Kernel Name", ("", ""))[0])]
        if not rows:
            print("ERROR: no launches found", file=sys.stderr)
            return 2
        text = ncu_markdown(rows, args.title, args.command, args.flops, args.bytes)
    if args.output:
        Path(args.output).write_text(text, encoding="utf-8")
    else:
        sys.stdout.write(text)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
