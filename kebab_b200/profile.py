"""One Nsight Compute capture of one GEMM launch, summarised to Markdown: the
role of the reference's ``make tune-gemm-cuda`` (``Makefile:934-995``: ncu
over the single-launch ``runonce_gemm_cuda`` binary) followed by ``make
report`` (``Makefile:1347-1411``).

What it runs, in order:

1. ``kebab_b200/bin/runonce_gemm`` with the requested problem, plainly; the
   capture happens only if this exits 0 (a profiler run of a program that
   faults can leave the GPU unusable).
2. ``ncu --set <set> --clock-control none -k regex:<kernel> -c <launches>
   -o <out> runonce_gemm ...``: the clocks are never locked, one kernel and at
   most a few launches are captured.
3. ``python -m kebab_b200.report ncu <out>.ncu-rep`` into ``<out>.md`` with
   the algorithmic FLOPs of the launch.

Problems above ``--max-gib`` of operands (A + B + C, default 4 GiB) are
refused: every ncu pass saves and restores device memory, and full-size
captures of large workloads have hung GPUs. Capture a smaller case of the
same kernel instead.

Usage::

    python -m kebab_b200.profile --version 107 --m 4096 --n 4096 --k 4096 --out profiles_run/v107
"""
from __future__ import annotations

import argparse
import shlex
import subprocess
import sys
from pathlib import Path
from typing import List, Optional, Sequence

from kebab_b200 import report

REPO = Path(__file__).resolve().parents[1]
RUNONCE = REPO / "kebab_b200" / "bin" / "runonce_gemm"


def operand_gib(M: int, N: int, K: int) -> float:
    return 2.0 * (M * K + K * N + M * N) / 2 ** 30


def commands(version: int, M: int, N: int, K: int, precision: str, mode: str, out: Path, section_set: str,
             launches: int, kernel_regex: str, ncu: str = "ncu", runonce: Path = RUNONCE) -> List[List[str]]:
    """The plain run and the ncu capture, as argument lists."""
    if launches < 1 or launches > 3:
        raise ValueError("capture 1 to 3 launches")
    plain = [str(runonce), "--version", str(version), "--m", str(M), "--n", str(N), "--k", str(K),
             "--mode", mode, "--precision", precision]
    cap = [ncu, "--set", section_set, "--clock-control", "none", "-k", "regex:" + kernel_regex, "-c",
           str(launches), "-o", str(out), "-f"] + plain
    return [plain, cap]


def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(description="ncu capture of one GEMM launch + Markdown summary")
    ap.add_argument("--version", type=int, default=120)
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--precision", default="float16", choices=["float16", "bfloat16"])
    ap.add_argument("--mode", default="RC")
    ap.add_argument("--set", dest="section_set", default="full")
    ap.add_argument("--launches", type=int, default=1)
    ap.add_argument("--kernel", default="gemm_", help="regex for the kernel name (ncu -k)")
    ap.add_argument("--out", default="profiles_run/capture", help="output stem (.ncu-rep and .md)")
    ap.add_argument("--max-gib", type=float, default=4.0)
    ap.add_argument("--ncu", default="ncu")
    ap.add_argument("--dry-run", action="store_true", help="print the commands only")
    args = ap.parse_args(argv)

    gib = operand_gib(args.m, args.n, args.k)
    if gib > args.max_gib:
        print(f"ERROR: {gib:.1f} GiB of operands exceeds --max-gib {args.max_gib}: capture a smaller case",
              file=sys.stderr)
        return 2
    out = Path(args.out)
    plain, cap = commands(args.version, args.m, args.n, args.k, args.precision, args.mode, out, args.section_set,
                          args.launches, args.kernel, args.ncu)
    if args.dry_run:
        print(shlex.join(plain))
        print(shlex.join(cap))
        return 0
    if not RUNONCE.exists():
        print(f"ERROR: {RUNONCE} not built (python -m kebab_b200.build)", file=sys.stderr)
        return 2
    out.parent.mkdir(parents=True, exist_ok=True)
    r = subprocess.run(plain, capture_output=True, text=True)
    if r.returncode != 0:
        print("plain run failed; not profiling:\n" + r.stdout[-2000:] + r.stderr[-2000:], file=sys.stderr)
        return 3
    r = subprocess.run(cap, capture_output=True, text=True)
    if r.returncode != 0:
        print("ncu failed:\n" + r.stdout[-2000:] + r.stderr[-2000:], file=sys.stderr)
        return 4
    flops = 2.0 * args.m * args.n * args.k
    title = f"{args.kernel} — v{args.version} {args.mode} {args.precision} {args.m}x{args.n}x{args.k}"
    rep = out.with_suffix(".ncu-rep") if out.suffix != ".ncu-rep" else out
    return report.main(["ncu", str(rep), "--flops", str(flops), "--title", title, "--command", shlex.join(cap),
                        "-o", str(out.with_suffix(".md"))])


if __name__ == "__main__":
    raise SystemExit(main())
