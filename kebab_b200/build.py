"""Build recipe for libkebab_b200.so (sm_100a only).

Compiles every kebab_b200/csrc/*.cu with
    nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3
in parallel into kebab_b200/_build/, links kebab_b200/lib/libkebab_b200.so
in-tree (so it travels with the repository snapshot), and records the
`-Xptxas -v` resource report in kebab_b200/_build/ptxas.txt.

Usage: python -m kebab_b200.build [--force] [-j N]
"""
import concurrent.futures as cf
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libkebab_b200.so")
HARNESS = os.path.join(PKG, "harness")
BINDIR = os.path.join(PKG, "bin")
HARNESS_BINS = {"bench_gemm": ["bench_gemm.cpp", "config_parser.cpp"],
                "runonce_gemm": ["runonce_gemm.cpp", "config_parser.cpp"],
                "simple_gemm": ["simple_gemm.cpp"]}
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    inc = os.path.join(ROOT, "include")
    for d, _, fs in os.walk(inc):
        hs += [os.path.join(d, f) for f in fs if f.endswith(".h")]
    return hs


def _mtime(p):
    return os.path.getmtime(p) if os.path.exists(p) else 0.0


def _compile(src, force, hdr_time):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if not force and _mtime(obj) > max(_mtime(src), hdr_time):
        return obj, ""
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (os.path.basename(src), r.stdout, r.stderr))
    return obj, r.stderr


def build(force=False, jobs=None, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = _sources()
    hdr_time = max([_mtime(h) for h in _headers()] + [_mtime(__file__)])
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda s: _compile(s, force, hdr_time), srcs))
    objs = [o for o, _ in results]
    report = "".join(log for _, log in results)
    if report:
        with open(os.path.join(BUILD, "ptxas.txt"), "w") as f:
            f.write(report)
    if force or _mtime(LIB) < max(_mtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart_static", "-ldl",
               "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s\n%s" % (r.stdout, r.stderr))
    build_harness(force)
    if verbose:
        print(LIB)
    return LIB


def build_harness(force=False):
    """C++ harness binaries (config.yaml runner, single-launch runner) linked
    against the in-tree library, cuBLAS and the CUDA runtime."""
    os.makedirs(BINDIR, exist_ok=True)
    hdrs = [os.path.join(HARNESS, f) for f in os.listdir(HARNESS) if f.endswith(".h")]
    for name, srcs in HARNESS_BINS.items():
        out = os.path.join(BINDIR, name)
        deps = [os.path.join(HARNESS, s) for s in srcs] + hdrs + [LIB]
        if not force and _mtime(out) > max(_mtime(d) for d in deps):
            continue
        cmd = ["g++", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA_HOME, "include"),
               *[os.path.join(HARNESS, s) for s in srcs], "-o", out, "-L", LIBDIR, "-lkebab_b200",
               "-L", os.path.join(CUDA_HOME, "lib64"), "-lcublas", "-lcudart", "-Wl,-rpath,$ORIGIN/../lib",
               "-Wl,-rpath," + os.path.join(CUDA_HOME, "lib64")]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("harness build failed for %s:\n%s\n%s" % (name, r.stdout, r.stderr))


if __name__ == "__main__":
    j = None
    if "-j" in sys.argv:
        j = int(sys.argv[sys.argv.index("-j") + 1])
    build(force="--force" in sys.argv, jobs=j, verbose=True)
