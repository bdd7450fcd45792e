"""Build recipe for the CPU oracle (test infrastructure only).

Outputs:
  oracle/lib/libkebab_oracle.so        the restatement (kebab_oracle.cpp)
  oracle/_ref/libkebab_ref.so          reference_gemm.h + matrix_init.h, compiled
                                       from the reference tree (ref_shim.cpp)
  oracle/_ref/libkebab_ref_sparse.so   cutlass_meta_probe.cu host packers
  oracle/_ref/libkebab_ref_sparse_mma.so  sparse_mma.cu host encoders

The oracle/_ref libraries are built only where the reference tree exists
(KEBAB_REFERENCE_ROOT, else a checkout named `reference` beside this
repository's directory, i.e. ../reference from the repository root); on a
machine without it, previously built files are used as they are.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.environ.get("KEBAB_REFERENCE_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")


def _cutlass_include():
    try:
        import site
        for sp in site.getsitepackages():
            p = os.path.join(sp, "flashinfer", "data", "cutlass", "include")
            if os.path.isdir(p):
                return p
    except Exception:
        pass
    return None


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed: %s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))


def _stale(out, srcs):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs if os.path.exists(s))


def build_oracle(force=False):
    os.makedirs(os.path.join(HERE, "lib"), exist_ok=True)
    src = os.path.join(HERE, "kebab_oracle.cpp")
    out = os.path.join(HERE, "lib", "libkebab_oracle.so")
    if force or _stale(out, [src]):
        _run(["g++", "-std=c++17", "-O3", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
              "-pthread", src, "-o", out])
    return out


def build_ref(force=False):
    """Compile the reference's own CPU code. Returns the list of built libraries."""
    built = []
    if not os.path.isdir(os.path.join(REF_ROOT, "kebab", "include")):
        return built
    refdir = os.path.join(HERE, "_ref")
    os.makedirs(refdir, exist_ok=True)
    inc = ["-I", os.path.join(REF_ROOT, "kebab", "include"), "-I", os.path.join(CUDA_HOME, "include")]
    # 1) reference_gemm.h + matrix_init.h: same flags as the restatement.
    out = os.path.join(refdir, "libkebab_ref.so")
    shim = os.path.join(HERE, "ref_shim.cpp")
    if force or _stale(out, [shim]):
        _run(["g++", "-std=c++17", "-O3", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", *inc,
              shim, "-o", out])
    built.append(out)
    # 2) cutlass_meta_probe.cu host functions (needs CUTLASS layout headers).
    cut = _cutlass_include()
    if cut:
        out = os.path.join(refdir, "libkebab_ref_sparse.so")
        shim = os.path.join(HERE, "ref_sparse_shim.cpp")
        if force or _stale(out, [shim]):
            _run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-x", "c++", *inc, "-I", REF_ROOT,
                  "-I", cut, shim, "-o", out])
        built.append(out)
    # 3) sparse_mma.cu host encoders (CUDA source; device code compiled, never run).
    out = os.path.join(refdir, "libkebab_ref_sparse_mma.so")
    shim = os.path.join(HERE, "ref_sparse_mma_shim.cu")
    if force or _stale(out, [shim]):
        try:
            _run([NVCC, "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC",
                  "-gencode", "arch=compute_100a,code=sm_100a", *inc, "-I", REF_ROOT, shim, "-o", out])
        except RuntimeError as e:  # keep going: the restatement is still pinned by (2)
            sys.stderr.write("warning: sparse_mma.cu shim did not build: %s\n" % str(e)[:400])
            return built
    built.append(out)
    return built


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    print(build_ref(force="--force" in sys.argv))
