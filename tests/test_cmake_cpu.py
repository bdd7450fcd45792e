"""The CMake build (CMakeLists.txt at the repository root): it configures
standalone, every CUDA translation unit is compiled for sm_100a and nothing
else, and a parent project (the way kebab's kebab/lib/CMakeLists.txt would)
can add_subdirectory() it and link the `kebab_b200` target. Configure only:
no GPU and no full build in the CPU suite."""
import glob
import json
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NVCC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")

pytestmark = pytest.mark.skipif(shutil.which("cmake") is None or not os.path.exists(NVCC),
                                reason="cmake or nvcc not available")


def _configure(src, build, *extra):
    r = subprocess.run(["cmake", "-S", src, "-B", build, "-DCMAKE_EXPORT_COMPILE_COMMANDS=ON",
                        "-DCMAKE_CUDA_COMPILER=" + NVCC, *extra], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    with open(os.path.join(build, "compile_commands.json")) as f:
        return json.load(f)


def test_standalone_configure_sm100a_only(tmp_path):
    cmds = _configure(ROOT, str(tmp_path / "b"))
    cu = [c for c in cmds if c["file"].endswith(".cu")]
    srcs = sorted(glob.glob(os.path.join(ROOT, "kebab_b200", "csrc", "*.cu")))
    assert sorted(os.path.realpath(c["file"]) for c in cu) == [os.path.realpath(s) for s in srcs]
    for c in cu:
        cmd = c["command"]
        assert "arch=compute_100a,code=[sm_100a]" in cmd, cmd
        arches = [t for t in cmd.split() if "arch=" in t or t.startswith("-arch")]
        assert len(arches) == 1, arches
    harness = {os.path.basename(c["file"]) for c in cmds if c["file"].endswith(".cpp")}
    assert {"bench_gemm.cpp", "runonce_gemm.cpp", "simple_gemm.cpp", "config_parser.cpp"} <= harness


def test_parent_project_add_subdirectory(tmp_path):
    parent = tmp_path / "parent"
    parent.mkdir()
    (parent / "app.cpp").write_text(
        '#include "kebab/cuda/cuda_gemm.h"\n'
        "int main() { return baseline::gemm_cuda_version_feature_name(120) == nullptr; }\n")
    (parent / "CMakeLists.txt").write_text(
        "cmake_minimum_required(VERSION 3.28)\n"
        "project(parent LANGUAGES CXX CUDA)\n"
        "set(CMAKE_CUDA_ARCHITECTURES 90a)  # the parent's own setting must not leak into the ladder\n"
        "add_subdirectory(%s kebab_b200)\n"
        "add_executable(app app.cpp)\n"
        "target_link_libraries(app PRIVATE kebab_b200::kebab_b200)\n" % ROOT)
    cmds = _configure(str(parent), str(tmp_path / "pb"))
    cu = [c["command"] for c in cmds if c["file"].endswith(".cu")]
    assert cu and all("arch=compute_100a,code=[sm_100a]" in c and "compute_90a" not in c for c in cu)
    app = [c["command"] for c in cmds if c["file"].endswith("app.cpp")]
    assert app and os.path.join(ROOT, "include") in app[0]
    # harness binaries are not built by a parent project unless asked for
    assert not any(c["file"].endswith("bench_gemm.cpp") for c in cmds)
