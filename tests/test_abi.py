"""The C-ABI library loads and exports every symbol the public headers
declare, and its host-side validation behaves like the reference operator
(null pointers / bad dims / float / unknown version rejected) — no GPU."""
import ctypes
import os
import re
import subprocess

import pytest

import kebab_b200 as kb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")


def declared_c_functions():
    names = set()
    for d, _, fs in os.walk(INC):
        for f in fs:
            if f.endswith(".h"):
                src = open(os.path.join(d, f)).read()
                names |= set(re.findall(r"\b(kebab_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_library_loads():
    assert os.path.exists(kb.LIB_PATH)
    kb.lib()


@pytest.mark.parametrize("name", declared_c_functions())
def test_c_symbol_exported(name):
    assert hasattr(kb.lib(), name), name


def test_cpp_mirror_symbols_exported():
    out = subprocess.run(["nm", "-DC", kb.LIB_PATH], capture_output=True, text=True).stdout
    src = open(os.path.join(INC, "kebab", "cuda", "cuda_gemm.h")).read()
    rungs = re.findall(r"KEBAB_DECLARE_RUNG\((gemm_\w+)\)", src)
    assert len(rungs) >= 6
    for r in rungs:
        for suf in ("_fp16", "_bf16"):
            assert "baseline::%s%s(" % (r, suf) in out
    assert "baseline::gemm(__half const*" in out
    assert "baseline::gemm(__nv_bfloat16 const*" in out
    assert "baseline::gemm(float const*" in out
    assert "baseline::gemm_cuda_version_feature_name(int)" in out


def test_reference_launcher_aliases_exported():
    """The reference's own launcher names (its cuda_gemm.h:43-257) are exported
    with their reference argument types, and each id maps to a real rung."""
    out = subprocess.run(["nm", "-DC", kb.LIB_PATH], capture_output=True, text=True).stdout
    src = open(os.path.join(INC, "kebab", "cuda", "cuda_gemm.h")).read()
    aliases = re.findall(r"KEBAB_REFERENCE_ALIAS_(F16|BF16)\((gemm_\w+), (\d+)\)", src)
    assert len(aliases) == 16
    for dt, name, vid in aliases:
        elem = "__half" if dt == "F16" else "__nv_bfloat16"
        assert "baseline::%s(%s const*" % (name, elem) in out, name
        assert kb.version_name(int(vid)) != "unknown", name


def test_null_and_dims_rejected():
    L = kb.lib()
    assert L.kebab_gemm(kb.F16, None, None, None, 8, 8, 8, b"RC", 104, None) == kb.EINVAL
    assert "null pointer" in kb.last_error()
    p = ctypes.c_void_p(16)
    assert L.kebab_gemm(kb.F16, p, p, p, 0, 8, 8, b"RC", 104, None) == kb.EINVAL
    assert "invalid dimensions" in kb.last_error()
    assert L.kebab_gemm(kb.F16, p, p, p, 8, -1, 8, b"RC", 104, None) == kb.EINVAL


def test_float_not_implemented():
    p = ctypes.c_void_p(16)
    assert kb.lib().kebab_gemm(kb.F32, p, p, p, 8, 8, 8, b"RC", 104, None) == kb.ENOTSUP
    assert "not implemented" in kb.last_error()


def test_bad_opmode_and_version():
    p = ctypes.c_void_p(16)
    assert kb.lib().kebab_gemm(kb.F16, p, p, p, 8, 8, 8, b"XY", 104, None) == kb.EINVAL
    assert kb.lib().kebab_gemm(kb.F16, p, p, p, 8, 8, 8, b"RC", 999, None) == kb.EINVAL
    assert "unsupported version" in kb.last_error()


def test_version_names_and_mapping():
    assert kb.version_name(104) == "tma_umma_tmem_warpspecialized_persistent"
    assert kb.version_name(999) == "unknown"
    assert kb.version_name(20) == "decomposition_heuristic"
    for ref_id, rung in kb.REFERENCE_ID_MAP.items():
        if rung != 120:
            assert kb.lib().kebab_resolve_version(ref_id, kb.F16, 512, 512, 512) == rung
    assert set(kb.RUNGS) <= set(kb.list_versions())
    assert 120 in kb.list_versions()


def test_v120_heuristic_without_gpu():
    # Falls back to 148 SMs when no device can be queried.
    r = lambda M, N, K: kb.lib().kebab_resolve_version(120, kb.F16, M, N, K)
    assert r(8192, 8192, 8192) == 107 and r(4096, 4096, 8192) == 107 and r(4096, 4096, 4096) == 107
    assert r(16384, 28672, 8192) == 107
    assert r(2048, 28672, 8192) == 107 and r(4096, 28672, 8192) == 107  # config 4a shards on 8 / 4 GPUs
    assert r(4096, 3840, 4096) == 105     # N % 512 != 0: 256 x 256 pair tiles
    assert r(2560, 8192, 4096) == 112     # 256 x 384 pair tiles: 3 waves against 5 (256) and 3 (512)
    assert r(3072, 2048, 2048) == 112 and r(2048, 3072, 4096) == 112  # one wave of 256 x 384
    assert r(3072, 3072, 3072) == 107     # 72 wide tiles: one wave on 74 pairs
    assert r(64, 8192, 8192) == 106 and r(128, 4096, 4096) == 106 and r(64, 2048, 2048) == 106
    assert r(256, 1024, 1024) == 111      # too little of B for the skinny rung
    assert r(2048, 2048, 2048) == 104 and r(4096, 1024, 1024) == 104
    assert r(1536, 1536, 1536) == 110 and r(1280, 1280, 1280) == 110
    assert r(2048, 1024, 4096) == 106 and r(1024, 1024, 8192) == 106 and r(512, 512, 8192) == 106  # split K
    assert r(1024, 1024, 1024) == 111 and r(512, 512, 512) == 111 and r(256, 256, 256) == 111
    assert r(1024, 256, 8192) == 106
    assert r(1536, 1536, 3072) == 106 and r(1536, 1536, 2048) == 110
    assert kb.lib().kebab_resolve_version(120, kb.F16, 4096, 4096, 8192) == 107


def test_sparse24_tile_choice_without_gpu(monkeypatch):
    # 148 SMs assumed when no device can be queried: 74 pairs.
    assert kb.sparse24_tile(8192, 8192) == (512, 224)  # 16 x 37 = 592 tiles = 8 waves
    assert kb.sparse24_tile(4096, 4096) == (512, 240)  # 8 x 18 = 144 tiles, 97 % of 2 waves
    monkeypatch.setenv("KEBAB_SPARSE_BN", "160")
    assert kb.sparse24_tile(8192, 8192) == (512, 160)
    monkeypatch.setenv("KEBAB_SPARSE_CG", "2")
    assert kb.sparse24_tile(8192, 8192) == (256, 256)


@pytest.mark.parametrize("mode,rung", [("dp", 103), ("persistent", 104), ("pair", 105), ("wide", 107),
                                       ("streamk", 109), ("streamk1", 108), ("n128", 110), ("n64", 111),
                                       ("skinny", 106), ("heuristic", 107)])
def test_v120_mode_override(monkeypatch, mode, rung):
    monkeypatch.setenv("KEBAB_V120_MODE", mode)
    assert kb.lib().kebab_resolve_version(120, kb.F16, 8192, 8192, 8192) == rung


def test_shutdown_is_idempotent_without_gpu():
    # Frees workspaces and clears the tensor-map cache; safe to call repeatedly.
    kb.lib().kebab_shutdown()
    kb.lib().kebab_shutdown()
    assert kb.lib().kebab_resolve_version(120, kb.F16, 8192, 8192, 8192) == 107
