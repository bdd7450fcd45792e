"""ctypes front-end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this package, as the checker or the timed CPU baseline. The
GPU product path (kebab_b200) never does.

`lib()` is the restatement (kebab_oracle.cpp); `ref()`, `ref_sparse()` and
`ref_sparse_mma()` are the reference's own code compiled from its sources by
build_oracle.py (None where they were not built).
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
F16, BF16 = 0, 1
UNIFORM, NORMAL = 0, 1

_c = ctypes
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")

_lib = None
_refs = {}


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "lib", "libkebab_oracle.so")
        if not os.path.exists(path):
            from .build_oracle import build_oracle
            build_oracle()
        L = ctypes.CDLL(path)
        L.kbo_fill_pair.argtypes = [_u16p, _c.c_int64, _c.c_int, _c.c_double, _u16p, _c.c_int64, _c.c_int,
                                    _c.c_double, _c.c_uint32, _c.c_int]
        L.kbo_fill_pair.restype = None
        L.kbo_gemm.argtypes = [_u16p, _u16p, _f32p, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int, _c.c_int]
        L.kbo_gemm_rows.argtypes = [_u16p, _u16p, _i64p, _c.c_int64, _f32p, _c.c_int64, _c.c_int64, _c.c_int64,
                                    _c.c_int, _c.c_int]
        L.kbo_gemm_elems.argtypes = [_u16p, _u16p, _i64p, _i64p, _c.c_int64, _f32p, _c.c_int64, _c.c_int64,
                                     _c.c_int64, _c.c_int, _c.c_int]
        L.kbo_float_to_half.argtypes = [_c.c_float]
        L.kbo_float_to_half.restype = _c.c_uint16
        L.kbo_float_to_bf16.argtypes = [_c.c_float]
        L.kbo_float_to_bf16.restype = _c.c_uint16
        L.kbo_prune_2of4.argtypes = [_u16p, _u16p, _c.c_int64, _c.c_int64]
        L.kbo_pack_2of4.argtypes = [_u16p, _u16p, _u32p, _c.c_int64, _c.c_int64]
        L.kbo_encode_2of4.argtypes = [_c.c_int, _c.c_int]
        L.kbo_encode_2of4.restype = _c.c_uint32
        L.kbo_group_codes.argtypes = [_u32p, _c.c_int64, _c.c_int64, _u32p]
        L.kbo_meta_cutlass_il2.argtypes = [_u32p, _c.c_int64, _c.c_int64, _u32p]
        L.kbo_meta_rowpair.argtypes = [_u32p, _c.c_int64, _c.c_int64, _u32p]
        L.kbo_meta_il2_ordered.argtypes = [_u32p, _c.c_int64, _c.c_int64, _u32p]
        _lib = L
    return _lib


def _load_ref(name):
    if name not in _refs:
        path = os.path.join(HERE, "_ref", name)
        _refs[name] = ctypes.CDLL(path) if os.path.exists(path) else None
    return _refs[name]


def ref():
    L = _load_ref("libkebab_ref.so")
    if L is not None and not getattr(L, "_typed", False):
        L.kbr_gemm_f32.argtypes = [_f32p, _f32p, _f32p, _c.c_int, _c.c_int, _c.c_int]
        L.kbr_gemm_f32.restype = None
        L.kbr_init_rand_f16.argtypes = [_u16p, _c.c_int, _c.c_int, _u16p, _c.c_int, _c.c_int, _c.c_uint32]
        L.kbr_init_rand_bf16.argtypes = [_u16p, _c.c_int, _c.c_int, _u16p, _c.c_int, _c.c_int, _c.c_uint32]
        L.kbr_float2half.argtypes = [_c.c_float]
        L.kbr_float2half.restype = _c.c_uint16
        L.kbr_float2bf16.argtypes = [_c.c_float]
        L.kbr_float2bf16.restype = _c.c_uint16
        L._typed = True
    return L


def ref_sparse():
    L = _load_ref("libkebab_ref_sparse.so")
    if L is not None and not getattr(L, "_typed", False):
        L.kbr_prune_16x32.argtypes = [_u16p, _u16p]
        L.kbr_pack_16x32.argtypes = [_u16p, _u16p, _u32p]
        L.kbr_meta_cutlass_16x32.argtypes = [_u32p, _u32p]
        L.kbr_meta_cutlass_decode_16x32.argtypes = [_u32p, _u32p]
        L.kbr_encode_2of4.restype = _c.c_uint32
        L._typed = True
    return L


def ref_sparse_mma():
    L = _load_ref("libkebab_ref_sparse_mma.so")
    if L is not None and not getattr(L, "_typed", False):
        L.kbr_sm_prune.argtypes = [_u16p, _u16p]
        L.kbr_sm_pack.argtypes = [_u16p, _u16p, _u32p]
        L.kbr_sm_meta_rowpair.argtypes = [_u32p, _u32p]
        L.kbr_sm_meta_il2.argtypes = [_u32p, _u32p]
        L.kbr_sm_encode_2of4.restype = _c.c_uint32
        L._typed = True
    return L


# ---------------------------------------------------------------------------
# numpy conveniences
# ---------------------------------------------------------------------------
def fill_pair(M, N, K, seed=0, dtype=F16, dist=UNIFORM, scale_a=1.0, scale_b=1.0, dist_b=None):
    """A (M x K row-major) then B (K x N column-major, stored N x K) from one
    mt19937(seed) stream, as uint16 bit patterns of `dtype`."""
    A = np.empty(M * K, np.uint16)
    B = np.empty(K * N, np.uint16)
    lib().kbo_fill_pair(A, A.size, dist, scale_a, B, B.size, dist if dist_b is None else dist_b, scale_b,
                        seed, dtype)
    return A, B


def gemm(A, B, M, N, K, dtype=F16, threads=0):
    """Oracle C = A*B, FP32, column-major (flat array of M*N, C[j*M + i])."""
    C = np.empty(M * N, np.float32)
    rc = lib().kbo_gemm(np.ascontiguousarray(A), np.ascontiguousarray(B), C, M, N, K, dtype, threads)
    if rc:
        raise ValueError("kbo_gemm rc=%d" % rc)
    return C


def gemm_rows(A, B, rows, M, N, K, dtype=F16, threads=0):
    rows = np.ascontiguousarray(rows, np.int64)
    out = np.empty(rows.size * N, np.float32)
    rc = lib().kbo_gemm_rows(A, B, rows, rows.size, out, M, N, K, dtype, threads)
    if rc:
        raise ValueError("kbo_gemm_rows rc=%d" % rc)
    return out.reshape(rows.size, N)


def gemm_elems(A, B, ii, jj, M, N, K, dtype=F16, threads=0):
    ii = np.ascontiguousarray(ii, np.int64)
    jj = np.ascontiguousarray(jj, np.int64)
    out = np.empty(ii.size, np.float32)
    rc = lib().kbo_gemm_elems(A, B, ii, jj, ii.size, out, M, N, K, dtype, threads)
    if rc:
        raise ValueError("kbo_gemm_elems rc=%d" % rc)
    return out


def to_float(bits, dtype):
    """uint16 bit patterns -> float32 (exact)."""
    bits = np.asarray(bits, np.uint16)
    if dtype == BF16:
        return (bits.astype(np.uint32) << 16).view(np.float32)
    return bits.view(np.float16).astype(np.float32)


def check_tolerance(c_dev, c_ref, rel_fro=1e-3, elem=1e-2):
    """The north-star bar: ||d - r||_F / ||r||_F <= rel_fro and, for every
    element, |d - r| <= elem * (1 + |r|). Returns (ok, rel_fro_err, worst_ratio)."""
    d = np.asarray(c_dev, np.float64)
    r = np.asarray(c_ref, np.float64)
    diff = d - r
    nr = np.linalg.norm(r)
    rel = float(np.linalg.norm(diff) / nr) if nr > 0 else float(np.linalg.norm(diff))
    ratio = np.abs(diff) / (elem * (1.0 + np.abs(r)))
    worst = float(ratio.max()) if ratio.size else 0.0
    ok = bool(rel <= rel_fro and worst <= 1.0 and np.all(np.isfinite(d)))
    return ok, rel, worst
