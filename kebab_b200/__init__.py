"""kebab_b200 — B200-native (sm_100a) GEMM ladder behind kebab's operator surface.

The product is libkebab_b200.so (kebab_b200/csrc, C ABI in
include/kebab/kebab.h). This module is the Python mirror of that ABI used by
the tests and bench.py: it loads the in-tree library with ctypes and passes
raw device pointers, sizes and the current CUDA stream — PyTorch only
provides device memory and streams. There is no fallback: if the library is
missing or a call fails, an exception is raised.

Layout (reference kebab/include/kebab/cuda/cuda_gemm.h:10-33): opmode "RC",
A is M x K row-major, B is K x N column-major (a torch tensor of shape
[N, K]), C is M x N column-major (a torch tensor of shape [N, M]).
"""
import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
# KEBAB_B200_LIB selects another build of the same library (e.g. an
# instrumented one); the default is the in-tree build.
LIB_PATH = os.environ.get("KEBAB_B200_LIB") or os.path.join(PKG, "lib", "libkebab_b200.so")

F16, BF16, F32 = 0, 1, 2
OK, EINVAL, ENOTSUP, ECUDA, ETIMEOUT, ESPARSE = 0, 22, 95, 1001, 1002, 1003
RUNGS = (1, 101, 102, 103, 104, 105, 106, 107, 108, 109, 110, 111, 112, 141)
HEURISTIC = 120
# Reference version ids and the B200 rung each one maps to.
REFERENCE_ID_MAP = {2: 102, 3: 102, 17: 102, 4: 103, 15: 103, 5: 104, 6: 104, 7: 104, 13: 104, 14: 104,
                    16: 104, 18: 104, 19: 104, 8: 105, 9: 105, 10: 105, 11: 105, 12: 105, 20: 120,
                    41: 141}


class KebabError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__("kebab status %d: %s" % (code, msg))
        self.code = code


_lib = None


def lib():
    """The loaded C ABI (ctypes.CDLL). Raises if the library was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise KebabError(ECUDA, "libkebab_b200.so not built: run `python -m kebab_b200.build` "
                                    "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        c = ctypes
        L.kebab_gemm.argtypes = [c.c_int, c.c_void_p, c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_int64,
                                 c.c_char_p, c.c_int, c.c_void_p]
        L.kebab_gemm.restype = c.c_int
        L.kebab_version_name.argtypes = [c.c_int]
        L.kebab_version_name.restype = c.c_char_p
        L.kebab_resolve_version.argtypes = [c.c_int, c.c_int, c.c_int64, c.c_int64, c.c_int64]
        L.kebab_resolve_version.restype = c.c_int
        L.kebab_list_versions.argtypes = [c.POINTER(c.c_int), c.c_int]
        L.kebab_list_versions.restype = c.c_int
        L.kebab_last_error.argtypes = []
        L.kebab_last_error.restype = c.c_char_p
        L.kebab_device_status.argtypes = [c.c_void_p, c.POINTER(c.c_uint32), c.c_int]
        L.kebab_device_status.restype = c.c_int
        L.kebab_set_wait_timeout_us.argtypes = [c.c_uint64]
        L.kebab_set_wait_timeout_us.restype = c.c_int
        L.kebab_probe_wait_timeout.argtypes = [c.c_void_p, c.c_uint64]
        L.kebab_probe_wait_timeout.restype = c.c_int
        L.kebab_gemm_gated.argtypes = [c.c_int, c.c_void_p, c.c_void_p, c.c_void_p, c.c_int64, c.c_int64,
                                       c.c_int64, c.c_int, c.c_void_p, c.c_int64, c.c_uint32, c.c_void_p]
        L.kebab_gemm_gated.restype = c.c_int
        L.kebab_ipc_export.argtypes = [c.c_void_p, c.c_void_p, c.POINTER(c.c_int64)]
        L.kebab_ipc_export.restype = c.c_int
        L.kebab_ipc_open.argtypes = [c.c_void_p, c.c_int64, c.POINTER(c.c_void_p)]
        L.kebab_ipc_open.restype = c.c_int
        L.kebab_ipc_close.argtypes = [c.c_void_p]
        L.kebab_ipc_close.restype = c.c_int
        L.kebab_flag_write.argtypes = [c.c_void_p, c.c_uint32, c.c_void_p]
        L.kebab_flag_write.restype = c.c_int
        L.kebab_ring_pull.argtypes = [c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_void_p, c.c_uint32,
                                      c.c_void_p, c.c_void_p, c.c_void_p, c.c_void_p, c.c_uint64]
        L.kebab_ring_pull.restype = c.c_int
        L.kebab_chain_push.argtypes = [c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_void_p, c.c_uint32,
                                       c.c_void_p, c.c_void_p, c.c_void_p, c.c_void_p, c.c_uint64]
        L.kebab_chain_push.restype = c.c_int
        L.kebab_clock_probe.argtypes = [c.c_void_p, c.c_int64]
        L.kebab_clock_probe.restype = c.c_int
        L.kebab_shutdown.argtypes = []
        L.kebab_shutdown.restype = None
        _lib = L
    return _lib


def last_error():
    return lib().kebab_last_error().decode()


def check(rc):
    if rc != OK:
        raise KebabError(rc, last_error())
    return rc


def version_name(version):
    return lib().kebab_version_name(version).decode()


def list_versions():
    n = lib().kebab_list_versions(None, 0)
    arr = (ctypes.c_int * n)()
    lib().kebab_list_versions(arr, n)
    return list(arr)


def _dtype_code(t):
    import torch
    if t.dtype == torch.float16:
        return F16
    if t.dtype == torch.bfloat16:
        return BF16
    if t.dtype == torch.float32:
        return F32
    raise KebabError(EINVAL, "unsupported dtype %s" % t.dtype)


def _stream_ptr(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def gemm_raw(dtype, a_ptr, b_ptr, c_ptr, M, N, K, opmode="RC", version=HEURISTIC, stream_ptr=None):
    """Direct C-ABI call with raw device pointers; returns the status code."""
    return lib().kebab_gemm(dtype, a_ptr, b_ptr, c_ptr, M, N, K, opmode.encode() if opmode else None, version,
                            stream_ptr)


def gemm(A, B, C=None, opmode="RC", version=HEURISTIC, stream=None):
    """C = A * B in RC mode through kebab_gemm.

    A: [M, K] row-major tensor; B: [N, K] tensor (B column-major, K x N);
    C: [N, M] tensor (C column-major, M x N), allocated if None. Asynchronous
    on `stream` (default: torch's current stream). Raises KebabError on a
    non-zero status."""
    import torch
    if A.dim() != 2 or B.dim() != 2:
        raise KebabError(EINVAL, "A and B must be 2-D")
    M, K = A.shape
    N, Kb = B.shape
    if Kb != K:
        raise KebabError(EINVAL, "inner dimensions differ: A is %dx%d, B^T is %dx%d" % (M, K, N, Kb))
    if not (A.is_contiguous() and B.is_contiguous()):
        raise KebabError(EINVAL, "A and B must be contiguous")
    if C is None:
        C = torch.empty((N, M), dtype=A.dtype, device=A.device)
    elif tuple(C.shape) != (N, M) or not C.is_contiguous():
        raise KebabError(EINVAL, "C must be a contiguous [N, M] tensor (column-major M x N)")
    if A.dtype != B.dtype or A.dtype != C.dtype:
        raise KebabError(EINVAL, "A, B and C must share a dtype")
    check(gemm_raw(_dtype_code(A), A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, opmode, version,
                   _stream_ptr(stream)))
    return C


def gemm_gated(A, B, C, b_ready, chunk_cols, epoch, version=HEURISTIC, stream=None):
    """kebab_gemm_gated: C = A * B (RC, shapes as gemm()) while B's columns
    arrive in chunks of `chunk_cols`; a tile needing chunk j waits until the
    int32 CUDA tensor b_ready[j] equals `epoch`."""
    M, K = A.shape
    N = B.shape[0]
    check(lib().kebab_gemm_gated(_dtype_code(A), A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, version,
                                 b_ready.data_ptr(), chunk_cols, epoch, _stream_ptr(stream)))
    return C


def flag_write(flag_ptr, value, stream=None):
    """kebab_flag_write: a stream memory operation storing `value` at the
    device address `flag_ptr` after the work already on `stream`."""
    check(lib().kebab_flag_write(ctypes.c_void_p(flag_ptr), value, _stream_ptr(stream)))


def device_status(stream=None, clear=True):
    """(status, raw code) of the device status word; synchronizes `stream`."""
    code = ctypes.c_uint32(0)
    rc = lib().kebab_device_status(_stream_ptr(stream), ctypes.byref(code), 1 if clear else 0)
    return rc, code.value


def set_wait_timeout_us(us):
    check(lib().kebab_set_wait_timeout_us(us))


def clock_probe(buf):
    """Arms the clock probe for this thread's next tcgen05 GEMM launch: `buf`
    is an int64 CUDA tensor of shape [ctas, 4] (None disarms)."""
    if buf is None:
        check(lib().kebab_clock_probe(None, 0))
    else:
        check(lib().kebab_clock_probe(ctypes.c_void_p(buf.data_ptr()), buf.shape[0]))


def clock_probe_mhz(buf):
    """SM clock (MHz) from clock-probe records: `buf` is [ctas, 4] (one
    launch) or [launches, ctas, 4] (one launch per row, each armed with its
    own slice). Per launch, the median over its CTAs of cycles and of
    nanoseconds; over launches, total cycles / total nanoseconds, so the
    figure is the time-weighted clock of the whole loop."""
    import numpy as np
    r = buf.cpu().numpy().astype(np.float64)
    if r.ndim == 2:
        r = r[None]
    cyc, ns, ctas, mhz = 0.0, 0.0, 0, []
    for rec in r:
        rec = rec[(rec[:, 3] > rec[:, 1]) & (rec[:, 2] > rec[:, 0])]
        if rec.shape[0] == 0:
            continue
        c = np.median(rec[:, 2] - rec[:, 0])
        t = np.median(rec[:, 3] - rec[:, 1])
        cyc += c
        ns += t
        ctas = max(ctas, rec.shape[0])
        mhz.append(c / t * 1e3)
    if ns == 0:
        return None
    return {"sm_mhz": cyc / ns * 1e3, "launches": len(mhz), "ctas": ctas,
            "cta_us_median_per_launch": ns / len(mhz) / 1e3, "sm_mhz_min_launch": min(mhz),
            "sm_mhz_max_launch": max(mhz)}


def probe_wait_timeout(timeout_us=1000, stream=None):
    return lib().kebab_probe_wait_timeout(_stream_ptr(stream), timeout_us)


# ----------------------------------------------------------------------------- 2:4 sparsity
def _sp():
    L = lib()
    if not getattr(L, "_sp_typed", False):
        c = ctypes
        for name, args in {
            "kebab_sparse24_prune": [c.c_int, c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_void_p],
            "kebab_sparse24_pack": [c.c_int, c.c_void_p, c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_void_p],
            "kebab_sparse24_group_codes": [c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_void_p],
            "kebab_sparse24_meta_cutlass": [c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_void_p],
            "kebab_sparse24_meta_ordered": [c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_int, c.c_void_p],
            "kebab_sparse24_compress": [c.c_int, c.c_void_p, c.c_void_p, c.c_void_p, c.c_int64, c.c_int64,
                                        c.c_void_p],
            "kebab_gemm_sparse24": [c.c_int, c.c_void_p, c.c_void_p, c.c_void_p, c.c_void_p, c.c_int64, c.c_int64,
                                    c.c_int64, c.c_void_p],
            "kebab_sparse24_tile": [c.c_int64, c.c_int64, c.POINTER(c.c_int), c.POINTER(c.c_int)],
        }.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = c.c_int
        L.kebab_sparse24_e_bytes.argtypes = [c.c_int64, c.c_int64]
        L.kebab_sparse24_e_bytes.restype = c.c_int64
        L._sp_typed = True
    return L


def sparse24_prune(A, out=None, stream=None):
    import torch
    M, K = A.shape
    out = torch.empty_like(A) if out is None else out
    check(_sp().kebab_sparse24_prune(_dtype_code(A), A.data_ptr(), out.data_ptr(), M, K, _stream_ptr(stream)))
    return out


def sparse24_pack(A_pruned, stream=None):
    """-> (A_packed [M, K/2], meta [M, K/2] int32 positions). Raises
    KebabError(ESPARSE) if a group does not hold exactly two non-zeros."""
    import torch
    M, K = A_pruned.shape
    packed = torch.empty((M, K // 2), dtype=A_pruned.dtype, device=A_pruned.device)
    meta = torch.empty((M, K // 2), dtype=torch.int32, device=A_pruned.device)
    check(_sp().kebab_sparse24_pack(_dtype_code(A_pruned), A_pruned.data_ptr(), packed.data_ptr(), meta.data_ptr(),
                                    M, K, _stream_ptr(stream)))
    return packed, meta


def sparse24_group_codes(meta, K, stream=None):
    import torch
    M = meta.shape[0]
    codes = torch.empty((M, K // 4), dtype=torch.int32, device=meta.device)
    check(_sp().kebab_sparse24_group_codes(meta.data_ptr(), codes.data_ptr(), M, K, _stream_ptr(stream)))
    return codes


def sparse24_meta_cutlass(meta, K, stream=None):
    import torch
    M = meta.shape[0]
    out = torch.empty(((M // 16) * (K // 32) * 64,), dtype=torch.int32, device=meta.device)
    check(_sp().kebab_sparse24_meta_cutlass(meta.data_ptr(), out.data_ptr(), M, K, _stream_ptr(stream)))
    return out


def sparse24_meta_ordered(codes, K, rowpair, stream=None):
    import torch
    M = codes.shape[0]
    out = torch.empty(((M // 16) * (K // 32) * 32,), dtype=torch.int32, device=codes.device)
    check(_sp().kebab_sparse24_meta_ordered(codes.data_ptr(), out.data_ptr(), M, K, 1 if rowpair else 0,
                                            _stream_ptr(stream)))
    return out


def sparse24_compress(A_pruned, stream=None):
    """-> (A_packed [M, K/2], E uint8 buffer) operands of gemm_sparse24."""
    import torch
    M, K = A_pruned.shape
    nbytes = _sp().kebab_sparse24_e_bytes(M, K)
    if nbytes < 0:
        raise KebabError(-nbytes, "2:4 compress needs M % 128 == 0 and K % 128 == 0")
    packed = torch.empty((M, K // 2), dtype=A_pruned.dtype, device=A_pruned.device)
    E = torch.empty((nbytes,), dtype=torch.uint8, device=A_pruned.device)
    check(_sp().kebab_sparse24_compress(_dtype_code(A_pruned), A_pruned.data_ptr(), packed.data_ptr(), E.data_ptr(),
                                        M, K, _stream_ptr(stream)))
    return packed, E


def sparse24_tile(M, N):
    """(rows, columns) of the tile kebab_gemm_sparse24 uses for an M x N output."""
    import ctypes as c
    tm, tn = c.c_int(), c.c_int()
    check(_sp().kebab_sparse24_tile(M, N, c.byref(tm), c.byref(tn)))
    return tm.value, tn.value


def gemm_sparse24(A_packed, E, B, C=None, stream=None):
    """C = A * B with A 2:4 sparse (A_packed [M, K/2], E from sparse24_compress),
    B [N, K] (column-major K x N); C [N, M] column-major."""
    import torch
    M, Kh = A_packed.shape
    N, K = B.shape
    if K != 2 * Kh:
        raise KebabError(EINVAL, "A_packed must be [M, K/2]")
    if C is None:
        C = torch.empty((N, M), dtype=B.dtype, device=B.device)
    check(_sp().kebab_gemm_sparse24(_dtype_code(B), A_packed.data_ptr(), E.data_ptr(), B.data_ptr(), C.data_ptr(),
                                    M, N, K, _stream_ptr(stream)))
    return C
