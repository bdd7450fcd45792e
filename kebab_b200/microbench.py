"""Runner of the sm_100a microbenchmark probes (include/kebab/microbench.h):
the role of the reference's mbench_* executables. Prints a table, or one
JSON object with --json.

Usage: python -m kebab_b200.microbench [--json]
"""
import ctypes
import json
import sys

import kebab_b200 as kb


def _L():
    L = kb.lib()
    c = ctypes
    L.kebab_mbench_umma_once.argtypes = [c.c_int, c.c_int, c.POINTER(c.c_float), c.c_int64]
    L.kebab_mbench_umma.argtypes = [c.c_int, c.c_int, c.c_int, c.c_int, c.POINTER(c.c_double),
                                    c.POINTER(c.c_double)]
    L.kebab_mbench_umma_latency.argtypes = [c.c_int, c.POINTER(c.c_double)]
    L.kebab_mbench_umma_sp.argtypes = [c.c_int, c.c_int, c.c_int, c.POINTER(c.c_double), c.POINTER(c.c_double)]
    L.kebab_mbench_tmem_ld.argtypes = [c.c_int, c.POINTER(c.c_double), c.POINTER(c.c_double)]
    L.kebab_mbench_tma_load.argtypes = [c.c_void_p, c.c_int64, c.c_int64, c.c_int, c.POINTER(c.c_double)]
    L.kebab_mbench_tma_ingest.argtypes = [c.c_void_p, c.c_int64, c.c_int64, c.c_int, c.c_int, c.c_int,
                                          c.POINTER(c.c_double), c.POINTER(c.c_double)]
    return L


def umma_once(bf16=False, cta_group=1):
    import numpy as np
    n = 128 * cta_group * 256
    buf = (ctypes.c_float * n)()
    kb.check(_L().kebab_mbench_umma_once(1 if bf16 else 0, cta_group, buf, n))
    return np.frombuffer(buf, dtype=np.float32).reshape(128 * cta_group, 256).copy()


def umma(cta_group=1, n=256, bf16=False, iters=20000):
    t, c = ctypes.c_double(), ctypes.c_double()
    kb.check(_L().kebab_mbench_umma(cta_group, n, 1 if bf16 else 0, iters, ctypes.byref(t), ctypes.byref(c)))
    return t.value, c.value


def umma_sp(cta_group=1, n=256, iters=20000):
    """2:4 sparse MMA throughput: (dense-equivalent TFLOP/s, cycles per instruction)."""
    t, cyc = ctypes.c_double(), ctypes.c_double()
    kb.check(_L().kebab_mbench_umma_sp(cta_group, n, iters, ctypes.byref(t), ctypes.byref(cyc)))
    return t.value, cyc.value


def umma_latency(iters=1000):
    c = ctypes.c_double()
    kb.check(_L().kebab_mbench_umma_latency(iters, ctypes.byref(c)))
    return c.value


def tmem_ld(iters=20000):
    b, t = ctypes.c_double(), ctypes.c_double()
    kb.check(_L().kebab_mbench_tmem_ld(iters, ctypes.byref(b), ctypes.byref(t)))
    return b.value, t.value


def tma_load(buf, box_rows=128):
    rows, cols = buf.shape
    g = ctypes.c_double()
    kb.check(_L().kebab_mbench_tma_load(ctypes.c_void_p(buf.data_ptr()), rows, cols, box_rows, ctypes.byref(g)))
    return g.value


def tma_ingest(buf, box_rows=128, stages=6, passes=20):
    """L2-resident TMA loads: (aggregate GB/s, bytes per SM cycle)."""
    rows, cols = buf.shape
    g, b = ctypes.c_double(), ctypes.c_double()
    kb.check(_L().kebab_mbench_tma_ingest(ctypes.c_void_p(buf.data_ptr()), rows, cols, box_rows, stages, passes,
                                          ctypes.byref(g), ctypes.byref(b)))
    return g.value, b.value


def run_all():
    import torch
    out = {}
    for cg in (1, 2):
        d = umma_once(False, cg)
        out["umma_once_cg%d_ok" % cg] = bool((d == 64.0).all())
    for cg in (1, 2):
        for n in (64, 128, 256):
            t, c = umma(cg, n)
            out["umma_cg%d_n%d" % (cg, n)] = {"tflops": t, "cycles_per_mma": c,
                                              "flops_per_clk_per_sm": 2 * 128 * n * 16 / c}
    for cg in (1, 2):
        for n in (128, 224, 256):
            t, c = umma_sp(cg, n)
            out["umma_sp_cg%d_n%d" % (cg, n)] = {"tflops_dense_equiv": t, "cycles_per_mma": c,
                                                 "dense_equiv_flops_per_clk_per_sm": 2 * 128 * n * 32 / c}
    out["umma_latency_cycles"] = umma_latency()
    b, t = tmem_ld()
    out["tmem_ld"] = {"bytes_per_clk_per_sm": b, "tbps": t}
    buf = torch.empty((1 << 16, 16384), dtype=torch.float16, device="cuda")  # 2 GiB, > L2
    for box in (64, 128, 256):
        out["tma_load_box%d_gbs" % box] = tma_load(buf, box)
    del buf
    small = torch.empty((148 * 256, 512), dtype=torch.float16, device="cuda")  # 37 MiB, stays in L2
    for box in (128, 256):
        for stages in (1, 2, 3, 4, 6):
            if stages * box * 128 > 200 * 1024:
                continue
            g, b = tma_ingest(small, box, stages)
            out["tma_ingest_box%d_stages%d" % (box, stages)] = {"gbs": g, "bytes_per_clk_per_sm": b,
                                                                 "bytes_in_flight": stages * box * 128}
    return out


if __name__ == "__main__":
    res = run_all()
    if "--json" in sys.argv:
        print(json.dumps(res))
    else:
        for k, v in res.items():
            print("%-28s %s" % (k, v))
