"""kebab_gemm_streamk_noalloc — the stream-K GEMM for callers that cannot
allocate device memory (allocator callbacks, fixed-budget serving loops,
plugin hosts that forbid cudaMalloc after start-up). Its output must match
the regular entry point (kebab_gemm, rung 109, which allocates its stream-K
workspace) within the north-star tolerance, on two calls in a row: the
static scratch keeps the previous call's contents, so the second call checks
that nothing stale leaks in. Collected last so that a run stopping at the
first failure has already run every other test."""
import ctypes

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _noalloc():
    import kebab_b200 as kb
    L = kb.lib()
    f = L.kebab_gemm_streamk_noalloc
    f.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                  ctypes.c_int64, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


@pytest.mark.parametrize("shape,dtype", [((4096, 4096, 1024), 0), ((2048, 3072, 512), 1), ((512, 768, 256), 0)])
def test_noalloc_matches_regular_entry_point(cuda, shape, dtype):
    import torch
    import kebab_b200 as kb
    M, N, K = shape
    td = torch.float16 if dtype == 0 else torch.bfloat16
    stream = torch.cuda.current_stream().cuda_stream
    f = _noalloc()
    g = torch.Generator(device=cuda).manual_seed(M + N + K)
    for call in range(2):  # two calls in a row, different inputs
        A = (torch.randn((M, K), generator=g, device=cuda) / K ** 0.5).to(td)
        B = (torch.randn((N, K), generator=g, device=cuda) / K ** 0.5).to(td)
        ref = torch.full((N, M), float("nan"), dtype=td, device=cuda)
        out = torch.full((N, M), float("nan"), dtype=td, device=cuda)
        assert kb.gemm_raw(dtype, A.data_ptr(), B.data_ptr(), ref.data_ptr(), M, N, K, "RC", 109, stream) == kb.OK
        rc = f(dtype, A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K, stream)
        assert rc == kb.OK, kb.last_error()
        torch.cuda.synchronize()
        assert kb.device_status()[0] == kb.OK
        ok, rel, worst = O.check_tolerance(out.float().cpu().numpy().reshape(-1),
                                           ref.float().cpu().numpy().reshape(-1))
        assert ok, "call %d: rel_fro=%.3e worst=%.3f" % (call, rel, worst)


def test_noalloc_rejects_bad_arguments(cuda):
    import kebab_b200 as kb
    f = _noalloc()
    assert f(0, None, None, None, 128, 128, 128, None) == kb.EINVAL
    p = ctypes.c_void_p(256)
    assert f(2, p, p, p, 128, 128, 128, None) == kb.EINVAL
