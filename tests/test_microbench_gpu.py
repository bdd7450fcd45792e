"""sm_100a microbenchmark probes run, verify their one-shot result and report
plausible numbers (bounded by the B200's nominal limits)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("bf16", [False, True])
def test_umma_once(cuda, cg, bf16):
    from kebab_b200 import microbench as mb
    d = mb.umma_once(bf16, cg)
    assert d.shape == (128 * cg, 256)
    assert np.all(d == 64.0)


@pytest.mark.parametrize("cg", [1, 2])
def test_umma_throughput(cuda, cg):
    from kebab_b200 import microbench as mb
    tflops, cyc = mb.umma(cg, 256, iters=4000)
    # nominal dense FP16 peak 2250 TFLOP/s at boost clock; measured must be real work
    assert 300 < tflops < 2600, tflops
    assert 32 <= cyc <= 2048, cyc


def test_latency_tmem_tma(cuda):
    import torch
    from kebab_b200 import microbench as mb
    lat = mb.umma_latency(200)
    assert 50 < lat < 100000, lat
    b, t = mb.tmem_ld(2000)
    assert b > 1 and t > 1, (b, t)
    buf = torch.empty((1 << 16, 4096), dtype=torch.float16, device=cuda)  # 512 MiB > L2, 442 rows per SM
    for box in (64, 128, 256):
        gbs = mb.tma_load(buf, box)
        assert 500 < gbs < 12000, (box, gbs)


@pytest.mark.parametrize("cg", [1, 2])
def test_umma_sparse_throughput(cuda, cg):
    """tcgen05.mma.sp issue rate: on CTA pairs at N = 256 the 2:4 MMA runs at
    twice the dense rate (dense-equivalent FLOPs); single CTAs reach less."""
    from kebab_b200 import microbench as mb
    sp_tflops, sp_cyc = mb.umma_sp(cg, 256, iters=4000)
    d_tflops, d_cyc = mb.umma(cg, 256, iters=4000)
    assert 300 < sp_tflops < 5200, sp_tflops
    ratio = sp_tflops / d_tflops
    assert (ratio > 1.8) if cg == 2 else (ratio > 1.2), ratio
