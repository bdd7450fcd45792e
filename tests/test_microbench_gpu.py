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


def test_tma_ingest_l2(cuda):
    """L2-resident TMA loads: the per-SM intake rises with the bytes in flight
    and stays within physical bounds (the figure is derived from SM cycles)."""
    import torch
    from kebab_b200 import microbench as mb
    small = torch.ones((148 * 256, 512), dtype=torch.float16, device=cuda)  # 37 MiB, stays in L2
    g1, b1 = mb.tma_ingest(small, 128, 1, passes=4)
    g4, b4 = mb.tma_ingest(small, 128, 4, passes=4)
    assert 0.5 < b1 < 1024 and 0.5 < b4 < 1024, (b1, b4)
    assert 100 < g1 < 200000 and 100 < g4 < 200000, (g1, g4)
    assert b4 > b1, (b1, b4)
    import kebab_b200 as kb
    with pytest.raises(kb.KebabError):
        mb.tma_ingest(small, 128, 9)  # more than 8 slots


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
