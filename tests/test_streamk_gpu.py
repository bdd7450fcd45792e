"""Stream-K rungs (v108 1-CTA, v109 CTA pairs) against the oracle: tile
counts below one wave (every tile split over several CTAs, several
contributors per owner), a partial last wave after full waves, ragged edges,
other layouts, repeated launches (flag epochs) and bit-determinism."""
import numpy as np
import pytest

import oracle as O
from gemm_util import assert_close, inputs, run

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("version", [108, 109])
@pytest.mark.parametrize("shape", [(1024, 1024, 512), (2048, 2048, 2048), (264, 520, 1000), (128, 256, 64),
                                   (3072, 2048, 1536)])
def test_streamk_parity(cuda, version, shape):
    M, N, K = shape
    A, B = inputs(M, N, K, seed=M + K, dtype=O.F16)
    assert_close(run(A, B, M, N, K, O.F16, version, cuda), O.gemm(A, B, M, N, K, O.F16), "v%d %s" % (version, shape))


@pytest.mark.parametrize("version", [108, 109])
def test_streamk_bf16_and_repeats(cuda, version):
    M = N = 2048
    K = 1024
    A, B = inputs(M, N, K, seed=4, dtype=O.BF16)
    ref = O.gemm(A, B, M, N, K, O.BF16)
    first = run(A, B, M, N, K, O.BF16, version, cuda)
    assert_close(first, ref, "v%d bf16" % version, O.BF16)
    for _ in range(3):  # later launches see flags left with earlier epochs
        again = run(A, B, M, N, K, O.BF16, version, cuda)
        assert np.array_equal(again.view(np.uint32), first.view(np.uint32))


@pytest.mark.parametrize("version", [108, 109])
def test_streamk_4096_sampled(cuda, version):
    from test_gemm_gpu import _sampled_check
    _sampled_check(4096, 4096, 4096, O.F16, version, cuda, 1 / 64.0, 1 / 64.0, nrows=4, nelem=20000)
