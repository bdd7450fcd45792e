"""GPU parity of every rung against the CPU oracle (restatement of the
reference's referenceGemmCpp<float>, kebab/include/kebab/utils/
reference_gemm.h:41-92), through the C ABI, under the north-star tolerance:
relative Frobenius error <= 1e-3 and |d| <= 1e-2 * (1 + |ref|) per element.
C is poisoned with NaN before every launch so unwritten tiles fail."""
import numpy as np
import pytest

import oracle as O
from gemm_util import assert_close, inputs, run

pytestmark = pytest.mark.gpu

TC_RUNGS = [101, 102, 103, 104, 105]
ALL_RUNGS = [1] + TC_RUNGS


@pytest.mark.parametrize("version", ALL_RUNGS)
@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
def test_c1_512_uniform(cuda, version, dtype):
    # 512^3, uniform[-1,1] from seed 0 (matrix_init.h RAND).
    M = N = K = 512
    A, B = inputs(M, N, K, seed=0, dtype=dtype, dist=O.UNIFORM)
    ref = O.gemm(A, B, M, N, K, dtype)
    assert_close(run(A, B, M, N, K, dtype, version, cuda), ref, "v%d" % version, dtype)


@pytest.mark.parametrize("version", ALL_RUNGS)
@pytest.mark.parametrize("shape", [(128, 256, 64), (264, 200, 72), (136, 520, 1000), (1024, 128, 8), (8, 8, 8)])
def test_ragged_shapes(cuda, version, shape):
    M, N, K = shape
    A, B = inputs(M, N, K, seed=11, dtype=O.F16)
    ref = O.gemm(A, B, M, N, K, O.F16)
    assert_close(run(A, B, M, N, K, O.F16, version, cuda), ref, "v%d %s" % (version, shape))


@pytest.mark.parametrize("version", [103, 104, 105, 120])
@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
def test_2048_full(cuda, version, dtype):
    M = N = K = 2048
    A, B = inputs(M, N, K, seed=1, dtype=dtype)
    ref = O.gemm(A, B, M, N, K, dtype)
    assert_close(run(A, B, M, N, K, dtype, version, cuda), ref, "v%d" % version, dtype)


@pytest.mark.parametrize("version", [104, 105])
def test_deterministic(cuda, version):
    M, N, K = 1024, 1536, 2048
    A, B = inputs(M, N, K, seed=5)
    c1 = run(A, B, M, N, K, O.F16, version, cuda)
    c2 = run(A, B, M, N, K, O.F16, version, cuda)
    assert np.array_equal(c1.view(np.uint32), c2.view(np.uint32))


def test_reference_ids_map(cuda):
    # Reference version ids dispatch to their B200 rung and stay correct.
    M, N, K = 512, 512, 256
    A, B = inputs(M, N, K, seed=2)
    ref = O.gemm(A, B, M, N, K, O.F16)
    for v in (2, 4, 5, 10, 20):
        assert_close(run(A, B, M, N, K, O.F16, v, cuda), ref, "ref id %d" % v)


def test_timeout_probe(cuda):
    import kebab_b200 as kb
    rc = kb.probe_wait_timeout(2000)
    assert rc == kb.ETIMEOUT
    assert "timed out" in kb.last_error()
    # The context is still usable afterwards and the word was cleared.
    assert kb.device_status()[0] == kb.OK
    M = N = K = 256
    A, B = inputs(M, N, K, seed=3)
    assert_close(run(A, B, M, N, K, O.F16, 104, cuda), O.gemm(A, B, M, N, K, O.F16))
