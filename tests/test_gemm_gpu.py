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

TC_RUNGS = [101, 102, 103, 104, 105, 107, 110, 111, 112]
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


@pytest.mark.parametrize("version", [103, 104, 105, 107, 112, 120])
@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
def test_2048_full(cuda, version, dtype):
    M = N = K = 2048
    A, B = inputs(M, N, K, seed=1, dtype=dtype)
    ref = O.gemm(A, B, M, N, K, dtype)
    assert_close(run(A, B, M, N, K, dtype, version, cuda), ref, "v%d" % version, dtype)


@pytest.mark.parametrize("version", [104, 105, 107])
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


# ----------------------------------------------------------------------------- skinny (v106)
@pytest.mark.parametrize("M", [8, 64, 72, 128, 200, 256])
@pytest.mark.parametrize("splits,fit", [("", ""), ("1", ""), ("2", ""), ("8", ""), ("", "1"), ("2", "1")])
def test_skinny_v106(cuda, M, splits, fit, monkeypatch):
    """fit=1: overlapping 128-row tiles started every < 128 columns."""
    monkeypatch.setenv("KEBAB_V106_SPLITS", splits)
    monkeypatch.setenv("KEBAB_V106_FIT", fit)
    N, K = 1000, 1536
    A, B = inputs(M, N, K, seed=M, dtype=O.F16)
    assert_close(run(A, B, M, N, K, O.F16, 106, cuda), O.gemm(A, B, M, N, K, O.F16), "v106 M=%d s=%s" % (M, splits))


@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
def test_c4b_decode_64x8192x8192(cuda, dtype):
    # BASELINE config 4b: activations N(0,1), weights N(0,0.02), full oracle check.
    M, N, K = 64, 8192, 8192
    A, B = inputs(M, N, K, seed=4, dtype=dtype, scale_a=1.0, scale_b=0.02)
    ref = O.gemm(A, B, M, N, K, dtype)
    for v in (106, 120):
        assert_close(run(A, B, M, N, K, dtype, v, cuda), ref, "v%d" % v, dtype)


# ----------------------------------------------------------------------------- full-size, sampled oracle
def _sampled_check(M, N, K, dtype, version, cuda, scale_a, scale_b, nrows=256, nelem=65536, seed=0):
    """Inputs from a seeded torch generator on the device; the oracle checks
    `nrows` full rows of C (the first, the last and seeded random ones) plus
    `nelem` random elements, on the same input bits: the sampled check the
    parity plan asks for at sizes a full CPU GEMM cannot reach."""
    import torch
    import kebab_b200 as kb
    from gemm_util import round_to, torch_dtype, TOL_ELEM, TOL_REL_FRO, TOL_REL_FRO_BF16_RAW
    g = torch.Generator(device=cuda)
    g.manual_seed(seed)
    td = torch_dtype(dtype)
    A = (torch.randn((M, K), generator=g, device=cuda) * scale_a).to(td)
    B = (torch.randn((N, K), generator=g, device=cuda) * scale_b).to(td)
    C = torch.full((N, M), float("nan"), dtype=td, device=cuda)
    kb.gemm(A, B, C, version=version)
    torch.cuda.synchronize()
    assert kb.device_status()[0] == kb.OK
    rs = np.random.RandomState(seed)
    rows = np.concatenate([[0, M - 1], rs.randint(0, M, nrows - 2)])
    ii = np.concatenate([np.repeat(rows, N), rs.randint(0, M, nelem)])
    jj = np.concatenate([np.tile(np.arange(N), len(rows)), rs.randint(0, N, nelem)])
    Ab = A.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
    Bb = B.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
    ref = O.gemm_elems(Ab, Bb, ii, jj, M, N, K, dtype)
    dev = C[torch.from_numpy(jj).to(cuda), torch.from_numpy(ii).to(cuda)].float().cpu().numpy()
    if dtype == O.BF16:
        ok, rel, _ = O.check_tolerance(dev, ref, TOL_REL_FRO_BF16_RAW, TOL_ELEM)
        assert ok, "raw rel %.3e" % rel
        ref = round_to(ref, dtype)
    ok, rel, worst = O.check_tolerance(dev, ref, TOL_REL_FRO, TOL_ELEM)
    assert ok, "v%d %dx%dx%d: rel_fro=%.3e worst=%.3f" % (version, M, N, K, rel, worst)


@pytest.mark.parametrize("version", [104, 105, 107])
def test_c2_8192_sampled(cuda, version):
    _sampled_check(8192, 8192, 8192, O.F16, version, cuda, 1 / np.sqrt(8192), 1 / np.sqrt(8192))


def test_c4a_prefill_ffn_sampled(cuda):
    # BASELINE config 4a: 16384 x 28672 x 8192, activations N(0,1), weights N(0,0.02).
    _sampled_check(16384, 28672, 8192, O.F16, 120, cuda, 1.0, 0.02)


def test_c3_32768_bf16_sampled(cuda):
    # BASELINE config 3 (one GPU's worth): 32768^3 BF16, N(0,1)/sqrt(K).
    _sampled_check(32768, 32768, 32768, O.BF16, 120, cuda, 1 / np.sqrt(32768), 1 / np.sqrt(32768))
