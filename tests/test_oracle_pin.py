"""Pins the CPU oracle (oracle/kebab_oracle.cpp) to the reference.

1. Against the committed golden fixtures (tests/golden/*.npz, made by
   tests/golden/make_golden.py from the reference's own code): these run
   everywhere, including machines without the reference tree.
2. Against the reference compiled from its sources (oracle/_ref), on fresh
   random cases, where those libraries exist.
"""
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def bits_equal(a, b):
    return np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


@pytest.fixture(scope="module")
def gg():
    return np.load(os.path.join(GOLD, "gemm_golden.npz"))


@pytest.mark.parametrize("tag", ["u0_f16_64", "u0_f16_96x80x136", "u42_f16_128", "u0_bf16_64x48x72"])
def test_golden_init_and_gemm(gg, tag):
    M, N, K, seed, dt = (int(x) for x in gg[tag + "_shape"])
    A, B = O.fill_pair(M, N, K, seed=seed, dtype=dt, dist=O.UNIFORM)
    # initializeMatrix RAND: mt19937(seed), uniform(-1,1), A then B, RNE to FP16/BF16.
    assert np.array_equal(A, gg[tag + "_A"]) and np.array_equal(B, gg[tag + "_B"])
    # referenceGemmCpp<float>, bit for bit.
    assert bits_equal(O.gemm(A, B, M, N, K, dt), gg[tag + "_C"])


def test_golden_magic4(gg):
    # runonce_gemm_ref.cu magic case: value = storage index, exact in FP16.
    vals = np.arange(16, dtype=np.float16).view(np.uint16)
    assert bits_equal(O.gemm(vals, vals, 4, 4, 4, O.F16), gg["magic4_C"])


def test_rows_and_elems_match_full():
    M, N, K = 72, 136, 200
    A, B = O.fill_pair(M, N, K, seed=9, dist=O.NORMAL, scale_a=0.1, scale_b=0.1)
    C = O.gemm(A, B, M, N, K).reshape(N, M)  # column-major
    rows = np.array([0, 5, 71, 33])
    assert bits_equal(O.gemm_rows(A, B, rows, M, N, K), C[:, rows].T.copy())
    ii = np.array([0, 71, 12, 40]); jj = np.array([0, 135, 77, 3])
    assert bits_equal(O.gemm_elems(A, B, ii, jj, M, N, K), C[jj, ii])


def test_normal_generator_moments():
    A, B = O.fill_pair(256, 256, 256, seed=3, dist=O.NORMAL, scale_a=1.0, scale_b=0.02)
    a = O.to_float(A, O.F16); b = O.to_float(B, O.F16)
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1.0) < 0.02
    assert abs(b.std() - 0.02) < 0.001


# --------------------------------------------------------------------------- reference-compiled pins
ref = O.ref()
needs_ref = pytest.mark.skipif(ref is None, reason="oracle/_ref not built (reference tree absent)")


@needs_ref
@pytest.mark.parametrize("shape", [(1, 1, 1), (17, 33, 65), (128, 64, 256), (257, 31, 130), (512, 512, 512)])
@pytest.mark.parametrize("dt", [O.F16, O.BF16])
def test_gemm_bitexact_vs_reference(shape, dt):
    M, N, K = shape
    A, B = O.fill_pair(M, N, K, seed=M + N + K, dtype=dt, dist=O.NORMAL, scale_a=1 / np.sqrt(K),
                       scale_b=1 / np.sqrt(K))
    Cr = np.empty(M * N, np.float32)
    ref.kbr_gemm_f32(O.to_float(A, dt), O.to_float(B, dt), Cr, M, N, K)
    assert bits_equal(O.gemm(A, B, M, N, K, dt), Cr)


@needs_ref
@pytest.mark.parametrize("dt", [O.F16, O.BF16])
def test_init_vs_reference(dt):
    M, N, K = 33, 65, 47
    A, B = O.fill_pair(M, N, K, seed=12345, dtype=dt, dist=O.UNIFORM)
    A2 = np.empty_like(A); B2 = np.empty_like(B)
    (ref.kbr_init_rand_bf16 if dt == O.BF16 else ref.kbr_init_rand_f16)(A2, M, K, B2, K, N, 12345)
    assert np.array_equal(A, A2) and np.array_equal(B, B2)


@needs_ref
def test_conversions_vs_reference():
    L = O.lib()
    rs = np.random.RandomState(0)
    xs = np.concatenate([rs.standard_normal(20000) * 10, rs.standard_normal(20000) * 1e-5,
                         [0.0, -0.0, 65504, 65519.99, 65520, 6e-8, 2.98e-8, 1e30, -np.inf, np.inf]]).astype(np.float32)
    for x in xs:
        assert L.kbo_float_to_half(float(x)) == ref.kbr_float2half(float(x))
        assert L.kbo_float_to_bf16(float(x)) == ref.kbr_float2bf16(float(x))
