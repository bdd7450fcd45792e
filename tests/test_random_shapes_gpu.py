"""Seeded random shapes through every tensor-core rung (and the 2:4 sparse
GEMM), against the CPU oracle. The fixed shape lists elsewhere pin the
reference's configs and the obvious edges; this sweep looks for the
non-obvious ones (partial last waves, stream-K splits that leave clusters
without K work, N tails narrower than a sub-MMA, K tails inside a stage).

Shapes: M, N, K multiples of 8 (the TMA pitch rule) up to ~1.5k, so the
oracle finishes each in about a second."""
import numpy as np
import pytest

import oracle as O
from gemm_util import assert_close, inputs, run

pytestmark = pytest.mark.gpu

RUNGS = [103, 104, 105, 106, 107, 108, 109, 110, 111, 112, 120]


def _shapes(n, seed):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        M, N, K = (int(x) * 8 for x in rng.integers(1, 192, size=3))
        out.append((M, N, K))
    return out


SHAPES = _shapes(12, seed=2026)


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "%dx%dx%d" % s)
def test_random_shape_all_rungs(cuda, shape):
    M, N, K = shape
    dtype = O.F16 if (M + N + K) % 16 == 0 else O.BF16
    A, B = inputs(M, N, K, seed=M * 7 + N * 3 + K, dtype=dtype)
    ref = O.gemm(A, B, M, N, K, dtype)
    for version in RUNGS:
        assert_close(run(A, B, M, N, K, dtype, version, cuda), ref, "v%d %dx%dx%d" % (version, M, N, K), dtype)


SPARSE_SHAPES = [(128 * int(a), 8 * int(b), 128 * int(c))
                 for a, b, c in np.random.default_rng(7).integers([1, 1, 1], [9, 160, 9], size=(6, 3))]


@pytest.mark.parametrize("shape", SPARSE_SHAPES, ids=lambda s: "%dx%dx%d" % s)
def test_random_shape_sparse24(cuda, shape):
    import torch

    import kebab_b200 as kb
    from gemm_util import to_device, torch_dtype

    M, N, K = shape
    A, B = O.fill_pair(M, N, K, seed=N, dtype=O.F16, dist=O.NORMAL, scale_a=1.0, scale_b=1 / np.sqrt(K))
    Ad = to_device(A, (M, K), O.F16, cuda)
    Bd = to_device(B, (N, K), O.F16, cuda)
    pr = kb.sparse24_prune(Ad)
    packed, E = kb.sparse24_compress(pr)
    C = torch.full((N, M), float("nan"), dtype=torch_dtype(O.F16), device=cuda)
    kb.gemm_sparse24(packed, E, Bd, C)
    torch.cuda.synchronize()
    pr_bits = pr.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
    ref = O.gemm(pr_bits, B, M, N, K, O.F16)
    assert_close(C.float().cpu().numpy().reshape(-1), ref, "sparse %dx%dx%d" % shape, O.F16)
