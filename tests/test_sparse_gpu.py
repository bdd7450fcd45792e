"""2:4 GPU kernels against the CPU oracle (itself pinned to the reference's
host packers): prune / pack / codes / metadata layouts bit-exact, including
every tie pattern; the sparse GEMM (tcgen05.mma.sp) against the dense
oracle GEMM of the pruned A under the north-star tolerance."""
import os

import numpy as np
import pytest

import oracle as O
from gemm_util import assert_close, to_device, torch_dtype

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _u16(t):
    import torch
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)


def _oracle_prune(A, M, K):
    out = np.empty_like(A)
    assert O.lib().kbo_prune_2of4(A, out, M, K) == 0
    return out


def _dense_fp16(M, K, seed, coarse=False):
    rs = np.random.RandomState(seed)
    if coarse:  # many exact magnitude ties, signs and zeros
        v = (rs.randint(-3, 4, size=M * K) * 0.5).astype(np.float16)
    else:
        v = rs.standard_normal(M * K).astype(np.float16)
    return v.view(np.uint16).copy()


def test_prune_golden_ties(cuda):
    import kebab_b200 as kb
    sg = np.load(os.path.join(GOLD, "sparse_golden.npz"))
    tiles = sg["ties_in"]
    A = to_device(np.ascontiguousarray(tiles.reshape(-1)), (tiles.shape[0] * 16, 32), O.F16, cuda)
    got = _u16(kb.sparse24_prune(A))
    assert np.array_equal(got, sg["ties_pruned"].reshape(-1))


@pytest.mark.parametrize("coarse", [False, True])
def test_prune_pack_codes_layouts(cuda, coarse):
    import torch
    import kebab_b200 as kb
    M, K = 256, 512
    A = _dense_fp16(M, K, seed=3, coarse=coarse)
    want_pr = _oracle_prune(A, M, K)
    Ad = to_device(A, (M, K), O.F16, cuda)
    pr = kb.sparse24_prune(Ad)
    assert np.array_equal(_u16(pr), want_pr)
    packed_want = np.empty(M * K // 2, np.uint16)
    meta_want = np.empty(M * K // 2, np.uint32)
    rc = O.lib().kbo_pack_2of4(want_pr, packed_want, meta_want, M, K)
    if rc != 0:  # coarse data can keep a zero -> both must reject
        with pytest.raises(kb.KebabError) as ei:
            kb.sparse24_pack(pr)
        assert ei.value.code == kb.ESPARSE
        return
    packed, meta = kb.sparse24_pack(pr)
    assert np.array_equal(_u16(packed), packed_want)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32).reshape(-1), meta_want)
    codes = kb.sparse24_group_codes(meta, K)
    codes_want = np.empty(M * K // 4, np.uint32)
    O.lib().kbo_group_codes(meta_want, M, K, codes_want)
    assert np.array_equal(codes.cpu().numpy().view(np.uint32).reshape(-1), codes_want)
    cut = kb.sparse24_meta_cutlass(meta, K).cpu().numpy().view(np.uint32)
    cut_want = np.empty((M // 16) * (K // 32) * 64, np.uint32)
    O.lib().kbo_meta_cutlass_il2(meta_want, M, K, cut_want)
    assert np.array_equal(cut, cut_want)
    for rowpair in (True, False):
        got = kb.sparse24_meta_ordered(codes, K, rowpair).cpu().numpy().view(np.uint32)
        want = np.empty((M // 16) * (K // 32) * 32, np.uint32)
        (O.lib().kbo_meta_rowpair if rowpair else O.lib().kbo_meta_il2_ordered)(codes_want, M, K, want)
        assert np.array_equal(got, want)


def test_pack_rejects_non_24(cuda):
    import kebab_b200 as kb
    A = np.zeros((128, 128), np.float16)
    A[:, 0::4] = 1.0
    A[:, 1::4] = 1.0
    A[5, 8:12] = [1, 1, 1, 0]  # one group with three non-zeros
    with pytest.raises(kb.KebabError) as ei:
        kb.sparse24_pack(to_device(A.view(np.uint16).reshape(-1), (128, 128), O.F16, cuda))
    assert ei.value.code == kb.ESPARSE
    with pytest.raises(kb.KebabError) as ei:
        kb.sparse24_compress(to_device(A.view(np.uint16).reshape(-1), (128, 128), O.F16, cuda))
    assert ei.value.code == kb.ESPARSE


def _sparse_case(cuda, M, N, K, dtype, cg, monkeypatch, seed=0):
    import torch
    import kebab_b200 as kb
    monkeypatch.setenv("KEBAB_SPARSE_CG", str(cg))
    A, B = O.fill_pair(M, N, K, seed=seed, dtype=dtype, dist=O.NORMAL, scale_a=1.0, scale_b=1 / np.sqrt(K))
    Ad = to_device(A, (M, K), dtype, cuda)
    Bd = to_device(B, (N, K), dtype, cuda)
    pr = kb.sparse24_prune(Ad)
    packed, E = kb.sparse24_compress(pr)
    C = torch.full((N, M), float("nan"), dtype=torch_dtype(dtype), device=cuda)
    kb.gemm_sparse24(packed, E, Bd, C)
    torch.cuda.synchronize()
    assert kb.device_status()[0] == kb.OK
    ref = O.gemm(_u16(pr), B, M, N, K, dtype)  # dense oracle GEMM of the pruned A
    assert_close(C.float().cpu().numpy().reshape(-1), ref, "sparse cg%d %dx%dx%d" % (cg, M, N, K), dtype)


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("shape", [(128, 128, 128), (256, 256, 256), (384, 520, 640), (1024, 1024, 2048)])
def test_gemm_sparse24(cuda, cg, shape, monkeypatch):
    _sparse_case(cuda, *shape, O.F16, cg, monkeypatch)


@pytest.mark.parametrize("cg", [1, 2])
def test_gemm_sparse24_bf16(cuda, cg, monkeypatch):
    _sparse_case(cuda, 512, 512, 1024, O.BF16, cg, monkeypatch, seed=2)
