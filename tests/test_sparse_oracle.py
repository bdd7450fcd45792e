"""2:4 oracle (kbo_prune_2of4 / kbo_pack_2of4 / metadata encoders) pinned to
the reference's host packers (kebab/lib/microbench/sparse_mma.cu:38-166,
cutlass_meta_probe.cu:43-173): golden fixtures everywhere, and the
reference code compiled into oracle/_ref where it exists. Bit-exact."""
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def sg():
    return np.load(os.path.join(GOLD, "sparse_golden.npz"))


def prune(A, M, K):
    out = np.empty_like(A)
    assert O.lib().kbo_prune_2of4(A, out, M, K) == 0
    return out


def pack(As, M, K):
    packed = np.empty(M * K // 2, np.uint16)
    meta = np.empty(M * K // 2, np.uint32)
    rc = O.lib().kbo_pack_2of4(As, packed, meta, M, K)
    return rc, packed, meta


@pytest.mark.parametrize("tag", ["t7", "t42"])
def test_golden_tiles(sg, tag):
    A = sg[tag + "_dense"]
    pr = prune(A, 16, 32)
    assert np.array_equal(pr, sg[tag + "_pruned"])
    rc, packed, meta = pack(pr, 16, 32)
    assert rc == 0 and np.array_equal(packed, sg[tag + "_packed"]) and np.array_equal(meta, sg[tag + "_meta"])
    cut = np.empty(64, np.uint32)
    assert O.lib().kbo_meta_cutlass_il2(meta, 16, 32, cut) == 0
    assert np.array_equal(cut, sg[tag + "_cutlass"])
    codes = np.empty(16 * 8, np.uint32)
    assert O.lib().kbo_group_codes(meta, 16, 32, codes) == 0
    assert np.array_equal(codes, sg[tag + "_codes"])
    if tag + "_rowpair" in sg:
        rp = np.empty(32, np.uint32); il = np.empty(32, np.uint32)
        O.lib().kbo_meta_rowpair(codes, 16, 32, rp)
        O.lib().kbo_meta_il2_ordered(codes, 16, 32, il)
        assert np.array_equal(rp[:16], sg[tag + "_rowpair"][:16]) and np.array_equal(il, sg[tag + "_il2"])


def test_golden_ties(sg):
    # All 75 weak orderings of 4 magnitudes x sign variants, and +/-0 groups.
    assert int(sg["ties_weak_orderings"][0]) == 75
    tiles, expect = sg["ties_in"], sg["ties_pruned"]
    for t in range(tiles.shape[0]):
        assert np.array_equal(prune(np.ascontiguousarray(tiles[t].reshape(-1)), 16, 32), expect[t].reshape(-1))


def test_golden_code_table(sg):
    tab = np.array([[O.lib().kbo_encode_2of4(i, j) for j in range(4)] for i in range(4)], np.uint32)
    assert np.array_equal(tab, sg["codes_table"])


def test_pack_rejects_non_24():
    A = np.zeros(16 * 32, np.float16)
    A[0:4] = [1, 2, 3, 0]  # three non-zeros in group 0
    assert pack(A.view(np.uint16), 16, 32)[0] == 1
    A[0:4] = [1, 0, 0, 0]  # one non-zero
    assert pack(A.view(np.uint16), 16, 32)[0] == 1


RS = O.ref_sparse()
needs_ref = pytest.mark.skipif(RS is None, reason="oracle/_ref not built (reference tree absent)")


@needs_ref
def test_reference_probe_main_passes():
    assert RS.kbr_probe_main() == 0


@needs_ref
@pytest.mark.parametrize("seed", range(20))
def test_random_tiles_vs_reference(seed):
    rs = np.random.RandomState(seed)
    # Coarse values make many magnitude ties inside groups.
    vals = rs.randint(-3, 4, size=16 * 32).astype(np.float16) * np.float16(0.5)
    A = vals.view(np.uint16).copy()
    want = np.empty_like(A)
    RS.kbr_prune_16x32(A, want)
    got = prune(A, 16, 32)
    assert np.array_equal(got, want)
    p1 = np.empty(256, np.uint16); m1 = np.empty(256, np.uint32)
    ok = RS.kbr_pack_16x32(want, p1, m1)
    rc, p2, m2 = pack(got, 16, 32)
    assert (ok == 1) == (rc == 0)
    if ok:
        assert np.array_equal(p1, p2) and np.array_equal(m1, m2)
        c1 = np.empty(64, np.uint32); c2 = np.empty(64, np.uint32)
        RS.kbr_meta_cutlass_16x32(m1, c1)
        O.lib().kbo_meta_cutlass_il2(m2, 16, 32, c2)
        assert np.array_equal(c1, c2)
