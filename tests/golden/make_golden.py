"""Generates the golden fixtures in tests/golden/ from the REFERENCE's own code
(compiled from its sources into oracle/_ref by oracle/build_oracle.py):

  gemm_golden.npz    initializeMatrix RAND (mt19937 seed 0 and 42, FP16 and
                     BF16) and referenceGemmCpp<float> outputs (RC, col-major C)
                     at small shapes, plus the <=4 "magic" case of
                     runonce_gemm_ref.cu (value = storage index).
  sparse_golden.npz  cutlass_meta_probe.cu's seed-7 16x32 tile and the
                     sparse_mma.cu seed-42 tile: dense A, pruned A, packed A,
                     per-entry positions, CUTLASS interleaved-2 metadata, group
                     codes, row-pair / interleaved-2 ordered metadata; and the
                     prune result of every 4-element magnitude tie pattern.

Run: python tests/golden/make_golden.py (needs the reference tree).
"""
import itertools
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle as O  # noqa: E402
from oracle.build_oracle import build_ref  # noqa: E402


def gemm_fixtures():
    R = O.ref()
    out = {}
    for tag, (M, N, K, seed, dt) in {
        "u0_f16_64": (64, 64, 64, 0, O.F16),
        "u0_f16_96x80x136": (96, 80, 136, 0, O.F16),
        "u42_f16_128": (128, 128, 128, 42, O.F16),
        "u0_bf16_64x48x72": (64, 48, 72, 0, O.BF16),
    }.items():
        A = np.empty(M * K, np.uint16)
        B = np.empty(K * N, np.uint16)
        (R.kbr_init_rand_bf16 if dt == O.BF16 else R.kbr_init_rand_f16)(A, M, K, B, K, N, seed)
        C = np.empty(M * N, np.float32)
        R.kbr_gemm_f32(O.to_float(A, dt), O.to_float(B, dt), C, M, N, K)
        out[tag + "_A"], out[tag + "_B"], out[tag + "_C"] = A, B, C
        out[tag + "_shape"] = np.array([M, N, K, seed, dt], np.int64)
    # Magic 4x4x4 (runonce_gemm_ref.cu:126-168): value = storage index.
    M = N = K = 4
    A = np.arange(M * K, dtype=np.float32)
    B = np.arange(K * N, dtype=np.float32)
    C = np.empty(M * N, np.float32)
    R.kbr_gemm_f32(A, B, C, M, N, K)
    out["magic4_C"] = C
    return out


def tie_patterns():
    """Every weak ordering of 4 magnitudes (75 patterns) as FP16 groups, with
    sign variants and +/-0 — the cases where partial_sort's tie order decides
    which two entries survive."""
    groups = []
    levels = [np.float16(0.0), np.float16(0.25), np.float16(0.5), np.float16(1.0)]
    seen = set()
    for ranks in itertools.product(range(4), repeat=4):
        # normalise to a weak ordering (dense ranks starting at 0)
        uniq = sorted(set(ranks))
        norm = tuple(uniq.index(r) for r in ranks)
        if norm in seen:
            continue
        seen.add(norm)
        mags = [levels[r + (4 - len(uniq))] for r in norm]
        for signs in ((1, 1, 1, 1), (-1, 1, -1, 1), (-1, -1, -1, -1), (1, -1, 1, 1)):
            groups.append([np.float16(s * m) for s, m in zip(signs, mags)])
    groups.append([np.float16(-0.0), np.float16(0.0), np.float16(-0.0), np.float16(0.0)])
    groups.append([np.float16(-0.0), np.float16(0.5), np.float16(0.0), np.float16(-0.5)])
    g = np.array(groups, np.float16)
    pad = (-len(g)) % 128  # whole 16 x 32 tiles (128 groups each)
    g = np.concatenate([g, np.zeros((pad, 4), np.float16)])
    return g.view(np.uint16).reshape(-1, 16, 32), len(seen)


def sparse_fixtures():
    RS = O.ref_sparse()
    RM = O.ref_sparse_mma()
    R = O.ref()
    out = {}
    for tag, seed in (("t7", 7), ("t42", 42)):
        A = np.empty(16 * 32, np.uint16)
        Bdummy = np.empty(32 * 8, np.uint16)
        R.kbr_init_rand_f16(A, 16, 32, Bdummy, 32, 8, seed)
        pruned = np.empty_like(A)
        RS.kbr_prune_16x32(A, pruned)
        packed = np.empty(16 * 16, np.uint16)
        meta = np.empty(16 * 16, np.uint32)
        assert RS.kbr_pack_16x32(pruned, packed, meta) == 1
        cut = np.empty(64, np.uint32)
        RS.kbr_meta_cutlass_16x32(meta, cut)
        codes = np.array([RS.kbr_encode_2of4(int(meta[m * 16 + 2 * g]), int(meta[m * 16 + 2 * g + 1]))
                          for m in range(16) for g in range(8)], np.uint32)
        out[tag + "_dense"], out[tag + "_pruned"], out[tag + "_packed"] = A, pruned, packed
        out[tag + "_meta"], out[tag + "_cutlass"], out[tag + "_codes"] = meta, cut, codes
        if RM is not None:
            rp = np.empty(32, np.uint32)
            il = np.empty(32, np.uint32)
            RM.kbr_sm_meta_rowpair(codes, rp)
            RM.kbr_sm_meta_il2(codes, il)
            out[tag + "_rowpair"], out[tag + "_il2"] = rp, il
    tiles, n = tie_patterns()
    pr = np.empty_like(tiles)
    for t in range(tiles.shape[0]):
        buf = np.empty(16 * 32, np.uint16)
        RS.kbr_prune_16x32(np.ascontiguousarray(tiles[t].reshape(-1)), buf)
        pr[t] = buf.reshape(16, 32)
    out["ties_in"], out["ties_pruned"], out["ties_weak_orderings"] = tiles, pr, np.array([n])
    out["codes_table"] = np.array([[RS.kbr_encode_2of4(i, j) for j in range(4)] for i in range(4)], np.uint32)
    return out


def main():
    build_ref()
    if O.ref() is None or O.ref_sparse() is None:
        raise SystemExit("reference libraries not built (reference tree missing)")
    np.savez_compressed(os.path.join(HERE, "gemm_golden.npz"), **gemm_fixtures())
    np.savez_compressed(os.path.join(HERE, "sparse_golden.npz"), **sparse_fixtures())
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
