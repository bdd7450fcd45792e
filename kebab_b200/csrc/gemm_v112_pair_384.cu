// v112: persistent CTA pairs with 256 x 384 tiles: two N = 192
// tcgen05.mma.cta_group::2 per k-step share one staged A tile (the v107 idea
// at three quarters of the width). The width exists to fit waves: where
// 256 x 256 tiles fall just past a whole number of waves on the 74 pairs
// (3072 x 2048 x 2048: 96 tiles, 1.3 waves) 256 x 384 tiles fill one wave
// (72 tiles) with fewer operand bytes per FLOP than 256 x 256. Column-major
// (K-major) B only: a sub-MMA starts 96 rows into each CTA's B tile, which an
// MN-major staging of 64-column boxes cannot express.
// Kernel: gemm_umma.cuh; host launch template: gemm_umma_launch.cuh.
#include "gemm_umma_launch.cuh"

namespace kb {

int launch_v112_pair_384(const GemmProblem& p) {
  if (p.rhs == 'R') return fail(KEBAB_ENOTSUP, "rung 112 needs column-major B (opmode RC or CC)");
  const int layout = (p.lhs == 'C' ? LAYOUT_A_MN : 0) | (p.c_row ? LAYOUT_C_ROW : 0);
  switch (layout) {
    case 0: return umma_launch::dispatch_dtype<2, true, 4, 0, 384, false>(p);
    case 1: return umma_launch::dispatch_dtype<2, true, 4, 1, 384, false>(p);
    case 4: return umma_launch::dispatch_dtype<2, true, 4, 4, 384, false>(p);
    default: return umma_launch::dispatch_dtype<2, true, 4, 5, 384, false>(p);
  }
}

}  // namespace kb
