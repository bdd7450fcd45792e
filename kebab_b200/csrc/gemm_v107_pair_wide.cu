// v107: persistent CTA pairs with 256 x 512 tiles: two N = 256
// tcgen05.mma.cta_group::2 per k-step share one staged A tile, so each CTA
// loads 48 KB per 64-wide K block for twice the FLOPs of v105 (25 % less
// L2-to-SM traffic per FLOP); the 512-column accumulator is single-buffered.
// Kernel: gemm_umma.cuh; host launch template: gemm_umma_launch.cuh.
#include "gemm_umma_launch.cuh"

namespace kb {

int launch_v107_pair_wide(const GemmProblem& p) { return umma_launch::dispatch<2, true, 4, 512>(p); }

}  // namespace kb
