// v103: warp-specialised, one tile per CTA (grid = #tiles).
// Kernel: gemm_umma.cuh; host launch template: gemm_umma_launch.cuh.
#include "gemm_umma_launch.cuh"

namespace kb {

int launch_v103_ws(const GemmProblem& p) { return umma_launch::dispatch<1, false, 4>(p); }

}  // namespace kb
