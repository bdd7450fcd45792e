// v105: persistent CTA pairs, tcgen05 cta_group::2, 256 x 256 tiles.
// Kernel: gemm_umma.cuh; host launch template: gemm_umma_launch.cuh.
#include "gemm_umma_launch.cuh"

namespace kb {

int launch_v105_pair(const GemmProblem& p) { return umma_launch::dispatch<2, true, 6>(p); }

}  // namespace kb
