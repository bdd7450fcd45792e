// v104: persistent (grid = #SMs), double-buffered accumulators.
// Kernel: gemm_umma.cuh; host launch template: gemm_umma_launch.cuh.
#include "gemm_umma_launch.cuh"

namespace kb {

int launch_v104_persistent(const GemmProblem& p) { return umma_launch::dispatch<1, true, 4>(p); }

}  // namespace kb
