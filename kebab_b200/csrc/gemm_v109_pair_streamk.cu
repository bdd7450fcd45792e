// v109: v105 (persistent CTA pairs, 256 x 256 tiles) with stream-K over the
// last partial wave plus one full wave (4096^3: 256 pair tiles on 74 pairs).
// Each CTA of a contributing pair publishes the partial of its own 128 rows;
// the owning pair's CTAs add those of the same rank.
// Kernel: gemm_umma.cuh; host launch template: gemm_umma_launch.cuh.
#include "gemm_umma_launch.cuh"

namespace kb {

int launch_v109_pair_streamk(const GemmProblem& p) { return umma_launch::dispatch<2, true, 6, 256, true>(p); }

}  // namespace kb
