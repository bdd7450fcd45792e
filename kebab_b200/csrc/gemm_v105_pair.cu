// v105: persistent CTA pairs, tcgen05 cta_group::2, 256 x 256 tiles.
// Kernel: gemm_umma.cuh; host launch template: gemm_umma_launch.cuh.
#include "gemm_umma_launch.cuh"

namespace kb {

// Ring: 3 stages of two K-blocks (64 KB per CTA, one barrier round trip per
// two K-blocks). Measured against 6 stages of one K-block (bench.py, 200
// launches, TFLOP/s): 2048^3 941 vs 910, 3072 x 2048 x 2048 926 vs 889,
// 4096^3 1330 vs 1290, 8192^3 1329 vs 1292 (0.954 vs 0.879 of the clock
// peak). KEBAB_KPS=1 selects the 6 x 1 ring.
int launch_v105_pair(const GemmProblem& p) {
  if (kps_env(2) == 1) return umma_launch::dispatch<2, true, 6>(p);
  return umma_launch::dispatch<2, true, 3, 256, false, 2>(p);
}

}  // namespace kb
