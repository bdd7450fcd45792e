// v110 / v111: the persistent 1-CTA kernel (v104) with narrower tiles for
// problems whose 128 x 256 tiles would leave SMs idle: 128 x 128 tiles with a
// 6-stage ring (v110) and 128 x 64 tiles with an 8-stage ring (v111), both
// ~192 KB of operands in flight. At 1024^3, 128 x 256 tiles give 32 CTAs on
// 148 SMs; 128 x 64 tiles give 128.
// Kernel: gemm_umma.cuh; host launch template: gemm_umma_launch.cuh.
#include "gemm_umma_launch.cuh"

namespace kb {

// Rings of two K-blocks per stage (v110: 3 x 64 KB, v111: 4 x 48 KB), one
// barrier round trip per two K-blocks. Measured with CUDA-graph replay (no
// host launch cost), TFLOP/s, two K-blocks vs one per stage: v110 1280^3 475
// vs 405, 1536^3 724 vs 607, 2048 x 1024 x 4096 869 vs 702; v111 1024^3 320
// vs 274, 1280^3 327 vs 263. KEBAB_KPS=1 selects the one-K-block rings.
int launch_v110_persistent_n128(const GemmProblem& p) {
  if (kps_env(2) == 1) return umma_launch::dispatch<1, true, 6, 128>(p);
  return umma_launch::dispatch<1, true, 3, 128, false, 2>(p);
}
int launch_v111_persistent_n64(const GemmProblem& p) {
  if (kps_env(2) == 1) return umma_launch::dispatch<1, true, 8, 64>(p);
  return umma_launch::dispatch<1, true, 4, 64, false, 2>(p);
}

}  // namespace kb

#ifdef KEBAB_SK_TRACE
// Debug builds only: copy this translation unit's unit trace to the host.
extern "C" int kebab_debug_sk_trace_v110(void* host, size_t bytes) {
  return (int)cudaMemcpyFromSymbol(host, kb::g_sk_trace, bytes);
}
#endif
