// v108: v104 (persistent, 128 x 256 tiles) with stream-K: the K-iterations
// of the last partial wave plus one full wave are split evenly over the CTAs,
// so shapes whose tile count is not a multiple of the SM count (2048^3: 128
// tiles on 148 SMs) keep every SM busy. Partial tiles are combined through a
// per-CTA FP32 workspace slot and release/acquire flags, in a fixed order.
// Kernel: gemm_umma.cuh; host launch template: gemm_umma_launch.cuh.
#include "gemm_umma_launch.cuh"

namespace kb {

int launch_v108_streamk(const GemmProblem& p) { return umma_launch::dispatch<1, true, 4, 256, true>(p); }

}  // namespace kb

#ifdef KEBAB_SK_TRACE
// Debug builds only: copy this translation unit's stream-K trace to the host.
extern "C" int kebab_debug_sk_trace_v108(void* host, size_t bytes) {
  return (int)cudaMemcpyFromSymbol(host, kb::g_sk_trace, bytes);
}
#endif
