// The reference's CuTe-API entry point (kebab/include/kebab/cute/gemm.h:64,
// kebab/lib/cute/cute_gemm.cu:25-179) as a thin alias over the B200 ladder, so
// that callers such as kebab/lib/examples/simple_gemm.cu:35 keep working.
// Same opmode rule as the reference's CuTe path: <lhs><rhs> with R/C,
// a missing rhs meaning 'R' ("default" is taken as "RR"); C is column-major
// (ldC = M), as the reference's CuTe kernels store it. The reference's CuTe
// versions (1..3: WGMMA without/with TMA) all resolve to the decomposition
// heuristic (rung 120). Accumulation is FP32 (the reference's CuTe kernels
// accumulated in FP16). Errors are printed, as in the reference.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace kebab {
namespace cute {

template <typename T>
void gemm(const T* A, const T* B, T* C, int M, int N, int K, const char* opmode = "default", int version = 1,
          cudaStream_t stream = 0);

}  // namespace cute
}  // namespace kebab
