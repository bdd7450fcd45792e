// The reference's example (kebab/lib/examples/simple_gemm.cu:17-38) against
// the B200 library: A = ones (row-major), B = row index (row-major), C = A*B
// through the CuTe-API alias in RR mode; every C[i][j] must equal
// sum_k k = K(K-1)/2. Prints PASS/FAIL.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <random>
#include <vector>

#include "harness_common.h"
#include "kebab/cute/gemm.h"

using namespace kebab::harness;

int main() {
  const int M = 256, N = 256, K = 64;
  std::vector<__half> hA(M * K), hB(K * N), hC(M * N);
  std::mt19937 gen(42);
  init_matrix(hA.data(), M, K, InitMode::ONE, gen, 'R');
  init_matrix(hB.data(), K, N, InitMode::ROW, gen, 'R');
  DeviceBuffer<__half> dA(M * K), dB(K * N), dC(M * N);
  dA.upload(hA);
  dB.upload(hB);
  kebab::cute::gemm(dA.p, dB.p, dC.p, M, N, K, "RR");
  CHECK_CUDA(cudaDeviceSynchronize());
  hC = dC.download();
  const float want = K * (K - 1) / 2.0f;
  int bad = 0;
  for (int i = 0; i < M * N; ++i) bad += __half2float(hC[i]) != want;
  std::printf("C[0] = %.1f (want %.1f), mismatches %d: %s\n", __half2float(hC[0]), want, bad, bad ? "FAIL" : "PASS");
  return bad ? 1 : 0;
}
