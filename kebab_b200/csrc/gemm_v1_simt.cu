// v1: CUDA-core (SIMT) register-tiled GEMM, the ladder's floor.
//
// Same role as the reference's v1 warp-tiling kernel
// (kebab/lib/cuda/cuda_gemm_v1_warptiling_baseline.cu:32-150): no tensor
// cores, shared-memory tiles, FP32 FMA accumulation, column-major C. Unlike
// the reference it guards every edge, so any M, N, K > 0 works, and it takes
// every storage layout (A and B row- or column-major, C column- or row-major);
// it is the one rung with no alignment or divisibility requirements.
//
// CTA tile 128 x 128 x 16, 256 threads, 8 x 8 outputs per thread.
#include "gemm_umma.cuh"
#include "internal.h"

namespace kb {

namespace {
constexpr int BM = 128, BN = 128, BK = 16, TM = 8, TN = 8;

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) {
  return static_cast<float>(*p);
}

template <typename T>
__global__ void __launch_bounds__(256) gemm_v1_kernel(const T* __restrict__ A, const T* __restrict__ B,
                                                      T* __restrict__ C, int64_t M, int64_t N, int64_t K, int a_row,
                                                      int b_col, int c_row) {
  __shared__ float As[BK][BM + 4];  // As[k][m]
  __shared__ float Bs[BK][BN + 4];  // Bs[k][n]
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;  // 16 x 16 threads, each 8 x 8
  const int64_t m0 = (int64_t)blockIdx.x * BM, n0 = (int64_t)blockIdx.y * BN;
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  for (int64_t k0 = 0; k0 < K; k0 += BK) {
    // A tile: 128 rows x 16 k (row-major A, k contiguous) -> As[k][m]
    for (int e = tid; e < BM * BK; e += 256) {
      const int r = e / BK, k = e % BK;
      const int64_t gm = m0 + r, gk = k0 + k;
      As[k][r] = (gm < M && gk < K) ? ld_f(A + (a_row ? gm * K + gk : gk * M + gm)) : 0.f;
    }
    // B tile: 128 columns x 16 k (column-major B, k contiguous) -> Bs[k][n]
    for (int e = tid; e < BN * BK; e += 256) {
      const int c = e / BK, k = e % BK;
      const int64_t gn = n0 + c, gk = k0 + k;
      Bs[k][c] = (gn < N && gk < K) ? ld_f(B + (b_col ? gn * K + gk : gk * N + gn)) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = As[k][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = Bs[k][tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < TN; ++j) {
    const int64_t gn = n0 + tx * TN + j;
    if (gn >= N) continue;
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int64_t gm = m0 + ty * TM + i;
      if (gm < M) C[c_row ? gm * N + gn : gn * M + gm] = ElemTraits<T>::cvt(acc[i][j]);
    }
  }
}

template <typename T>
int launch(const GemmProblem& p) {
  DeviceInfo* d = nullptr;
  int rc = device_info(&d);
  if (rc) return rc;
  const int64_t gx = (p.M + BM - 1) / BM, gy = (p.N + BN - 1) / BN;
  if (gx > INT32_MAX || gy > 65535) return fail(KEBAB_EINVAL, "grid too large for v1");
  gemm_v1_kernel<T><<<dim3((unsigned)gx, (unsigned)gy), 256, 0, p.stream>>>(
      static_cast<const T*>(p.A), static_cast<const T*>(p.B), static_cast<T*>(p.C), p.M, p.N, p.K, p.lhs == 'R',
      p.rhs == 'C', p.c_row ? 1 : 0);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm_v1 launch");
  return KEBAB_OK;
}
}  // namespace

int launch_v1_simt(const GemmProblem& p) {
  return p.dtype == KEBAB_F16 ? launch<__half>(p) : launch<__nv_bfloat16>(p);
}

}  // namespace kb
