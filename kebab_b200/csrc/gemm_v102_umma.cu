// v102: TMA staging + tcgen05.mma with the accumulator in TMEM, no pipelining.
//
// The second Blackwell idea of the ladder, in its plainest form: one thread
// loads a K-block of A and B with TMA (128-byte swizzle), waits, issues four
// 128 x 128 x 16 tcgen05.mma into a 128-column TMEM accumulator, commits to an
// mbarrier and waits again — load and MMA never overlap. The epilogue reads
// TMEM with tcgen05.ld (32 lanes x 32 columns per warp) and stores C directly
// (column-major, ldC = M). Plays the role of the reference's single-stage
// v2/v3 WGMMA kernels (kebab/lib/cuda/cuda_gemm_v2_wgmma_tma.cu:115-184,
// cuda_gemm_v3_*:282-330).
#include "gemm_umma.cuh"
#include "internal.h"

namespace kb {

namespace {
constexpr int BM = 128, BN = 128, BK = 64;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
// Padded so that at most 3 CTAs share an SM: 3 x 128 TMEM columns fit in 512,
// so tcgen05.alloc never has to wait for another CTA to free columns.
constexpr int SMEM_NEEDED = 1024 + A_BYTES + B_BYTES + 64;
constexpr int SMEM = SMEM_NEEDED > 60 * 1024 ? SMEM_NEEDED : 60 * 1024;

template <typename T>
__global__ void __launch_bounds__(128, 1)
    gemm_v102_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, T* C, int M,
                     int N, int K, WaitCtx ctx) {
  constexpr uint32_t IDESC = umma_idesc_f16(BM, BN, ElemTraits<T>::kBf16);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + A_BYTES;
  uint64_t* tma_bar = reinterpret_cast<uint64_t*>(smem + A_BYTES + B_BYTES);
  uint64_t* mma_bar = tma_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tma_bar + 2);
  int* ok_flag = reinterpret_cast<int*>(tma_bar + 3);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;

  if (threadIdx.x == 0) {
    mbar_init(tma_bar, 1);
    mbar_init(mma_bar, 1);
    fence_barrier_init();
    *ok_flag = 1;
  }
  if (warp == 0) {
    tmem_alloc<1>(tmem_slot, BN);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (threadIdx.x == 0) {
    const int nkb = (K + BK - 1) / BK;
    uint32_t phase = 0;
    for (int kb = 0; kb < nkb; ++kb) {
      mbar_arrive_expect_tx(tma_bar, A_BYTES + B_BYTES);
      tma_load_2d(sA, &tmA, tma_bar, kb * BK, m0);
      tma_load_2d(sB, &tmB, tma_bar, kb * BK, n0);
      if (!mbar_wait(tma_bar, phase, ctx, SITE_TMA_DONE)) {
        WaitCtx d{ctx.status, 50000000ull};
        mbar_wait(tma_bar, phase, d, SITE_DRAIN);
        *ok_flag = 0;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < BK / 16; ++k)
        umma_f16_cg1(tmem, umma_desc_sw128(smem_u32(sA) + k * 32), umma_desc_sw128(smem_u32(sB) + k * 32), IDESC,
                     (kb | k) != 0 ? 1u : 0u);
      umma_commit_cg1(mma_bar);
      if (!mbar_wait(mma_bar, phase, ctx, SITE_MMA_DONE)) {
        WaitCtx d{ctx.status, 50000000ull};
        mbar_wait(mma_bar, phase, d, SITE_DRAIN);
        *ok_flag = 0;
        break;
      }
      phase ^= 1u;
    }
  }
  __syncthreads();
  tc_fence_after();
  if (*ok_flag) {
    const int row = m0 + warp * 32 + lane;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32), v);
      tmem_ld_wait();
      if (row < M) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int col = n0 + c * 32 + j;
          if (col < N) C[(size_t)col * M + row] = ElemTraits<T>::cvt(__uint_as_float(v[j]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc<1>(tmem, BN);
  }
}

template <typename T>
int launch(const GemmProblem& p) {
  int rc = check_tma_shapes(p);
  if (rc) return rc;
  if (p.lhs != 'R' || p.rhs != 'C' || p.c_row)
    return fail(KEBAB_ENOTSUP, "this rung implements opmode RC with column-major C only");
  WaitCtx ctx;
  if ((rc = wait_ctx(&ctx))) return rc;
  CUtensorMap tA, tB;
  if ((rc = make_tmap_2d(&tA, p.A, p.dtype, p.M, p.K, p.K, BM, BK, true))) return rc;
  if ((rc = make_tmap_2d(&tB, p.B, p.dtype, p.N, p.K, p.K, BN, BK, true))) return rc;
  if ((p.M + BM - 1) / BM > INT32_MAX || (p.N + BN - 1) / BN > 65535)
    return fail(KEBAB_EINVAL, "grid too large for v102");
  cudaError_t e = cudaFuncSetAttribute(gemm_v102_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  dim3 grid((unsigned)((p.M + BM - 1) / BM), (unsigned)((p.N + BN - 1) / BN));
  gemm_v102_kernel<T><<<grid, 128, SMEM, p.stream>>>(tA, tB, static_cast<T*>(p.C), (int)p.M, (int)p.N, (int)p.K,
                                                     ctx);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm_v102 launch");
  return KEBAB_OK;
}
}  // namespace

int launch_v102_umma(const GemmProblem& p) {
  return p.dtype == KEBAB_F16 ? launch<__half>(p) : launch<__nv_bfloat16>(p);
}

}  // namespace kb
