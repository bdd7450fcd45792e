// v101: TMA-fed shared-memory staging feeding the legacy mma.sync tensor path.
//
// The first Blackwell idea of the ladder on its own: A and B K-blocks arrive
// by TMA (cp.async.bulk.tensor, 128-byte swizzle) into a 2-stage ring guarded
// by mbarrier transaction counts, while the math still runs as warp-level
// mma.sync.m16n8k16 with register accumulators (ldmatrix from the swizzled
// tiles). This is the baseline the tcgen05 rungs have to beat; it plays the
// role of the reference's TMA + tensor-core v2 kernel
// (kebab/lib/cuda/cuda_gemm_v2_wgmma_tma.cu:115-184) without WGMMA, which
// does not exist on sm_100a.
//
// CTA tile 128 x 128 x 64, 8 warps as 2 (M) x 4 (N), warp tile 64 x 32.
#include "gemm_umma.cuh"
#include "internal.h"

namespace kb {

namespace {
constexpr int BM = 128, BN = 128, BK = 64, STAGES = 2;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
constexpr int SMEM = 1024 + STAGES * (A_BYTES + B_BYTES) + 64;

template <typename T>
struct MmaSync;
template <>
struct MmaSync<__half> {
  __device__ static __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <>
struct MmaSync<__nv_bfloat16> {
  __device__ static __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Byte address of 16-byte chunk `chunk` (0..7) of row `row` in a tile written
// by TMA with 128-byte swizzle (rows of 128 bytes, tile base 1024-aligned).
__device__ __forceinline__ uint32_t sw128(uint32_t base, int row, int chunk) {
  return base + row * 128 + ((chunk ^ (row & 7)) << 4);
}

template <typename T>
__global__ void __launch_bounds__(256, 1)
    gemm_v101_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, T* C, int M,
                     int N, int K, WaitCtx ctx) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * (A_BYTES + B_BYTES));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wm = warp >> 2, wn = warp & 3;  // 2 x 4 warps
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int nkb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  auto issue = [&](int kb) {
    const int s = kb % STAGES;
    mbar_arrive_expect_tx(&full[s], A_BYTES + B_BYTES);
    tma_load_2d(smem + s * (A_BYTES + B_BYTES), &tmA, &full[s], kb * BK, m0);
    tma_load_2d(smem + s * (A_BYTES + B_BYTES) + A_BYTES, &tmB, &full[s], kb * BK, n0);
  };
  if (threadIdx.x == 0) issue(0);

  float acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[i][j][r] = 0.f;

  bool ok = true;
  for (int kb = 0; kb < nkb; ++kb) {
    // Stage (kb+1)%2 was released by the __syncthreads at the end of kb-1.
    if (threadIdx.x == 0 && kb + 1 < nkb) issue(kb + 1);
    const int s = kb % STAGES;
    if (!mbar_wait(&full[s], (uint32_t)((kb / STAGES) & 1), ctx, SITE_FULL)) {
      ok = false;
    }
    if (__syncthreads_or(!ok)) {
      ok = false;
      break;
    }
    const uint32_t aBase = sbase + s * (A_BYTES + B_BYTES);
    const uint32_t bBase = aBase + A_BYTES;
#pragma unroll
    for (int kk = 0; kk < BK / 16; ++kk) {
      uint32_t af[4][4];
#pragma unroll
      for (int mi = 0; mi < 4; ++mi) {
        const int row = wm * 64 + mi * 16 + (lane & 15);
        ldmatrix_x4(sw128(aBase, row, kk * 2 + (lane >> 4)), af[mi][0], af[mi][1], af[mi][2], af[mi][3]);
      }
      uint32_t bf[4][2];
#pragma unroll
      for (int nj = 0; nj < 2; ++nj) {
        const int nrow = wn * 32 + nj * 16 + (lane & 7) + ((lane >> 4) << 3);
        ldmatrix_x4(sw128(bBase, nrow, kk * 2 + ((lane >> 3) & 1)), bf[2 * nj][0], bf[2 * nj][1],
                    bf[2 * nj + 1][0], bf[2 * nj + 1][1]);
      }
#pragma unroll
      for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) MmaSync<T>::mma(acc[mi][ni], af[mi], bf[ni][0], bf[ni][1]);
    }
    __syncthreads();
  }
  if (!ok) {
    // Let the copy that may still be in flight land before the CTA exits.
    if (threadIdx.x == 0) {
      WaitCtx d{ctx.status, 50000000ull};
      for (int kb = 0; kb < nkb && kb < STAGES; ++kb) mbar_wait(&full[kb], 0, d, SITE_DRAIN);
    }
    return;
  }
  // Fragment layout of m16n8: c0,c1 -> (row g, cols 2t, 2t+1); c2,c3 -> row g+8.
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = m0 + wm * 64 + mi * 16 + g + h * 8;
        const int col = n0 + wn * 32 + ni * 8 + 2 * t;
        if (row < M) {
          if (col < N) C[(size_t)col * M + row] = ElemTraits<T>::cvt(acc[mi][ni][2 * h]);
          if (col + 1 < N) C[(size_t)(col + 1) * M + row] = ElemTraits<T>::cvt(acc[mi][ni][2 * h + 1]);
        }
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
  if ((p.N + BN - 1) / BN > 65535) return fail(KEBAB_EINVAL, "grid too large for v101");
  cudaError_t e = cudaFuncSetAttribute(gemm_v101_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  dim3 grid((unsigned)((p.M + BM - 1) / BM), (unsigned)((p.N + BN - 1) / BN));
  gemm_v101_kernel<T><<<grid, 256, SMEM, p.stream>>>(tA, tB, static_cast<T*>(p.C), (int)p.M, (int)p.N, (int)p.K,
                                                     ctx);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm_v101 launch");
  return KEBAB_OK;
}
}  // namespace

int launch_v101_tma_mmasync(const GemmProblem& p) {
  return p.dtype == KEBAB_F16 ? launch<__half>(p) : launch<__nv_bfloat16>(p);
}

}  // namespace kb
