// v106: skinny / decode-shaped GEMM (M <= 256), HBM-bound.
//
// For M = 64, N = K = 8192 the work is 8.6 GFLOP but B is 128 MiB: the kernel
// must stream B from HBM at full bandwidth, which needs far more CTAs than the
// 64 output tiles a 128-row M tile would give. Two ideas:
//
//  * swap A and B: C^T = B^T A^T. B (stored N x K, K-major) becomes the MMA's
//    128-row operand and A (M x K row-major, K-major) the N-side operand of
//    width BNM = 64/128/256 >= M. In TMEM the accumulator has lane = n and
//    column = m, so every epilogue thread owns one contiguous run of the
//    column-major C (C[n*M + m], m = 0..M-1): plain vector stores.
//  * split K across a thread-block cluster of S CTAs (S = 1..8). Each CTA
//    accumulates its K range in TMEM, parks the FP32 partial in its own
//    shared memory, and after a cluster barrier CTA r reduces column slice r
//    over all S partials through distributed shared memory, in rank order
//    (deterministic), and stores it. No global workspace, no atomics.
//
// Reference counterpart: none (the reference has no skinny path; its kernels
// require M % 64 or 128 == 0 and launch one CTA per 64..256-row tile).
#include <algorithm>
#include <cstdlib>

#include "gemm_umma.cuh"
#include "internal.h"

namespace kb {

namespace {
constexpr int BMM = 128;  // MMA M: rows of B^T (= columns n of C) per CTA
constexpr int BK = 64;
constexpr int STAGES = 4;

template <int BNM>
struct SkinnySmem {
  static constexpr int BT_STAGE = BMM * BK * 2;
  static constexpr int A_STAGE = BNM * BK * 2;
  static constexpr int STAGE = BT_STAGE + A_STAGE;
  static constexpr int RING = STAGES * STAGE;
  static constexpr int PSTRIDE = BNM + 4;  // floats per partial row (padding: conflict-free v4 access)
  static constexpr int PARTIAL = BMM * PSTRIDE * 4;
  static_assert(PARTIAL <= RING, "partial buffer reuses the ring");
  static constexpr int OFF_BAR = RING;
  static constexpr int BYTES = RING + (2 * STAGES + 1) * 8 + 16;
  static constexpr int ALLOC = BYTES + 1024;
};

__device__ __forceinline__ float4 ld_cluster_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

template <typename T, int BNM>
__global__ void __launch_bounds__(192, 2)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmBt, const __grid_constant__ CUtensorMap tmA, T* C, int M,
                       int N, int K, int splits, WaitCtx ctx) {
  using L = SkinnySmem<BNM>;
  constexpr uint32_t IDESC = umma_idesc_f16(BMM, BNM, ElemTraits<T>::kBf16);
  constexpr uint32_t TMEM_COLS = BNM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = full + 2 * STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + 2 * STAGES + 1);
  float* partial = reinterpret_cast<float*>(smem);  // valid after the main loop

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = (int)cluster_ctarank();
  const int n0 = (blockIdx.x / splits) * BMM;
  const int kb_total = (K + BK - 1) / BK;
  const int kb_per = (kb_total + splits - 1) / splits;
  const int kb0 = min(kb_total, ks * kb_per);
  const int nkb = min(kb_total, kb0 + kb_per) - kb0;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmBt);
    tma_prefetch_desc(&tmA);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc<1>(tmem_slot, TMEM_COLS);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0 && lane == 0) {
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0; i < nkb; ++i) {
      if (!mbar_wait(&empty[stage], phase ^ 1u, ctx, SITE_EMPTY)) break;
      uint8_t* sBt = smem + stage * L::STAGE;
      mbar_arrive_expect_tx(&full[stage], L::STAGE);
      tma_load_2d(sBt, &tmBt, &full[stage], (kb0 + i) * BK, n0);
      tma_load_2d(sBt + L::BT_STAGE, &tmA, &full[stage], (kb0 + i) * BK, 0);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
  } else if (warp == 1 && lane == 0) {
    int stage = 0;
    uint32_t phase = 0;
    int i = 0;
    for (; i < nkb; ++i) {
      if (!mbar_wait(&full[stage], phase, ctx, SITE_FULL)) break;
      tc_fence_after();
      const uint32_t bt = smem_u32(smem + stage * L::STAGE);
      const uint32_t a = bt + L::BT_STAGE;
#pragma unroll
      for (int k = 0; k < BK / 16; ++k)
        umma_f16_cg1(tmem, umma_desc_sw128(bt + k * 32), umma_desc_sw128(a + k * 32), IDESC, (i | k) != 0 ? 1u : 0u);
      umma_commit_cg1(&empty[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (nkb > 0) umma_commit_cg1(acc_full);  // also drains a partial loop after an abort
  } else if (warp >= 2) {
    // Park this CTA's FP32 partial (lane = n, column = m) in shared memory.
    const int q = warp & 3;
    const int row = q * 32 + lane;
    float* prow = partial + row * L::PSTRIDE;
    if (nkb > 0 && mbar_wait(acc_full, 0, ctx, SITE_TMEM_FULL)) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < BNM / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(prow + c * 32 + j) =
              make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                          __uint_as_float(v[j + 3]));
      }
    } else {
      if (nkb > 0) ok = false;
      for (int j = 0; j < BNM; j += 4) *reinterpret_cast<float4*>(prow + j) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // every partial of the cluster is written and visible

  if (warp >= 2) {
    // Reduce column slice `ks` over the S partials, in rank order.
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int cs = BNM / splits;  // multiple of 8
    const int c0 = ks * cs;
    const int n = n0 + row;
    const uint32_t local = smem_u32(partial + row * L::PSTRIDE + c0);
    T* out = C + (size_t)n * M;
    for (int cc = 0; cc < cs; cc += 8) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      for (int r = 0; r < splits; ++r) {
        const uint32_t ra = mapa_shared(local + cc * 4, (uint32_t)r);
        const float4 x = ld_cluster_v4(ra), y = ld_cluster_v4(ra + 16);
        acc[0] += x.x; acc[1] += x.y; acc[2] += x.z; acc[3] += x.w;
        acc[4] += y.x; acc[5] += y.y; acc[6] += y.z; acc[7] += y.w;
      }
      const int m = c0 + cc;
      if (n < N && m < M) {
        if ((M & 7) == 0) {  // 16-byte aligned run of 8 outputs
          alignas(16) T h[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) h[j] = ElemTraits<T>::cvt(acc[j]);
          *reinterpret_cast<uint4*>(out + m) = *reinterpret_cast<const uint4*>(h);
        } else {
          for (int j = 0; j < 8 && m + j < M; ++j) out[m + j] = ElemTraits<T>::cvt(acc[j]);
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // peers are done reading this CTA's partial
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem, TMEM_COLS);
  }
  (void)ok;
}

template <typename T, int BNM>
int launch(const GemmProblem& p, int splits_override) {
  using L = SkinnySmem<BNM>;
  int rc = check_tma_shapes(p);
  if (rc) return rc;
  if (p.lhs != 'R' || p.rhs != 'C' || p.c_row)
    return fail(KEBAB_ENOTSUP, "this rung implements opmode RC with column-major C only");
  DeviceInfo* dev = nullptr;
  if ((rc = device_info(&dev))) return rc;
  WaitCtx ctx;
  if ((rc = wait_ctx(&ctx))) return rc;
  CUtensorMap tBt, tA;
  if ((rc = make_tmap_2d(&tBt, p.B, p.dtype, p.N, p.K, p.K, BMM, BK, true))) return rc;
  if ((rc = make_tmap_2d(&tA, p.A, p.dtype, p.M, p.K, p.K, BNM, BK, true))) return rc;
  const int64_t tiles = (p.N + BMM - 1) / BMM;
  const int kb_total = (int)((p.K + BK - 1) / BK);
  int splits = splits_override;
  if (splits <= 0) {
    // Enough CTAs for two per SM, in powers of two up to the portable cluster size.
    splits = 1;
    while (splits < 8 && tiles * splits * 2 <= 2LL * dev->sm_count && splits * 2 <= kb_total) splits *= 2;
  }
  if (splits < 1 || splits > 8 || (splits & (splits - 1))) return fail(KEBAB_EINVAL, "splits must be 1, 2, 4 or 8");
  if (tiles * splits > INT32_MAX) return fail(KEBAB_EINVAL, "grid too large for v106");
  auto kern = gemm_skinny_kernel<T, BNM>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles * splits), 1, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = L::ALLOC;
  cfg.stream = p.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tBt, tA, static_cast<T*>(p.C), (int)p.M, (int)p.N, (int)p.K, splits, ctx);
  if (e != cudaSuccess) return cuda_fail(e, "gemm_v106 launch");
  return KEBAB_OK;
}

template <typename T>
int launch_m(const GemmProblem& p, int splits) {
  if (p.M <= 64) return launch<T, 64>(p, splits);
  if (p.M <= 128) return launch<T, 128>(p, splits);
  if (p.M <= 256) return launch<T, 256>(p, splits);
  return fail(KEBAB_EINVAL, "v106 handles M <= 256 (use 104/105 for larger M)");
}
}  // namespace

int launch_v106_skinny_splits(const GemmProblem& p, int splits) {
  return p.dtype == KEBAB_F16 ? launch_m<__half>(p, splits) : launch_m<__nv_bfloat16>(p, splits);
}
// KEBAB_V106_SPLITS (1, 2, 4, 8) overrides the split-K cluster size.
int launch_v106_skinny(const GemmProblem& p) {
  const char* e = std::getenv("KEBAB_V106_SPLITS");
  return launch_v106_skinny_splits(p, (e && *e) ? std::atoi(e) : 0);
}

}  // namespace kb
