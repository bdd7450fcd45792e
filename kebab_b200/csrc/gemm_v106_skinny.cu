// v106: skinny / decode-shaped GEMM (M <= 256, HBM-bound), and, tiling M in
// 256-row blocks, the split-K rung for problems with few tiles and a deep K.
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
//    accumulates its K range in TMEM; after a cluster barrier (every ring is
//    drained) it pushes column slice o of its FP32 partial into rank o's
//    shared memory with plain distributed-shared-memory stores, and after a
//    second barrier CTA r reduces slice r over the S partials from its own
//    shared memory, in rank order (deterministic), and stores it. No global
//    workspace, no atomics, and no remote load whose round trip the tail
//    would wait for.
//
// Reference counterpart: none (the reference has no skinny path; its kernels
// require M % 64 or 128 == 0 and launch one CTA per 64..256-row tile).
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "gemm_umma.cuh"
#include "internal.h"

namespace kb {

namespace {
constexpr int BMM = 128;  // MMA M: rows of B^T (= columns n of C) per CTA
constexpr int BK = 64;    // one 128-byte swizzled sub-tile along K

// A stage holds KSUB consecutive 64-wide K sub-tiles of B^T (128 rows) and of
// A (BNM rows): every B^T row is fetched as one KSUB*128-byte run.
//
// The receive area holds the split-K partials peers push: S blocks of
// 128 rows x (BNM/S + 4) floats (the padding keeps 16-byte accesses of a warp
// conflict-free), sized for S <= 8. When it fits beside the ring (SEPARATE)
// peers may push as soon as they are done, while this CTA's ring is still in
// use; otherwise it reuses the ring and a cluster barrier first confirms that
// every ring of the cluster is drained.
template <int BNM, int KSUB, int STAGES>
struct SkinnySmem {
  static constexpr int BT_SUB = BMM * BK * 2;
  static constexpr int A_SUB = BNM * BK * 2;
  static constexpr int STAGE = KSUB * (BT_SUB + A_SUB);
  static constexpr int RING = STAGES * STAGE;
  static constexpr int RECV = BMM * (BNM + 4 * 8) * 4;
  static constexpr int NUM_BARS = 2 * STAGES + 2;
  static constexpr int TAIL = NUM_BARS * 8 + 16;
  static constexpr bool SEPARATE = RING + RECV + TAIL + 1024 <= 232448;
  static constexpr int OFF_RECV = SEPARATE ? RING : 0;
  static constexpr int AREA = SEPARATE ? RING + RECV : (RING > RECV ? RING : RECV);
  static constexpr int OFF_BAR = AREA;
  static constexpr int BYTES = AREA + TAIL;
  static constexpr int ALLOC = BYTES + 1024;
  static constexpr bool FITS = ALLOC <= 232448;
  static_assert(FITS, "shared memory budget exceeded");
  static constexpr int PER_SM = (2 * ALLOC + 2048 <= 233472) ? 2 : 1;
};

#ifdef KEBAB_SK_TRACE
// Debug builds only: per-CTA phase timestamps and SM cycle counts, [cta][16] u64.
__device__ unsigned long long g_skinny_trace[1024 * 32];
#define SKY_TRACE(ev)                                                  \
  do {                                                                 \
    g_skinny_trace[(size_t)blockIdx.x * 32 + (ev)] = globaltimer();    \
    g_skinny_trace[(size_t)blockIdx.x * 32 + 16 + (ev)] = clock64();   \
  } while (0)
#else
#define SKY_TRACE(ev) ((void)0)
#endif

// 16 bytes into a peer's shared memory; the bytes count towards the peer's
// mbarrier transaction (both given as shared::cluster addresses).
__device__ __forceinline__ void st_async_v4(uint32_t dst, uint32_t bar, const uint32_t* v) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   dst),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(bar)
               : "memory");
}

template <typename T, int BNM, int KSUB, int STAGES, int SPLITS>
__global__ void __launch_bounds__(192, 1)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmBt, const __grid_constant__ CUtensorMap tmA, T* C, int M,
                       int N, int K, int step, int pdl, WaitCtx ctx) {
  using L = SkinnySmem<BNM, KSUB, STAGES>;
  constexpr uint32_t IDESC = umma_idesc_f16(BMM, BNM, ElemTraits<T>::kBf16);
  constexpr uint32_t TMEM_COLS = BNM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = full + 2 * STAGES;
  uint64_t* recv_full = full + 2 * STAGES + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + L::NUM_BARS);
  float* recv = reinterpret_cast<float*>(smem + L::OFF_RECV);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = (int)cluster_ctarank();
  // Tiles start every `step` (<= BMM) columns n of C: with step < BMM the
  // 128-row MMA tiles overlap, so that tiles x splits can fill the SMs; each
  // CTA stores only its own `step` rows.
  const int n0 = (blockIdx.x / SPLITS) * step;
  const int m0 = blockIdx.y * BNM;  // M-tile (M > BNM)
  const int kb_total = (K + BK * KSUB - 1) / (BK * KSUB);
  const int kb_per = (kb_total + SPLITS - 1) / SPLITS;
  const int kb0 = min(kb_total, ks * kb_per);
  const int nkb = min(kb_total, kb0 + kb_per) - kb0;
  constexpr int CS = BNM / SPLITS;  // columns m reduced by each rank
  constexpr int RSTRIDE = CS + 4;   // floats per received row
  static_assert(CS % 8 == 0, "each rank reduces whole 16-byte runs");

  if (threadIdx.x == 0) {
    SKY_TRACE(0);
    tma_prefetch_desc(&tmBt);
    tma_prefetch_desc(&tmA);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(recv_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc<1>(tmem_slot, TMEM_COLS);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  // First half of a cluster barrier: the peers wait on it (second half)
  // before they push into this CTA's receive barrier.
  cluster_arrive_release();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Everything above overlaps the previous kernel on the stream (launched
  // with programmatic stream serialisation); A, B and C are touched only
  // after it has completed.
  if (pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }
  bool ok = true;
  if (threadIdx.x == 0) SKY_TRACE(1);

  if (warp == 0 && lane == 0) {
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0; i < nkb; ++i) {
      if (!mbar_wait(&empty[stage], phase ^ 1u, ctx, SITE_EMPTY)) break;
      uint8_t* sBt = smem + stage * L::STAGE;
      uint8_t* sA = sBt + KSUB * L::BT_SUB;
      mbar_arrive_expect_tx(&full[stage], L::STAGE);
      const int k0 = (kb0 + i) * BK * KSUB;
#pragma unroll
      for (int s = 0; s < KSUB; ++s) tma_load_2d(sBt + s * L::BT_SUB, &tmBt, &full[stage], k0 + s * BK, n0);
#pragma unroll
      for (int s = 0; s < KSUB; ++s) tma_load_2d(sA + s * L::A_SUB, &tmA, &full[stage], k0 + s * BK, m0);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
  } else if (warp == 1 && lane == 0) {
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0; i < nkb; ++i) {
      if (!mbar_wait(&full[stage], phase, ctx, SITE_FULL)) break;
      if (i == 0) SKY_TRACE(2);
      tc_fence_after();
      const uint32_t bt = smem_u32(smem + stage * L::STAGE);
      const uint32_t a = bt + KSUB * L::BT_SUB;
#pragma unroll
      for (int s = 0; s < KSUB; ++s)
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          umma_f16_cg1(tmem, umma_desc_sw128(bt + s * L::BT_SUB + k * 32), umma_desc_sw128(a + s * L::A_SUB + k * 32),
                       IDESC, (i | s | k) != 0 ? 1u : 0u);
      umma_commit_cg1(&empty[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    SKY_TRACE(3);
    if (nkb > 0) umma_commit_cg1(acc_full);  // also drains a partial loop after an abort
  } else if (warp >= 2) {
    if (threadIdx.x == 64) {
      // The receive barrier completes once every peer's slice has landed.
      mbar_arrive_expect_tx(recv_full, (uint32_t)((SPLITS - 1) * BMM * CS * 4));
    }
    // Second half of the setup barrier (every peer's barriers are
    // initialised), taken while the main loop runs.
    __syncwarp();
    cluster_wait_acquire();
    if (nkb > 0) {
      if (mbar_wait(acc_full, 0, ctx, SITE_TMEM_FULL)) {
        if (threadIdx.x == 64) SKY_TRACE(4);
      } else {
        ok = false;
      }
    }
  }
  if constexpr (!L::SEPARATE) {
    if (warp >= 2) {
      // The receive area overlaps the ring: wait until every CTA of the
      // cluster has drained its ring (its MMAs, covered by acc_full, consumed
      // all of its TMA loads).
      __syncwarp();
      cluster_sync();
    }
  }
  if (threadIdx.x == 64) SKY_TRACE(5);

  if (warp >= 2) {
    // Push: column slice o of this CTA's accumulator (lane = n, column = m)
    // goes to rank o's recv[ks][row]; the local slice with plain stores.
    tc_fence_after();
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool have = nkb > 0 && ok;
    const uint32_t bar_local = smem_u32(recv_full);
#pragma unroll
    for (int c = 0; c < BNM / 32; ++c) {
      uint32_t v[32];
      if (have) {
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), v);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0u;
      }
      if (threadIdx.x == 64 && c < 2) SKY_TRACE(8 + 2 * c);
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const int col = c * 32 + j;
        const int o = col / CS;  // compile-time
        const uint32_t dst = smem_u32(recv + (ks * BMM + row) * RSTRIDE + (col - o * CS));
        if (o == ks) {
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(v[j]), "r"(v[j + 1]), "r"(v[j + 2]),
                       "r"(v[j + 3])
                       : "memory");
        } else {
          st_async_v4(mapa_shared(dst, (uint32_t)o), mapa_shared(bar_local, (uint32_t)o), &v[j]);
        }
      }
      if (threadIdx.x == 64 && c < 2) SKY_TRACE(9 + 2 * c);
    }
    if (threadIdx.x == 64) SKY_TRACE(6);
    // Reduce this rank's slice of this thread's row over the S partials, in
    // rank order (deterministic). The local block was written by this thread;
    // the peers' blocks are complete once recv_full flips.
    const bool got = SPLITS == 1 || mbar_wait(recv_full, 0, ctx, SITE_PARTIAL);
    if (threadIdx.x == 64) SKY_TRACE(12);
    const int c0 = m0 + ks * CS;
    const int n = n0 + row;
    T* out = C + (size_t)n * M;
    if (got && n < N && row < step) {
#pragma unroll
      for (int cc = 0; cc < CS; cc += 8) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
        for (int r = 0; r < SPLITS; ++r) {
          const float* src = recv + (r * BMM + row) * RSTRIDE + cc;
          const float4 x = *reinterpret_cast<const float4*>(src), y = *reinterpret_cast<const float4*>(src + 4);
          acc[0] += x.x; acc[1] += x.y; acc[2] += x.z; acc[3] += x.w;
          acc[4] += y.x; acc[5] += y.y; acc[6] += y.z; acc[7] += y.w;
        }
        const int m = c0 + cc;
        if (m < M) {
          if ((M & 7) == 0) {  // 16-byte aligned run of 8 outputs
            uint4 h;
            h.x = pack2(T(), acc[0], acc[1]);
            h.y = pack2(T(), acc[2], acc[3]);
            h.z = pack2(T(), acc[4], acc[5]);
            h.w = pack2(T(), acc[6], acc[7]);
            *reinterpret_cast<uint4*>(out + m) = h;
          } else {
            for (int j = 0; j < 8 && m + j < M; ++j) out[m + j] = ElemTraits<T>::cvt(acc[j]);
          }
        }
      }
    }
    if (threadIdx.x == 64) SKY_TRACE(7);
  }
  if (warp < 2) {
    __syncwarp();
    cluster_wait_acquire();
    if constexpr (!L::SEPARATE) cluster_sync();
  }
  // TMEM is read by the epilogue warps only; free it once they are done.
  // Peers finish writing into this CTA before its recv_full flips, which every
  // epilogue thread waited for, so the CTA may exit after this barrier.
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem, TMEM_COLS);
  }
}

template <typename T, int BNM, int KSUB, int STAGES, int SPLITS>
int launch_splits(const GemmProblem& p, const CUtensorMap& tBt, const CUtensorMap& tA, int64_t tiles_n,
                  int64_t tiles_m, int step, const WaitCtx& ctx) {
  using L = SkinnySmem<BNM, KSUB, STAGES>;
  auto kern = gemm_skinny_kernel<T, BNM, KSUB, STAGES, SPLITS>;
  // Shared-memory opt-in once per device (host cost, not per launch).
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  (void)cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC);
  });
  cudaError_t e = attr_err[dev & 63];
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles_n * SPLITS), (unsigned)tiles_m, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = L::ALLOC;
  cfg.stream = p.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = SPLITS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  e = cudaLaunchKernelEx(&cfg, kern, tBt, tA, static_cast<T*>(p.C), (int)p.M, (int)p.N, (int)p.K, step,
                         cfg.numAttrs == 2 ? 1 : 0, ctx);
  if (e != cudaSuccess) return cuda_fail(e, "gemm_v106 launch");
  return KEBAB_OK;
}

template <typename T, int BNM, int KSUB, int STAGES>
int launch(const GemmProblem& p, int splits_override) {
  using L = SkinnySmem<BNM, KSUB, STAGES>;
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
  int64_t tiles_n = (p.N + BMM - 1) / BMM;
  const int64_t tiles_m = (p.M + BNM - 1) / BNM;
  const int64_t tiles = tiles_n * tiles_m;
  const int kb_total = (int)((p.K + BK * KSUB - 1) / (BK * KSUB));
  const long long slots = (long long)L::PER_SM * dev->sm_count;
  int splits = splits_override;
  if (splits <= 0) {
    // As many CTAs as fit in one wave (L::PER_SM per SM), in powers of two up
    // to the portable cluster size.
    splits = 1;
    while (splits < 8 && tiles * splits * 2 <= slots && splits * 2 <= kb_total) splits *= 2;
  }
  // Fit the wave (KEBAB_V106_FIT=1, off by default): when tiles x splits
  // leaves SMs idle (64 x 8192 x 8192: 64 tiles x 2 = 128 CTAs on 148 SMs),
  // start tiles every `step` < 128 columns (a multiple of 8) so that more of
  // them fill the wave; neighbouring tiles then read a few B^T rows twice,
  // from L2. Measured at 64 x 8192 x 8192: 4813 GB/s against 4924 without
  // (148 vs 128 CTAs), so the idle SMs are not what bounds this shape.
  int step = BMM;
  const char* fit_s = std::getenv("KEBAB_V106_FIT");
  const bool fit_env = fit_s && fit_s[0] == '1';
  if (fit_env && tiles * splits < slots) {
    const long long want = slots / ((long long)splits * tiles_m);
    if (want > tiles_n) {
      const int64_t st = (((p.N + want - 1) / want) + 7) / 8 * 8;
      if (st < BMM) {
        step = (int)st;
        tiles_n = (p.N + st - 1) / st;
      }
    }
  }
  if (tiles_n * splits > INT32_MAX || tiles_m > 65535) return fail(KEBAB_EINVAL, "grid too large for v106");
  switch (splits) {
    case 1: return launch_splits<T, BNM, KSUB, STAGES, 1>(p, tBt, tA, tiles_n, tiles_m, step, ctx);
    case 2: return launch_splits<T, BNM, KSUB, STAGES, 2>(p, tBt, tA, tiles_n, tiles_m, step, ctx);
    case 4: return launch_splits<T, BNM, KSUB, STAGES, 4>(p, tBt, tA, tiles_n, tiles_m, step, ctx);
    case 8: return launch_splits<T, BNM, KSUB, STAGES, 8>(p, tBt, tA, tiles_n, tiles_m, step, ctx);
    default: return fail(KEBAB_EINVAL, "splits must be 1, 2, 4 or 8");
  }
}

// Stage shapes (KSUB x 64-wide K sub-tiles, STAGES deep): the receive area
// stays beside the ring for M <= 128 (192 KB and 208 KB of shared memory);
// for M <= 256 it reuses the ring.
template <typename T, int BNM>
int launch_cfg(const GemmProblem& p, int splits) {
  if constexpr (BNM <= 64) return launch<T, BNM, 2, 3>(p, splits);
  else return launch<T, BNM, 1, 4>(p, splits);
}

template <typename T>
int launch_m(const GemmProblem& p, int splits) {
  if (p.M <= 64) return launch_cfg<T, 64>(p, splits);
  if (p.M <= 128) return launch_cfg<T, 128>(p, splits);
  return launch_cfg<T, 256>(p, splits);  // M-tiles of 256
}
}  // namespace

int launch_v106_skinny_splits(const GemmProblem& p, int splits) {
  return p.dtype == KEBAB_F16 ? launch_m<__half>(p, splits) : launch_m<__nv_bfloat16>(p, splits);
}
#ifdef KEBAB_SK_TRACE
extern "C" int kebab_debug_skinny_trace(void* host, size_t bytes) {
  return (int)cudaMemcpyFromSymbol(host, g_skinny_trace, bytes);
}
#endif

// KEBAB_V106_SPLITS (1, 2, 4, 8) overrides the split-K cluster size.
int launch_v106_skinny(const GemmProblem& p) {
  const char* e = std::getenv("KEBAB_V106_SPLITS");
  return launch_v106_skinny_splits(p, (e && *e) ? std::atoi(e) : 0);
}

}  // namespace kb
