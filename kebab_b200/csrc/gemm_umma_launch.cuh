// Host launch template of the warp-specialised tcgen05 rungs (v103, v104,
// v105) for every operand layout; each rung instantiates it in its own
// translation unit (gemm_v103_ws.cu, gemm_v104_persistent.cu, gemm_v105_pair.cu).
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "gemm_umma.cuh"
#include "internal.h"

namespace kb {
namespace umma_launch {

template <typename T, int BN, int STAGES, int CG, bool PERSISTENT, int LAYOUT, bool SK = false, int KPS = 1>
int launch_umma(const GemmProblem& p) {
  using L = UmmaSmem<BN, STAGES, CG, KPS>;
  int rc = check_tma_shapes(p);
  if (rc) return rc;
  DeviceInfo* dev = nullptr;
  if ((rc = device_info(&dev))) return rc;
  UmmaArgs args;
  if ((rc = wait_ctx(&args.ctx))) return rc;

  constexpr int BM_T = 128 * CG;
  CUtensorMap tA, tB, tC;
  if (!(LAYOUT & LAYOUT_A_MN)) {
    // A row-major M x K: box = 128 rows x 64 K (one CTA's rows of a tile).
    if ((rc = make_tmap_2d(&tA, p.A, p.dtype, p.M, p.K, p.K, 128, 64, true))) return rc;
  } else {
    // A column-major M x K = row-major K x M: boxes of 64 K rows x 64 M.
    if ((rc = make_tmap_2d(&tA, p.A, p.dtype, p.K, p.M, p.M, 64, 64, true))) return rc;
  }
  if (!(LAYOUT & LAYOUT_B_MN)) {
    // B column-major K x N = row-major N x K: box = BN/CG columns x 64 K.
    if ((rc = make_tmap_2d(&tB, p.B, p.dtype, p.N, p.K, p.K, BN / CG, 64, true))) return rc;
  } else {
    // B row-major K x N: boxes of 64 K rows x 64 N.
    if ((rc = make_tmap_2d(&tB, p.B, p.dtype, p.K, p.N, p.N, 64, 64, true))) return rc;
  }
  if (!(LAYOUT & LAYOUT_C_ROW)) {
    // C column-major M x N = row-major N x M: box = 32 columns x 32 rows.
    if ((rc = make_tmap_2d(&tC, p.C, p.dtype, p.N, p.M, p.M, 32, 32, false))) return rc;
  } else {
    // C row-major M x N: box = 32 rows x 32 columns (64-byte rows, 64-byte swizzle).
    if ((rc = make_tmap_2d_sw(&tC, p.C, p.dtype, p.M, p.N, p.N, 32, 32, 64))) return rc;
  }

  args.M = (int)p.M;
  args.N = (int)p.N;
  args.K = (int)p.K;
  args.tiles_m = (int)((p.M + BM_T - 1) / BM_T);
  args.tiles_n = (int)((p.N + BN - 1) / BN);
  // M-blocks per raster group (KEBAB_GROUP_M overrides). A wave of C tiles
  // running at once streams (group) A panels and (wave / group) B panels; a B
  // panel is BN / BM_T times an A panel, so the bytes per wave are smallest
  // near group = sqrt(wave * BN / BM_T): ~8.6 for 256 x 256 pair tiles, ~12
  // for 256 x 512 (measured on B200: v105 8192^3 DRAM reads 1.17 GB at 8 vs
  // 1.31 at 16; v107 16384 x 28672 x 8192: 1239 TFLOP/s at 16, 1186 at 12,
  // 1152 at 8).
  static const int group_env = [] {
    const char* e = std::getenv("KEBAB_GROUP_M");
    return (e && *e) ? std::atoi(e) : 0;
  }();
  args.group_m = group_env;  // resolved below, once the wave size is known
  // Epilogue poll backoff in ns (KEBAB_EPI_BACKOFF_NS; default 0 = spin).
  static const uint32_t backoff_env = [] {
    const char* e = std::getenv("KEBAB_EPI_BACKOFF_NS");
    return (e && *e) ? (uint32_t)std::atoi(e) : 0u;
  }();
  args.epi_backoff_ns = backoff_env;
  // L2 eviction hints of the A / B loads (KEBAB_L2_HINT, see UmmaArgs; default none).
  static const int hint_env = [] {
    const char* e = std::getenv("KEBAB_L2_HINT");
    return (e && *e) ? std::atoi(e) : 0;
  }();
  args.l2_hint = hint_env;
  const long long tiles = (long long)args.tiles_m * args.tiles_n;
  if (tiles > INT32_MAX / 2) return fail(KEBAB_EINVAL, "too many tiles");

  auto kern = gemm_umma_ws_kernel<T, BN, STAGES, CG, PERSISTENT, LAYOUT, SK, KPS>;
  // Once per device and instantiation: the shared-memory opt-in and, for
  // pairs (which must be co-resident on a GPC), how many clusters fit.
  static std::once_flag attr_once[64];
  static cudaError_t attr_err[64];
  static int max_active[64];
  const int di = dev->device & 63;
  std::call_once(attr_once[di], [&] {
    attr_err[di] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC);
    max_active[di] = dev->sm_count / CG;
    if (attr_err[di] != cudaSuccess || CG == 1) return;
    cudaLaunchConfig_t qc = {};
    qc.gridDim = dim3(CG * (dev->sm_count / CG), 1, 1);
    qc.blockDim = dim3(UmmaEpi<BN>::THREADS, 1, 1);
    qc.dynamicSmemBytes = L::ALLOC;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = CG;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    qc.attrs = qa;
    qc.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &qc) == cudaSuccess && n > 0) max_active[di] = n;
    (void)cudaGetLastError();
  });
  if (attr_err[di] != cudaSuccess) return cuda_fail(attr_err[di], "cudaFuncSetAttribute(max dynamic smem)");

  int clusters;
  if (PERSISTENT) {
    int max_clusters = std::min(dev->sm_count / CG, max_active[di]);
    // Stream-K spreads K-iterations over every SM, even with fewer tiles.
    clusters = SK ? max_clusters : (int)std::min<long long>(tiles, max_clusters);
  } else {
    clusters = (int)tiles;
  }

  if (args.group_m <= 0) {
    // Target group size, snapped to a divisor of tiles_m (no ragged last
    // group, whose waves would straddle two groups); ties go to the larger.
    const double wave = PERSISTENT ? (double)clusters : (double)dev->sm_count / CG;
    const double target = std::sqrt(wave * BN / BM_T);
    int best = 1;
    double best_err = 1e30;
    for (int d = 1; d <= args.tiles_m; ++d) {
      if (args.tiles_m % d) continue;
      const double err = std::fabs(std::log((double)d / target));
      if (err <= best_err + 1e-9) {
        best = d;
        best_err = err;
      }
    }
    args.group_m = best;
  }
  // Work split: whole tiles round robin; with stream-K the last partial wave
  // plus one full wave (or all tiles when there is less than one wave) are
  // split by K-iterations evenly over the clusters.
  args.dp_tiles = (int)tiles;
  args.sk_tiles = 0;
  args.ws = nullptr;
  args.flags = nullptr;
  args.epoch = 0;
  if (SK) {
    const long long waves = tiles / clusters, rem = tiles % clusters;
    // KEBAB_SK_MODE: 0 = remainder + one full wave (default), 1 = remainder
    // only, 2 = every tile.
    static const int sk_mode = [] {
      const char* e = std::getenv("KEBAB_SK_MODE");
      return (e && *e) ? std::atoi(e) : 0;
    }();
    if (rem != 0 || sk_mode == 2) {
      args.sk_tiles = (int)(sk_mode == 2 ? tiles : (waves >= 1 && sk_mode == 0) ? rem + clusters : rem);
      args.dp_tiles = (int)(tiles - args.sk_tiles);
      const size_t ctas = (size_t)CG * clusters;
      if ((rc = sk_workspace(p.stream, ctas * 128 * BN * sizeof(float), ctas * 4, &args.ws, &args.flags,
                             &args.epoch)))
        return rc;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CG * clusters, 1, 1);
  cfg.blockDim = dim3(UmmaEpi<BN>::THREADS, 1, 1);
  cfg.dynamicSmemBytes = L::ALLOC;
  cfg.stream = p.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  args.pdl = pdl_enabled() ? 1 : 0;
  cfg.numAttrs = args.pdl ? 2 : 1;
  // Serpentine K order (see UmmaArgs::serp): on unless KEBAB_SERPENTINE=0.
  // It cuts DRAM reads (8192^3 on rung 107: 859 -> 725 MB per launch) at the
  // price of M-sharded results matching a single GPU within tolerance rather
  // than bit for bit.
  static const int serp_env = [] {
    const char* e = std::getenv("KEBAB_SERPENTINE");
    return (e && *e) ? std::atoi(e) : 1;
  }();
  args.serp = serp_env;
  if (p.b_ready != nullptr) {
    if (!PERSISTENT || SK || (LAYOUT & LAYOUT_B_MN))
      return fail(KEBAB_ENOTSUP, "gated B needs a persistent, non-stream-K rung with column-major B");
    if (p.b_chunk_cols <= 0 || p.b_chunk_cols % BN != 0)
      return fail(KEBAB_EINVAL, "gated B: chunk width " + std::to_string(p.b_chunk_cols) +
                                    " must be a positive multiple of the rung's tile width " + std::to_string(BN));
    args.b_ready = p.b_ready;
    args.b_chunk_cols = (int)p.b_chunk_cols;
    args.b_epoch = p.b_epoch;
  }
  args.clk = take_clock_probe((int)cfg.gridDim.x);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tA, tB, tC, args);
  if (e != cudaSuccess) return cuda_fail(e, "gemm_umma_ws launch");
  return KEBAB_OK;
}



template <int CG, bool PERSISTENT, int STAGES, int LAYOUT, int BN, bool SK, int KPS = 1>
int dispatch_dtype(const GemmProblem& p) {
  if (p.dtype == KEBAB_F16) return launch_umma<__half, BN, STAGES, CG, PERSISTENT, LAYOUT, SK, KPS>(p);
  return launch_umma<__nv_bfloat16, BN, STAGES, CG, PERSISTENT, LAYOUT, SK, KPS>(p);
}

// Layout from the problem: A column-major, B row-major, C row-major bits.
template <int CG, bool PERSISTENT, int STAGES, int BN = 256, bool SK = false, int KPS = 1>
int dispatch(const GemmProblem& p) {
  const int layout = (p.lhs == 'C' ? LAYOUT_A_MN : 0) | (p.rhs == 'R' ? LAYOUT_B_MN : 0) |
                     (p.c_row ? LAYOUT_C_ROW : 0);
  switch (layout) {
    case 0: return dispatch_dtype<CG, PERSISTENT, STAGES, 0, BN, SK, KPS>(p);
    case 1: return dispatch_dtype<CG, PERSISTENT, STAGES, 1, BN, SK, KPS>(p);
    case 2: return dispatch_dtype<CG, PERSISTENT, STAGES, 2, BN, SK, KPS>(p);
    case 3: return dispatch_dtype<CG, PERSISTENT, STAGES, 3, BN, SK, KPS>(p);
    case 4: return dispatch_dtype<CG, PERSISTENT, STAGES, 4, BN, SK, KPS>(p);
    case 5: return dispatch_dtype<CG, PERSISTENT, STAGES, 5, BN, SK, KPS>(p);
    case 6: return dispatch_dtype<CG, PERSISTENT, STAGES, 6, BN, SK, KPS>(p);
    default: return dispatch_dtype<CG, PERSISTENT, STAGES, 7, BN, SK, KPS>(p);
  }
}

}  // namespace umma_launch
}  // namespace kb
