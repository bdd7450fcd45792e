// 2:4 structured-sparse GEMM on tcgen05.mma.sp (kind::f16), FP32 accumulate.
//
// C (M x N, column-major) = A (M x K, 2:4 sparse, given compressed as
// A_packed M x K/2 + metadata E) * B (K x N, column-major). Same warp roles,
// ring and epilogue as the dense persistent kernel (gemm_umma.cuh); per
// 128-wide logical K block a stage holds
//   A_packed 128 x 64 (16 KB, 128-byte swizzle),
//   B        128 x 128 as two 64-wide swizzled sub-tiles (32 KB),
//   E        128 rows x 16 bytes (2 KB): the metadata of the 128 x 128 block,
//            already in the order tcgen05.cp.128x128b expects (see
//            sparse24.cu:compress_kernel);
// the MMA lane copies E to 4 TMEM columns (tcgen05.cp) and issues four
// 128 x BN x 32 sparse MMAs, MMA j reading metadata column j (addressed as
// the even column 2*(j/2) plus selector j%2 in the instruction descriptor).
// Tile shapes: see SparseCfg below.
// The reference has no sparse GEMM (its 2:4 path is one mma.sp tile,
// kebab/lib/microbench/sparse_mma.cu:347-428).
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "gemm_umma.cuh"
#include "internal.h"
#include "kebab/sparse24.h"

namespace kb {

namespace {

// Per stage (128 logical K): MT A_packed tiles of 128 x 64, B as two 64-wide
// sub-tiles of BNC rows (this CTA's share of the tile's N), MT metadata
// blocks; then the epilogue's C staging (two buffers of 32 x CW per warp).
template <int STAGES, int MT, int BNC, int EPI_WARPS, int CW>
struct SparseSmem {
  static constexpr int A_TILE = 128 * 64 * 2;
  static constexpr int A_STAGE = MT * A_TILE;
  static constexpr int B_SUB = BNC * 64 * 2;
  static constexpr int B_STAGE = 2 * B_SUB;
  static constexpr int E_TILE = 2048;
  static constexpr int E_STAGE = MT * E_TILE;
  static constexpr int C_SUB = 32 * CW * 2;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_STAGE;
  static constexpr int OFF_E = OFF_B + STAGES * B_STAGE;
  static constexpr int OFF_C = OFF_E + STAGES * E_STAGE;
  static constexpr int OFF_BAR = OFF_C + EPI_WARPS * 2 * C_SUB;
  static constexpr int NUM_BARS = 2 * STAGES + 4 + 1;
  static constexpr int BYTES = OFF_BAR + NUM_BARS * 8 + 16;
  static constexpr int ALLOC = BYTES + 1024;
  static_assert(B_SUB % 1024 == 0, "128-byte-swizzled sub-tiles stay 1024-byte aligned");
  static_assert(ALLOC <= 232448, "shared memory budget exceeded");
};

// Tile shapes:
//   CG=1, MT=1, BN=128: 128 x 128 tiles, two accumulators (the epilogue of a
//       tile overlaps the next tile's MMAs).
//   CG=2, MT=1, BN=256: CTA pairs, 256 x 256 tiles, one accumulator.
//   CG=2, MT=2, BN=240: CTA pairs, 512 x 240 tiles: two 256-row M-tiles share
//       every staged B tile. The sparse MMA runs at twice the dense rate, so
//       operand delivery from L2 bounds it: per CTA and cycle a 256 x 256 pair
//       tile needs ~96 bytes (A 32 + B 64), two M-tiles ~66 (B's share
//       halves), against the ~55 bytes per SM and cycle L2 delivers under a
//       dense GEMM. The two 240-column accumulators sit at TMEM columns 0 and
//       256; metadata uses a 2-slot ring in columns 496..511.
template <typename T, int CG, int STAGES, int MT, int BN>
struct SparseCfg {
  static constexpr int BNC = BN / CG;                      // B rows per CTA
  static constexpr int EPI_WARPS = 4 * MT;                 // one warp per TMEM lane quarter and M-tile
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int CW = (BN % 32 == 0) ? 32 : 16;     // epilogue chunk (columns)
  static constexpr int ACC_COLS = (MT == 1) ? BN : 256;    // TMEM columns per accumulator slot
  static constexpr int ACCS = (MT == 1 && 2 * BN + 4 * STAGES <= 512) ? 2 : 1;
  static constexpr int E_SLOTS = (MT == 1) ? STAGES : 2;  // TMEM metadata slots (MT x 4 columns each)
  static constexpr int E_COL0 = (ACCS * MT - 1) * ACC_COLS + BN;
  static_assert(E_COL0 + E_SLOTS * MT * 4 <= 512, "metadata columns must fit in TMEM");
  static_assert(BN % CW == 0 && BN % 16 == 0 && BN <= 256, "tile width");
  using L = SparseSmem<STAGES, MT, BNC, EPI_WARPS, CW>;
};

#ifdef KEBAB_SK_TRACE
// Debug builds only: per CTA, per tile slot (first 8 tiles), 8 timestamps.
__device__ unsigned long long g_sp_trace[296 * 8 * 8];
#define SP_TRACE(slot, ev) g_sp_trace[((size_t)blockIdx.x * 8 + (slot)) * 8 + (ev)] = globaltimer()
#else
#define SP_TRACE(slot, ev) ((void)0)
#endif

template <int CW>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, uint32_t (&r)[CW]) {
  if constexpr (CW == 32) tmem_ld_32x32b_x32(taddr, r);
  else tmem_ld_32x32b_x16(taddr, r);
}

template <typename T, int CG, int STAGES, int MT, int BN>
__global__ void __launch_bounds__(SparseCfg<T, CG, STAGES, MT, BN>::THREADS, 1)
    gemm_sparse_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmE, const __grid_constant__ CUtensorMap tmC,
                       const UmmaArgs args) {
  using Cfg = SparseCfg<T, CG, STAGES, MT, BN>;
  using L = typename Cfg::L;
  constexpr int BM_MMA = 128 * CG;        // rows of one MMA (one M-tile)
  constexpr int BM_T = BM_MMA * MT;       // rows of a tile
  constexpr int ACCS = Cfg::ACCS;
  constexpr int TMEM_COLS = 512;
  constexpr uint32_t IDESC = umma_idesc_f16_sparse(BM_MMA, BN, ElemTraits<T>::kBf16);
  constexpr uint32_t TX_BYTES = (L::A_STAGE + L::B_STAGE + L::E_STAGE) * CG;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tmem_full = bars + 2 * STAGES;
  uint64_t* tmem_empty = bars + 2 * STAGES + 2;
  uint64_t* drain = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::NUM_BARS);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = (CG == 2) ? cluster_ctarank() : 0u;
  const bool leader = (rank == 0);
  const WaitCtx& ctx = args.ctx;
  ClockProbe probe;
  probe.begin(args.clk);

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmE);
    tma_prefetch_desc(&tmC);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], Cfg::EPI_WARPS * CG);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc<CG>(tmem_slot, TMEM_COLS);
    tmem_relinquish<CG>();
  }
  tc_fence_before();
  if constexpr (CG == 2) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (args.pdl) {  // prologue overlapped the previous kernel; now it has completed
    pdl_wait();
    pdl_launch_dependents();
  }

  const int num_tiles = args.tiles_m * args.tiles_n;
  const int cluster_id = blockIdx.x / CG;
  const int num_clusters = gridDim.x / CG;
  const int num_kb = args.K / 128;  // K % 128 == 0 (checked on the host)

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint32_t full_leader0 = (CG == 2) ? mapa_shared(smem_u32(&full[0]), 0) : 0u;
      int pu = 0;
      for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
        int mb, nb;
        tile_coords(tile, args.tiles_m, args.tiles_n, args.group_m, mb, nb);
        const int n0 = nb * BN + (int)rank * Cfg::BNC;
        const bool rev = args.serp && (pu++ & 1);  // serpentine K order (see UmmaArgs::serp)
        for (int i = 0; i < num_kb; ++i) {
          const int kb = rev ? num_kb - 1 - i : i;
          if (!mbar_wait(&empty[stage], phase ^ 1u, ctx, SITE_EMPTY)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + L::OFF_A + stage * L::A_STAGE;
          uint8_t* sB = smem + L::OFF_B + stage * L::B_STAGE;
          uint8_t* sE = smem + L::OFF_E + stage * L::E_STAGE;
          if constexpr (CG == 1) {
            mbar_arrive_expect_tx(&full[stage], TX_BYTES);
          } else {
            if (leader) mbar_arrive_expect_tx(&full[stage], TX_BYTES);
          }
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const int m0 = mb * BM_T + t * BM_MMA + (int)rank * 128;
            // E block (m-block, k-block) is 2 KB of contiguous bytes: rows of
            // 128 bytes in the tensor map, 16 per block.
            const int e_row = ((m0 / 128) * num_kb + kb) * 16;
            if constexpr (CG == 1) {
              tma_load_2d(sA + t * L::A_TILE, &tmA, &full[stage], kb * 64, m0);
              tma_load_2d(sE + t * L::E_TILE, &tmE, &full[stage], 0, e_row);
            } else {
              const uint32_t fb = full_leader0 + stage * 8u;
              tma_load_2d_pair(sA + t * L::A_TILE, &tmA, fb, kb * 64, m0);
              tma_load_2d_pair(sE + t * L::E_TILE, &tmE, fb, 0, e_row);
            }
          }
          if constexpr (CG == 1) {
            tma_load_2d(sB, &tmB, &full[stage], kb * 128, n0);
            tma_load_2d(sB + L::B_SUB, &tmB, &full[stage], kb * 128 + 64, n0);
          } else {
            const uint32_t fb = full_leader0 + stage * 8u;
            tma_load_2d_pair(sB, &tmB, fb, kb * 128, n0);
            tma_load_2d_pair(sB + L::B_SUB, &tmB, fb, kb * 128 + 64, n0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      uint32_t e_slot = 0;
      bool ok = true, any = false;
      for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
        const int tslot = (tile - cluster_id) / num_clusters;
        if (tslot < 8) SP_TRACE(tslot, 0);
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, ctx, SITE_TMEM_EMPTY)) {
          ok = false;
          break;
        }
        if (tslot < 8) SP_TRACE(tslot, 1);
        tc_fence_after();
        for (int kb = 0; kb < num_kb; ++kb) {  // issue order; the K-block itself is the producer's choice
          if (!mbar_wait(&full[stage], phase, ctx, SITE_FULL)) {
            ok = false;
            break;
          }
          if (kb == 0 && tslot < 8) SP_TRACE(tslot, 2);
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + L::OFF_A + stage * L::A_STAGE);
          const uint32_t b_addr = smem_u32(smem + L::OFF_B + stage * L::B_STAGE);
          const uint32_t e_addr = smem_u32(smem + L::OFF_E + stage * L::E_STAGE);
          // Metadata slot: one per stage (MT = 1), or a 2-slot ring (MT = 2):
          // tcgen05.cp and tcgen05.mma issued by this thread execute in order,
          // so the copy into a slot follows the MMAs that read it before.
          const uint32_t slot = (MT == 1) ? (uint32_t)stage : e_slot;
          e_slot ^= 1u;
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const uint32_t d_tmem = tmem_base + (uint32_t)((acc * MT + t) * Cfg::ACC_COLS);
            const uint32_t e_tmem = tmem_base + (uint32_t)(Cfg::E_COL0 + (slot * MT + t) * 4);
            // 128 rows x 16 bytes, 8-row core matrices 128 bytes apart, no swizzle.
            tmem_cp_128x128b<CG>(e_tmem, umma_desc(e_addr + t * L::E_TILE, 16, 128, 0));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint64_t ad = umma_desc_sw128(a_addr + t * L::A_TILE + j * 32);
              const uint64_t bd = umma_desc_sw128(b_addr + (j >> 1) * L::B_SUB + (j & 1) * 64);
              // The metadata address must be 2-column aligned; the odd column
              // of a pair is chosen with the descriptor's selector (bits 0..1).
              umma_f16_sp<CG>(d_tmem, ad, bd, e_tmem + (uint32_t)(j & ~1), IDESC | (uint32_t)(j & 1),
                              (kb | j) != 0 ? 1u : 0u);
            }
          }
          any = true;
          if constexpr (CG == 1) umma_commit_cg1(&empty[stage]);
          else umma_commit_cg2_mc(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (tslot < 8) SP_TRACE(tslot, 3);
        if constexpr (CG == 1) umma_commit_cg1(&tmem_full[acc]);
        else umma_commit_cg2_mc(&tmem_full[acc], 0x3);
        if (++acc == ACCS) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && any) {
        if constexpr (CG == 1) umma_commit_cg1(drain);
        else umma_commit_cg2_mc(drain, 0x1);
        WaitCtx d{ctx.status, 50000000ull};
        mbar_wait(drain, 0, d, SITE_DRAIN);
      }
    }
  } else {
    // Epilogue. The whole accumulator slice of this warp (32 rows x BN
    // columns) is read from TMEM into registers, rounded to the output type
    // and packed two per register, and TMEM is released before any store:
    // every pair finishes a tile at about the same time, and the burst of C
    // stores that follows is paced by L2 / DRAM write bandwidth. Stores then
    // drain from registers while the next tile's MMAs run.
    constexpr int CW = Cfg::CW;
    constexpr int NC = BN / CW;
    const int q = warp & 3;              // TMEM lane quarter
    const int ew = warp - 2;             // epilogue warp index
    const int t = ew >> 2;               // M-tile drained by this warp
    T* stage_c = reinterpret_cast<T*>(smem + L::OFF_C + ew * 2 * L::C_SUB);
    const uint32_t tmem_empty_leader0 = (CG == 2) ? mapa_shared(smem_u32(&tmem_empty[0]), 0) : 0u;
    int acc = 0;
    uint32_t acc_phase = 0;
    int sub = 0;
    for (int tile = cluster_id; tile < num_tiles; tile += num_clusters) {
      int mb, nb;
      tile_coords(tile, args.tiles_m, args.tiles_n, args.group_m, mb, nb);
      const int m_rows = mb * BM_T + t * BM_MMA + (int)rank * 128 + q * 32;
      const int n0 = nb * BN;
      if (!mbar_wait(&tmem_full[acc], acc_phase, ctx, SITE_TMEM_FULL)) break;
      const int tslot = (tile - cluster_id) / num_clusters;
      if (ew == 0 && lane == 0 && tslot < 8) SP_TRACE(tslot, 4);
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)((acc * MT + t) * Cfg::ACC_COLS);
      // Loads in 16-column chunks, one chunk ahead of the packing.
      constexpr int NL = BN / 16;
      uint32_t packed[BN / 2];
      {
        uint32_t v[16], vn[16];
        tmem_ld_chunk<16>(t_row, v);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < NL; ++c) {
          if (c + 1 < NL) tmem_ld_chunk<16>(t_row + (uint32_t)((c + 1) * 16), vn);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            packed[c * 8 + j] = pack2(T(), __uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
          if (c + 1 < NL) {
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = vn[j];
          }
        }
      }
      // The accumulator is in registers: release it to the MMA warp.
      tc_fence_before();
      __syncwarp();
      if (ew == 0 && lane == 0 && tslot < 8) SP_TRACE(tslot, 5);
      if (lane == 0) {
        if constexpr (CG == 1) mbar_arrive(&tmem_empty[acc]);
        else mbar_arrive_cluster(tmem_empty_leader0 + (uint32_t)acc * 8u);
      }
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        T* buf = stage_c + (sub & 1) * (32 * CW);
        if (lane == 0) tma_store_wait_read<1>();
        __syncwarp();
        uint16_t* b16 = reinterpret_cast<uint16_t*>(buf);
#pragma unroll
        for (int j = 0; j < CW / 2; ++j) {
          b16[(2 * j) * 32 + lane] = (uint16_t)(packed[c * (CW / 2) + j] & 0xFFFFu);
          b16[(2 * j + 1) * 32 + lane] = (uint16_t)(packed[c * (CW / 2) + j] >> 16);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, buf, m_rows, n0 + c * CW);
          tma_store_commit();
        }
        ++sub;
      }
      if (ew == 0 && lane == 0 && tslot < 8) SP_TRACE(tslot, 6);
      if (++acc == ACCS) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // The CTA may exit once its last C stores have read their staging
    // buffers; the global writes complete with the grid.
    if (lane == 0) tma_store_wait_read<0>();
    __syncwarp();
  }

  __syncwarp();
  tc_fence_before();
  if constexpr (CG == 2) cluster_sync(); else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<CG>(tmem_base, TMEM_COLS);
  }
  probe.end(args.clk);
}

// E viewed as a 2-D array of uint16 with 128-byte rows (64 per row), 16 rows
// per 2 KB block: one block is 16 row copies for the TMA unit rather than 128
// copies of 16 bytes.
int make_tmap_e(CUtensorMap* out, const void* E, int64_t M, int64_t K) {
  const uint64_t rows = (uint64_t)(M / 128) * (uint64_t)(K / 128) * 16;
  return make_tmap_2d(out, E, KEBAB_F16, rows, 64, 64, 16, 64, false);
}

template <typename T, int CG, int STAGES, int MT, int BN>
int launch_sparse(int dtype, const void* Ap, const void* E, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                  cudaStream_t stream) {
  using Cfg = SparseCfg<T, CG, STAGES, MT, BN>;
  using L = typename Cfg::L;
  DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  UmmaArgs args;
  if ((rc = wait_ctx(&args.ctx))) return rc;
  CUtensorMap tA, tB, tE, tC;
  if ((rc = make_tmap_2d(&tA, Ap, dtype, M, K / 2, K / 2, 128, 64, true))) return rc;
  if ((rc = make_tmap_2d(&tB, B, dtype, N, K, K, Cfg::BNC, 64, true))) return rc;
  if ((rc = make_tmap_e(&tE, E, M, K))) return rc;
  if ((rc = make_tmap_2d(&tC, C, dtype, N, M, M, Cfg::CW, 32, false))) return rc;
  constexpr int BM_T = 128 * CG * MT;
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.tiles_m = (int)((M + BM_T - 1) / BM_T);
  args.tiles_n = (int)((N + BN - 1) / BN);
  // M-tiles per raster group (KEBAB_GROUP_M overrides) and the serpentine K
  // order (on unless KEBAB_SPARSE_SERPENTINE=0). Measured at 8192^3 (200
  // launches, clock-scaled): group 8 serpentine 0.772 of the 2:4 clock peak
  // and 467 MB of DRAM reads per launch, against 0.759 and 568 MB in order;
  // groups 2 / 4 / 16 with serpentine 0.725 / 0.757 / 0.770.
  static const int group_env = [] {
    const char* e = std::getenv("KEBAB_GROUP_M");
    return (e && *e) ? std::atoi(e) : 0;
  }();
  static const int serp_env = [] {
    const char* e = std::getenv("KEBAB_SPARSE_SERPENTINE");
    return (e && *e) ? std::atoi(e) : 1;
  }();
  args.group_m = group_env > 0 ? group_env : 8;
  args.serp = serp_env;
  args.epi_backoff_ns = 0;
  const long long tiles = (long long)args.tiles_m * args.tiles_n;
  auto kern = gemm_sparse_kernel<T, CG, STAGES, MT, BN>;
  // Once per device and instantiation: the shared-memory opt-in and, for
  // pairs, how many clusters fit.
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  static int max_active[64];
  const int di = dev->device & 63;
  std::call_once(once[di], [&] {
    attr_err[di] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC);
    max_active[di] = dev->sm_count / CG;
    if (attr_err[di] != cudaSuccess || CG == 1) return;
    cudaLaunchConfig_t qc = {};
    qc.gridDim = dim3(CG * (dev->sm_count / CG), 1, 1);
    qc.blockDim = dim3(Cfg::THREADS, 1, 1);
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
  if (attr_err[di] != cudaSuccess) return cuda_fail(attr_err[di], "cudaFuncSetAttribute");
  const int max_clusters = std::min(dev->sm_count / CG, max_active[di]);
  const int clusters = (int)std::min<long long>(tiles, max_clusters);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CG * clusters, 1, 1);
  cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
  cfg.dynamicSmemBytes = L::ALLOC;
  cfg.stream = stream;
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
  args.clk = take_clock_probe((int)cfg.gridDim.x);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tA, tB, tE, tC, args);
  if (e != cudaSuccess) return cuda_fail(e, "gemm_sparse launch");
  return KEBAB_OK;
}

// Width of the 512-row pair tiles: the candidate whose tiles fill the last
// wave of pairs best, N padding counted; ties go to the wider tile. For
// 8192^3, 224 gives 37 x 16 = 592 tiles = 8 full waves of 74 pairs, where 240
// gives 35 x 16 = 560 (7.6 waves) and pads N by 2.5 %.
int sparse_tile_n(int64_t M, int64_t N, int pairs) {
  static const int cand[] = {240, 224, 192, 160};
  int best = 240;
  double best_eff = -1.0;
  const int64_t tiles_m = (M + 511) / 512;
  for (int bn : cand) {
    const int64_t tiles = tiles_m * ((N + bn - 1) / bn);
    const int64_t slots = ((tiles + pairs - 1) / pairs) * pairs;
    const double eff = (double)(M * N) / ((double)slots * 512.0 * bn);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = bn;
    }
  }
  return best;
}

template <typename T>
int launch_wide(int bn, int dtype, const void* Ap, const void* E, const void* B, void* C, int64_t M, int64_t N,
                int64_t K, cudaStream_t s) {
  switch (bn) {
    case 240: return launch_sparse<T, 2, 3, 2, 240>(dtype, Ap, E, B, C, M, N, K, s);
    case 224: return launch_sparse<T, 2, 3, 2, 224>(dtype, Ap, E, B, C, M, N, K, s);
    case 192: return launch_sparse<T, 2, 3, 2, 192>(dtype, Ap, E, B, C, M, N, K, s);
    case 160: return launch_sparse<T, 2, 3, 2, 160>(dtype, Ap, E, B, C, M, N, K, s);
    default: return fail(KEBAB_EINVAL, "2:4 GEMM tile width must be 240, 224, 192 or 160");
  }
}

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" int kebab_gemm_sparse24(kebab_dtype dtype, const void* A_packed, const void* E, const void* B, void* C,
                                   int64_t M, int64_t N, int64_t K, kebab_stream_t stream) {
  if (!A_packed || !E || !B || !C) return fail(KEBAB_EINVAL, "null pointer passed to kebab_gemm_sparse24");
  if (dtype != KEBAB_F16 && dtype != KEBAB_BF16) return fail(KEBAB_EINVAL, "2:4 GEMM supports F16 and BF16");
  if (M <= 0 || N <= 0 || K <= 0 || M % 128 || K % 128)
    return fail(KEBAB_EINVAL, "2:4 GEMM needs M % 128 == 0 and K % 128 == 0 (N > 0)");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail(KEBAB_EINVAL, "sizes must fit in int32");
  if ((reinterpret_cast<uintptr_t>(A_packed) | reinterpret_cast<uintptr_t>(E) | reinterpret_cast<uintptr_t>(B) |
       reinterpret_cast<uintptr_t>(C)) & 15u)
    return fail(KEBAB_EINVAL, "2:4 GEMM buffers must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Tile shape: KEBAB_SPARSE_CG=1 forces 128 x 128 single-CTA tiles, =2 the
  // 256 x 256 CTA-pair tiles; the default is the pair with two M-tiles
  // (512 x BN), BN chosen by sparse_tile_n (KEBAB_SPARSE_BN overrides).
  const char* env = std::getenv("KEBAB_SPARSE_CG");
  const int mode = (env && *env) ? std::atoi(env) : 3;
  if (mode == 1 || mode == 2) {
    if (dtype == KEBAB_F16)
      return mode == 1 ? launch_sparse<__half, 1, 4, 1, 128>(dtype, A_packed, E, B, C, M, N, K, s)
                       : launch_sparse<__half, 2, 4, 1, 256>(dtype, A_packed, E, B, C, M, N, K, s);
    return mode == 1 ? launch_sparse<__nv_bfloat16, 1, 4, 1, 128>(dtype, A_packed, E, B, C, M, N, K, s)
                     : launch_sparse<__nv_bfloat16, 2, 4, 1, 256>(dtype, A_packed, E, B, C, M, N, K, s);
  }
  DeviceInfo* dev = nullptr;
  const int rc = device_info(&dev);
  if (rc) return rc;
  const char* be = std::getenv("KEBAB_SPARSE_BN");
  const int bn = (be && *be) ? std::atoi(be) : sparse_tile_n(M, N, dev->sm_count / 2);
  return dtype == KEBAB_F16 ? launch_wide<__half>(bn, dtype, A_packed, E, B, C, M, N, K, s)
                            : launch_wide<__nv_bfloat16>(bn, dtype, A_packed, E, B, C, M, N, K, s);
}

extern "C" int kebab_sparse24_tile(int64_t M, int64_t N, int* tile_m, int* tile_n) {
  if (!tile_m || !tile_n) return fail(KEBAB_EINVAL, "null pointer passed to kebab_sparse24_tile");
  if (M <= 0 || N <= 0) return fail(KEBAB_EINVAL, "invalid dimensions");
  const char* env = std::getenv("KEBAB_SPARSE_CG");
  const int mode = (env && *env) ? std::atoi(env) : 3;
  if (mode == 1 || mode == 2) {
    *tile_m = *tile_n = 128 * mode;
    return KEBAB_OK;
  }
  DeviceInfo* dev = nullptr;
  const int rc = device_info(&dev);
  const int pairs = rc == KEBAB_OK ? dev->sm_count / 2 : 74;
  const char* be = std::getenv("KEBAB_SPARSE_BN");
  *tile_m = 512;
  *tile_n = (be && *be) ? std::atoi(be) : sparse_tile_n(M, N, pairs);
  return KEBAB_OK;
}

#ifdef KEBAB_SK_TRACE
extern "C" int kebab_debug_sparse_trace(void* host, size_t bytes) {
  return (int)cudaMemcpyFromSymbol(host, kb::g_sp_trace, bytes);
}
#endif
