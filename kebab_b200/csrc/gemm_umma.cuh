// Warp-specialised tcgen05 GEMM (the v103 / v104 / v105 rungs of the ladder).
//
// C (M x N, column-major, ldC = M) = A (M x K, row-major) * B (K x N,
// column-major), FP16 or BF16 inputs, FP32 accumulation in TMEM, FP16/BF16
// output. This is the sm_100a replacement for the reference's warp-
// specialised WGMMA kernels (kebab/lib/cuda/cuda_gemm_v4_* ... v19_*, hot loop
// described at cuda_gemm_v10_*:313-473): same operator, different machine.
//
// Roles (192 threads = 6 warps; 320 = 10 warps for the 512-column tile):
//   warp 0        TMA producer: one elected lane streams K-blocks of A and B
//                 into a STAGES-deep shared-memory ring (128-byte swizzle).
//   warp 1        TMEM owner + MMA issuer: allocates 512 TMEM columns (two
//                 BN-column FP32 accumulators), one lane issues
//                 tcgen05.mma (kind::f16, 128 x BN x 16, or 256 x BN x 16 over
//                 a CTA pair) and tcgen05.commit to release ring slots.
//   warps 2..5    epilogue (warps 2..9 with two warps per TMEM lane quarter
//                 for BN = 512): tcgen05.ld 32 columns at a time, convert, stage
//                 32 x 32 column-major sub-tiles in shared memory and write
//                 them with TMA stores; the accumulator is released as soon
//                 as it has been read, so the next tile's MMAs overlap the
//                 stores.
// Template knobs, one per rung:
//   PERSISTENT=false  grid = #tiles, one tile per CTA                 (v103)
//   PERSISTENT=true   grid = #SMs, static grouped-raster schedule,
//                     double-buffered accumulators                     (v104)
//   CG=2              CTA pairs (cluster 2x1), tcgen05 cta_group::2,
//                     256 x BN tiles; each CTA TMA-loads its own half of
//                     A (rows) and of B (columns) — no multicast loads  (v105)
// Layouts (LAYOUT bits): A row-major (K-major) or column-major (MN-major,
// bit 1), B column-major (K-major) or row-major (MN-major, bit 2), C
// column-major or row-major (bit 4). MN-major operands are staged as
// 64-element x 64-K TMA boxes (128-byte swizzle) and described to the MMA
// with LBO = 8 KB (next 64 elements along M/N) and SBO = 1 KB (next 8 K rows).
// Every barrier wait is bounded (ptx.cuh); on expiry the kernel records an
// error code, drains what it has in flight and returns.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace kb {

template <typename T>
struct ElemTraits;
template <>
struct ElemTraits<__half> {
  static constexpr int kBf16 = 0;
  __device__ static __forceinline__ __half cvt(float v) { return __float2half_rn(v); }
};
template <>
struct ElemTraits<__nv_bfloat16> {
  static constexpr int kBf16 = 1;
  __device__ static __forceinline__ __nv_bfloat16 cvt(float v) { return __float2bfloat16_rn(v); }
};

// Two floats rounded to the output type, packed low column first.
__device__ __forceinline__ uint32_t pack2(__half, float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(__nv_bfloat16, float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Grouped rasterisation: consecutive tile ids walk down `group_m` M-blocks
// before moving to the next N-block, so concurrently running CTAs share A
// rows and B columns in L2.
__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int group_m, int& mb, int& nb) {
  const int group_size = group_m * tiles_n;
  const int g = tile / group_size;
  const int first_m = g * group_m;
  const int gm = min(group_m, tiles_m - first_m);
  const int r = tile - g * group_size;
  mb = first_m + r % gm;
  nb = r / gm;
}

// One unit of work of a CTA (pair): K-blocks [k0, k1) of a tile. role:
// 0 = the whole tile, 1 = the tile's last K-blocks (owner: adds the partials
// of the contributors, then stores C), 2 = earlier K-blocks (contributor:
// publishes an FP32 partial).
struct WorkUnit {
  int tile, k0, k1, role;
  int first_cluster;  // owner: first contributing cluster
};

// Enumerates a cluster's units in processing order: whole tiles first (round
// robin), then its stream-K range, contributor segment first so that owners,
// which are processed later by other clusters, rarely wait.
struct UnitIter {
  int cluster, clusters, num_kb;
  int dp_tiles, sk_tiles;
  bool sk, persistent;
  int num_tiles;
  // state
  int dp_next;
  long long s, e;           // stream-K iteration range [s, e)
  int seg, nseg, t_first, t_last;
  bool contrib_first;

  __device__ void init(int c, int nc, int kb, int dp, int skt, bool use_sk, bool pers, int tiles) {
    cluster = c;
    clusters = nc;
    num_kb = kb;
    dp_tiles = use_sk ? dp : tiles;
    sk_tiles = use_sk ? skt : 0;
    sk = use_sk;
    persistent = pers;
    num_tiles = tiles;
    dp_next = c;
    const long long S = (long long)sk_tiles * kb;
    s = S * c / nc;
    e = S * (c + 1) / nc;
    seg = 0;
    if (e > s) {
      t_first = (int)(s / kb);
      t_last = (int)((e - 1) / kb);
      nseg = t_last - t_first + 1;
      contrib_first = (e - (long long)t_last * kb) < kb;
    } else {
      nseg = 0;
    }
  }
  // does cluster `c` have a non-empty stream-K range (and so a partial)?
  __device__ bool has_range(int c) const {
    const long long S = (long long)sk_tiles * num_kb;
    return S * (c + 1) / clusters > S * c / clusters;
  }
  // first cluster whose range contains SK iteration `it`
  __device__ int cluster_of(long long it) const {
    const long long S = (long long)sk_tiles * num_kb;
    return (int)(((it + 1) * clusters + S - 1) / S) - 1;
  }
  __device__ bool next(WorkUnit& u) {
    if (dp_next < dp_tiles) {
      u.tile = dp_next;
      u.k0 = 0;
      u.k1 = num_kb;
      u.role = 0;
      u.first_cluster = cluster;
      dp_next = persistent ? dp_next + clusters : dp_tiles;
      return true;
    }
    if (seg >= nseg) return false;
    // segment order: contributor (the last tile) first when there is one
    int t;
    if (contrib_first) t = (seg == 0) ? t_last : t_first + seg - 1;
    else t = t_first + seg;
    ++seg;
    const long long base = (long long)t * num_kb;
    u.tile = dp_tiles + t;
    u.k0 = (int)((s > base) ? s - base : 0);
    u.k1 = (int)((e < base + num_kb) ? e - base : num_kb);
    if (u.k0 == 0 && u.k1 == num_kb) u.role = 0;
    else if (u.k1 == num_kb) u.role = 1;
    else u.role = 2;
    u.first_cluster = cluster_of(base);
    return true;
  }
};

// Bounded wait until a flag written by another CTA (or by a stream memory
// operation) equals `want`; `site` is recorded on expiry.
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t want, const WaitCtx& ctx,
                                          uint32_t site = SITE_PARTIAL) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
  if (v == want) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    __nanosleep(64);
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v == want) return true;
    if ((it & 63u) == 0u) {
      if (aborted(ctx.status)) return false;
      if (globaltimer() - t0 > ctx.timeout_ns) {
        record_error(ctx.status, DEV_TIMEOUT, site);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void set_flag(uint32_t* flag, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}

#ifdef KEBAB_SK_TRACE
// Debug builds only: per-CTA event timestamps, [cta][slot][8] u64.
__device__ unsigned long long g_sk_trace[296 * 8 * 8];
#define SK_TRACE(slot, ev) g_sk_trace[((size_t)blockIdx.x * 8 + (slot)) * 8 + (ev)] = globaltimer()
#else
#define SK_TRACE(slot, ev) ((void)0)
#endif

struct UmmaArgs {
  int M, N, K;
  int tiles_m, tiles_n, group_m;
  // Stream-K (SK kernels only): tiles [0, dp_tiles) are whole-tile work split
  // round-robin; the K-iterations of tiles [dp_tiles, dp_tiles + sk_tiles)
  // are split evenly over the clusters. Partials go to ws (one 128 x BN FP32
  // slot per CTA) and are announced in flags (one per CTA and epilogue warp)
  // with the value `epoch`.
  int dp_tiles, sk_tiles;
  uint32_t epoch;
  float* ws;
  uint32_t* flags;
  uint32_t epi_backoff_ns;  // sleep between polls of the epilogue's accumulator wait (0 = spin)
  int l2_hint;              // 0: no hint; bits 0..1 policy of A, bits 2..3 of B (1 last, 2 first, 3 normal)
  int pdl = 0;              // launched with programmatic stream serialisation
  // Whole tiles: odd units of a CTA walk K from the end, so each wave starts
  // on the K-blocks the previous wave read last (still in L2). It ties a
  // tile's summation order to its place in the schedule, so results match
  // between a single GPU and M-shards within tolerance, not bit for bit
  // (KEBAB_SERPENTINE=0 restores bit-identity).
  int serp = 0;
  unsigned long long* clk = nullptr;  // clock probe buffer (4 u64 per CTA) or null
  // Gated B (non-null b_ready): B arrives in chunks of b_chunk_cols columns
  // (a multiple of BN) while the kernel runs; chunk j may be read once
  // b_ready[j] == b_epoch. Flags are raised in chunk order, so seeing chunk j
  // ready implies every earlier chunk is.
  const uint32_t* b_ready = nullptr;
  int b_chunk_cols = 0;
  uint32_t b_epoch = 0;
  WaitCtx ctx;
};

// Epilogue warps: 4 (one per TMEM lane quarter), or 8 for the 512-column
// accumulator (two per quarter, each draining half of the columns).
template <int BN>
struct UmmaEpi {
  static constexpr int WARPS = BN > 256 ? 8 : 4;
  static constexpr int THREADS = 64 + 32 * WARPS;
};

// A stage holds KPS sub-tiles of 64 K (one 128-byte swizzle row each) of A
// and of B: a ring slot and its barrier per KPS K-blocks.
template <int BN, int STAGES, int CG, int KPS = 1>
struct UmmaSmem {
  static constexpr int BM = 128;  // rows of A per CTA
  static constexpr int BK = 64;   // 64 x 2 bytes = one 128-byte swizzle row
  static constexpr int A_SUB = BM * BK * 2;
  static constexpr int B_SUB = (BN / CG) * BK * 2;
  static constexpr int A_STAGE = KPS * A_SUB;
  static constexpr int B_STAGE = KPS * B_SUB;
  static constexpr int C_SUB = 32 * 32 * 2;  // one 32x32 staging sub-tile
  static constexpr int C_BYTES = UmmaEpi<BN>::WARPS * 2 * C_SUB;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_STAGE;
  static constexpr int OFF_C = OFF_B + STAGES * B_STAGE;
  static constexpr int OFF_BAR = OFF_C + C_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 4 + 1;
  static constexpr int BYTES = OFF_BAR + NUM_BARS * 8 + 16;
  static constexpr int ALLOC = BYTES + 1024;  // slack for 1024-byte alignment
  static_assert(BYTES + 1024 <= 232448, "shared memory budget exceeded");
};

enum : int { LAYOUT_A_MN = 1, LAYOUT_B_MN = 2, LAYOUT_C_ROW = 4 };
#define B_MN_OF(layout) (((layout) & LAYOUT_B_MN) != 0)

// Global column of accumulator column d of a tile starting at column n0.
// With two sub-MMAs (BN = 384 / 512, CTA pairs) each CTA of the pair holds
// BN/2 contiguous B rows and sub-MMA s takes H = BN/4 of them from each: its
// accumulator columns [2Hs, 2Hs + H) are the leader's rows n0 + Hs + [0, H)
// and [2Hs + H, 2H(s+1)) the peer's rows n0 + BN/2 + Hs + [0, H).
template <int BN, int NSUB>
__device__ __forceinline__ int pair_col(int n0, int d) {
  if constexpr (NSUB == 1) {
    return n0 + d;
  } else {
    constexpr int H = BN / 4;
    const int s = d / (2 * H), r = d % (2 * H);
    return n0 + (r >= H ? BN / 2 : 0) + H * s + (r % H);
  }
}

// Operand descriptor for k-step `k` (16 elements of K) of a staged tile.
template <bool MN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int k) {
  if constexpr (MN) return umma_desc(base + k * 2048, 8192, 1024, 2);  // 16 K rows = 2 x 1 KB groups
  else return umma_desc_sw128(base + k * 32);                          // 16 K elements = 32 bytes
}

// KPS: K-blocks of 64 per ring stage (2: half as many barrier round trips per
// byte; each stage then carries 2 A and 2 B boxes).
template <typename T, int BN, int STAGES, int CG, bool PERSISTENT, int LAYOUT = 0, bool SK = false, int KPS = 1>
__global__ void __launch_bounds__(UmmaEpi<BN>::THREADS, 1)
    gemm_umma_ws_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const UmmaArgs args) {
  using L = UmmaSmem<BN, STAGES, CG, KPS>;
  static_assert(KPS == 1 || !SK, "stream-K splits single K-blocks");
  constexpr int BM_T = 128 * CG;  // rows per (pair) tile
  constexpr int TMEM_COLS = 512;
  // BN = 384 or 512 (pairs only): two N = BN/2 MMAs per k-step share the A
  // tile; the accumulator takes more than half of TMEM, so it is
  // single-buffered. Sub-MMA s reads rows [s BN/4, (s+1) BN/4) of each CTA's
  // B tile (see pair_col for where its columns land in C).
  constexpr int NSUB = BN > 256 ? 2 : 1;
  constexpr int ACCS = (2 * BN <= TMEM_COLS) ? 2 : 1;
  static_assert(BN <= 256 || ((BN == 384 || BN == 512) && CG == 2), "BN = 384 / 512 needs CTA pairs");
  static_assert(BN != 384 || !B_MN_OF(LAYOUT), "BN = 384 needs column-major (K-major) B");
  static_assert(!SK || (PERSISTENT && BN <= 256), "stream-K needs the persistent 4-warp epilogue");
  constexpr bool A_MN = (LAYOUT & LAYOUT_A_MN) != 0;
  constexpr bool B_MN = (LAYOUT & LAYOUT_B_MN) != 0;
  constexpr bool C_ROW = (LAYOUT & LAYOUT_C_ROW) != 0;
  constexpr uint32_t IDESC = umma_idesc_f16(BM_T, BN / NSUB, ElemTraits<T>::kBf16) | (A_MN ? (1u << 15) : 0u) |
                             (B_MN ? (1u << 16) : 0u);
  constexpr uint32_t TX_BYTES = (L::A_STAGE + L::B_STAGE) * CG;  // bytes landing on the issuing CTA's barrier

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
#ifdef KEBAB_SK_TRACE
    g_sk_trace[((size_t)blockIdx.x * 8 + 7) * 8 + 5] = globaltimer();
#endif
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], UmmaEpi<BN>::WARPS * CG);
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
  // The prologue above overlaps the previous kernel on the stream when this
  // grid is PDL-launched; global memory is touched only after it completed.
  if (args.pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }
#ifdef KEBAB_SK_TRACE
  if (threadIdx.x == 0) g_sk_trace[((size_t)blockIdx.x * 8 + 7) * 8 + 6] = globaltimer();
#endif

  const int num_tiles = args.tiles_m * args.tiles_n;
  const int cluster_id = blockIdx.x / CG;
  const int num_clusters = gridDim.x / CG;
  const int num_kb = (args.K + L::BK * KPS - 1) / (L::BK * KPS);  // ring stages per tile

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued_parity[STAGES];
      bool issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false;
      const uint32_t full_leader0 = (CG == 2) ? mapa_shared(smem_u32(&full[0]), 0) : 0u;
      UnitIter it;
      it.init(cluster_id, num_clusters, num_kb, args.dp_tiles, args.sk_tiles, SK, PERSISTENT, num_tiles);
      WorkUnit u;
      int pu = 0;
      int chunk_seen = -1;  // gated B: highest chunk seen ready
      while (ok && it.next(u)) {
        int mb, nb;
        tile_coords(u.tile, args.tiles_m, args.tiles_n, args.group_m, mb, nb);
        const int m0 = mb * BM_T + (int)rank * 128;
        const int n0 = nb * BN + (int)rank * (BN / CG);
        if (args.b_ready != nullptr) {
          const int chunk = (nb * BN) / args.b_chunk_cols;
          if (chunk > chunk_seen) {
            if (!wait_flag(args.b_ready + chunk, args.b_epoch, ctx, SITE_BCHUNK)) {
              ok = false;
              break;
            }
            fence_proxy_async_global();
            chunk_seen = chunk;
          }
        }
        const bool rev = !SK && args.serp && (pu++ & 1);
        for (int i = 0; i < u.k1 - u.k0; ++i) {
          const int kb = rev ? u.k1 - 1 - i : u.k0 + i;
          if (!mbar_wait(&empty[stage], phase ^ 1u, ctx, SITE_EMPTY)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + L::OFF_A + stage * L::A_STAGE;
          uint8_t* sB = smem + L::OFF_B + stage * L::B_STAGE;
          // K-major tiles are one box (x = K, y = rows); MN-major tiles are
          // boxes of 64 rows-or-columns each (x = M or N, y = K).
          // kq: index of the 64-wide K-block within K.
          auto load = [&](uint8_t* dst, const CUtensorMap* tm, int rows0, int nrows, bool mn, int hint, int kq) {
            if (!mn && hint) {
              const uint64_t pol = hint == 1 ? l2_policy_evict_last()
                                   : hint == 2 ? l2_policy_evict_first() : l2_policy_evict_normal();
              if constexpr (CG == 1) tma_load_2d_hint(dst, tm, &full[stage], kq * L::BK, rows0, pol);
              else tma_load_2d_pair_hint(dst, tm, full_leader0 + stage * 8u, kq * L::BK, rows0, pol);
            } else if (!mn) {
              if constexpr (CG == 1) tma_load_2d(dst, tm, &full[stage], kq * L::BK, rows0);
              else tma_load_2d_pair(dst, tm, full_leader0 + stage * 8u, kq * L::BK, rows0);
            } else {
              for (int j = 0; j < nrows / 64; ++j) {
                if constexpr (CG == 1) tma_load_2d(dst + j * 8192, tm, &full[stage], rows0 + j * 64, kq * L::BK);
                else tma_load_2d_pair(dst + j * 8192, tm, full_leader0 + stage * 8u, rows0 + j * 64, kq * L::BK);
              }
            }
          };
          if (CG == 1 || leader) mbar_arrive_expect_tx(&full[stage], TX_BYTES);
#pragma unroll
          for (int q = 0; q < KPS; ++q) {
            load(sA + q * L::A_SUB, &tmA, m0, 128, A_MN, args.l2_hint & 3, kb * KPS + q);
            load(sB + q * L::B_SUB, &tmB, n0, BN / CG, B_MN, (args.l2_hint >> 2) & 3, kb * KPS + q);
          }
          issued[stage] = true;
          issued_parity[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && (CG == 1 || leader)) {
        // Abort: let our own copies still in flight land before the CTA exits.
        WaitCtx drain_ctx{ctx.status, 50000000ull};
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) mbar_wait(&full[s], issued_parity[s], drain_ctx, SITE_DRAIN);
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool any_issued = false;
      UnitIter it;
      it.init(cluster_id, num_clusters, num_kb, args.dp_tiles, args.sk_tiles, SK, PERSISTENT, num_tiles);
      WorkUnit u;
      int uidx = 0;
      while (ok && it.next(u)) {
        SK_TRACE(uidx & 7, 0);
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, ctx, SITE_TMEM_EMPTY)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int i = 0; i < u.k1 - u.k0; ++i) {
          if (!mbar_wait(&full[stage], phase, ctx, SITE_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + L::OFF_A + stage * L::A_STAGE);
          const uint32_t b_addr = smem_u32(smem + L::OFF_B + stage * L::B_STAGE);
#pragma unroll
          for (int q = 0; q < KPS; ++q) {
#pragma unroll
            for (int k = 0; k < L::BK / 16; ++k) {
              const uint64_t ad = operand_desc<A_MN>(a_addr + q * L::A_SUB, k);
              const uint32_t acc_flag = (i != 0 || q != 0 || k != 0) ? 1u : 0u;
#pragma unroll
              for (int sub = 0; sub < NSUB; ++sub) {
                // Sub-MMA `sub` reads rows [sub BN/4, (sub+1) BN/4) of each CTA's B tile.
                const uint64_t bd = operand_desc<B_MN>(b_addr + q * L::B_SUB + sub * ((BN / 4) * L::BK * 2), k);
                if constexpr (CG == 1)
                  umma_f16_cg1(d_tmem + sub * (BN / NSUB), ad, bd, IDESC, acc_flag);
                else
                  umma_f16_cg2(d_tmem + sub * (BN / NSUB), ad, bd, IDESC, acc_flag);
              }
            }
          }
          any_issued = true;
          if constexpr (CG == 1) umma_commit_cg1(&empty[stage]);
          else umma_commit_cg2_mc(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        SK_TRACE(uidx & 7, 1);
        ++uidx;
        if constexpr (CG == 1) umma_commit_cg1(&tmem_full[acc]);
        else umma_commit_cg2_mc(&tmem_full[acc], 0x3);
        if (++acc == ACCS) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && any_issued) {
        // Abort: wait for the MMAs already issued before TMEM is freed.
        if constexpr (CG == 1) umma_commit_cg1(drain);
        else umma_commit_cg2_mc(drain, 0x1);
        WaitCtx drain_ctx{ctx.status, 50000000ull};
        mbar_wait(drain, 0, drain_ctx, SITE_DRAIN);
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int q = warp & 3;       // TMEM lane quarter this warp may access
    const int ew = warp - 2;      // epilogue warp index (staging buffers)
    constexpr int CHUNKS = BN / 32 / (UmmaEpi<BN>::WARPS / 4);  // 32-column chunks per warp
    const int c0 = (ew / 4) * CHUNKS;                           // this warp's first chunk
    T* stage_c = reinterpret_cast<T*>(smem + L::OFF_C + ew * 2 * L::C_SUB);
    const uint32_t tmem_empty_leader0 = (CG == 2) ? mapa_shared(smem_u32(&tmem_empty[0]), 0) : 0u;
    int acc = 0;
    uint32_t acc_phase = 0;
    int sub = 0;
    UnitIter it;
    it.init(cluster_id, num_clusters, num_kb, args.dp_tiles, args.sk_tiles, SK, PERSISTENT, num_tiles);
    WorkUnit u;
    bool ok = true;
    int uidx = 0;
    while (ok && it.next(u)) {
      int mb, nb;
      tile_coords(u.tile, args.tiles_m, args.tiles_n, args.group_m, mb, nb);
      const int m_rows = mb * BM_T + (int)rank * 128 + q * 32;
      const int n0 = nb * BN;
      if (!mbar_wait_backoff(&tmem_full[acc], acc_phase, ctx, SITE_TMEM_FULL, args.epi_backoff_ns)) break;
      if (q == 0 && lane == 0) SK_TRACE(uidx & 7, 2);
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      // Stream-K: this thread's row of this CTA's partial slot, and (owner)
      // the contributors, whose flags must carry this launch's epoch.
      float* my_slot = nullptr;
      if constexpr (SK) {
        // Slot layout: [chunk][lane quarter][column][row]: for each column a
        // warp reads or writes 32 consecutive floats (one 128-byte line).
        my_slot = args.ws + (size_t)blockIdx.x * 128 * BN + q * 1024 + lane;
        if (u.role == 1) {
          for (int cc = u.first_cluster; cc < cluster_id && ok; ++cc)
            if (it.has_range(cc) && lane == 0 &&
                !wait_flag(args.flags + (size_t)(cc * CG + rank) * 4 + q, args.epoch, ctx))
              ok = false;
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
          __syncwarp();
        }
        if (q == 0 && lane == 0) {
          SK_TRACE(uidx & 7, 3);
#ifdef KEBAB_SK_TRACE
          g_sk_trace[((size_t)blockIdx.x * 8 + (uidx & 7)) * 8 + 5] = (unsigned long long)u.tile << 32 | (uint32_t)(u.k0 << 16 | u.k1);
          g_sk_trace[((size_t)blockIdx.x * 8 + (uidx & 7)) * 8 + 6] = (unsigned long long)u.role << 32 | (uint32_t)u.first_cluster;
#endif
        }
      }
      if constexpr (ACCS == 1 && !SK && !C_ROW) {
        // Single accumulator: every pair finishes its tile at about the same
        // time and the C stores that follow are paced by L2 / DRAM write
        // bandwidth, so read this warp's whole slice out of TMEM first (FP16 /
        // BF16 pairs, CHUNKS x 16 registers), hand TMEM back to the MMA
        // issuer, and store while the next tile's MMAs run.
        uint32_t packed[CHUNKS][16];
#pragma unroll
        for (int l = 0; l < 2 * CHUNKS; ++l) {
          // 16-column loads (registers stay below the spill line with the
          // whole slice held packed).
          uint32_t v[16];
          tmem_ld_32x32b_x16(t_row + (uint32_t)(c0 * 32 + l * 16), v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            packed[l >> 1][(l & 1) * 8 + j] = pack2(T(), __uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (CG == 1) mbar_arrive(&tmem_empty[acc]);
          else mbar_arrive_cluster(tmem_empty_leader0 + (uint32_t)acc * 8u);
        }
#pragma unroll
        for (int i = 0; i < CHUNKS; ++i) {
          const int c = c0 + i;
          T* buf = stage_c + (sub & 1) * (32 * 32);
          if (lane == 0) tma_store_wait_read<1>();
          __syncwarp();
          uint16_t* b16 = reinterpret_cast<uint16_t*>(buf);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            b16[(2 * j) * 32 + lane] = (uint16_t)(packed[i][j] & 0xFFFFu);
            b16[(2 * j + 1) * 32 + lane] = (uint16_t)(packed[i][j] >> 16);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int d = c * 32;
            tma_store_2d(&tmC, buf, m_rows, pair_col<BN, NSUB>(n0, d));
            tma_store_commit();
          }
          ++sub;
        }
      } else {
#pragma unroll 1
      for (int c = c0; c < c0 + CHUNKS; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_row + (uint32_t)(c * 32), v);
        tmem_ld_wait();
        if constexpr (SK) {
          if (u.role == 2) {
            // Contributor: publish the FP32 partial of columns [32c, 32c + 32).
            float* dst = my_slot + c * 4096;
#pragma unroll
            for (int j = 0; j < 32; ++j) __stcg(dst + j * 32, __uint_as_float(v[j]));
          } else if (u.role == 1 && ok) {
            // Owner: add the contributors' partials in cluster order.
            for (int cc = u.first_cluster; cc < cluster_id; ++cc) {
              if (!it.has_range(cc)) continue;  // clusters with no K-iterations publish nothing
              const float* src = args.ws + (size_t)(cc * CG + rank) * 128 * BN + c * 4096 + q * 1024 + lane;
              float p[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) p[j] = __ldcg(src + j * 32);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + p[j]);
            }
          }
        }
        if (c == c0 + CHUNKS - 1) {
          // Accumulator fully read: hand it back to the MMA issuer.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (CG == 1) mbar_arrive(&tmem_empty[acc]);
            else mbar_arrive_cluster(tmem_empty_leader0 + (uint32_t)acc * 8u);
          }
        }
        if (SK && u.role == 2) continue;  // a contributor stores no C
        T* buf = stage_c + (sub & 1) * (32 * 32);
        if (lane == 0) tma_store_wait_read<1>();  // the store that used `buf` has read it
        __syncwarp();
        if constexpr (!C_ROW) {
          // [column][row] sub-tile: for each column the warp writes 64 contiguous bytes.
#pragma unroll
          for (int j = 0; j < 32; ++j) buf[j * 32 + lane] = ElemTraits<T>::cvt(__uint_as_float(v[j]));
        } else {
          // [row][column] sub-tile, 64-byte rows in the TMA 64-byte swizzle:
          // 16-byte chunk c of row r sits at chunk c ^ ((r >> 1) & 3).
          uint4* row = reinterpret_cast<uint4*>(buf + lane * 32);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            alignas(16) T h[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) h[j] = ElemTraits<T>::cvt(__uint_as_float(v[q4 * 8 + j]));
            row[q4 ^ ((lane >> 1) & 3)] = *reinterpret_cast<const uint4*>(h);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // Global column of accumulator column d = 32 c. With BN = 512 each CTA of
          // the pair holds 256 contiguous B rows, so sub-MMA s covers columns
          // n0 + 128 s + [0, 128) (leader) and n0 + 256 + 128 s + [0, 128) (peer).
          const int d = c * 32;
          const int gcol = pair_col<BN, NSUB>(n0, d);
          if constexpr (!C_ROW) tma_store_2d(&tmC, buf, m_rows, gcol);
          else tma_store_2d(&tmC, buf, gcol, m_rows);
          tma_store_commit();
        }
        ++sub;
      }
      }  // single-accumulator path / chunked path
      if constexpr (SK) {
        if (u.role == 2) {
          // Partial written: make it visible GPU-wide, then raise this warp's flag.
          __syncwarp();
          __threadfence();
          if (lane == 0) set_flag(args.flags + (size_t)blockIdx.x * 4 + q, args.epoch);
        }
      }
      if (q == 0 && lane == 0) SK_TRACE(uidx & 7, 4);
      ++uidx;
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

  // ------------------------------------------------------------- teardown
  __syncwarp();
  tc_fence_before();
  if constexpr (CG == 2) cluster_sync(); else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<CG>(tmem_base, TMEM_COLS);
  }
  probe.end(args.clk);
}

}  // namespace kb
