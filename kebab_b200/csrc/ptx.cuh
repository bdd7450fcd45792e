// Thin inline-PTX wrappers for the Blackwell (sm_100a) primitives the GEMM
// ladder is built from: mbarriers with bounded waits, TMA (cp.async.bulk.tensor)
// loads and stores, and the tcgen05 family (TMEM alloc, UMMA issue, commit,
// TMEM loads). Every wait in this file is bounded; on expiry it records an
// error code in the module's device status word and returns false, so no
// kernel built on these helpers can spin forever on a shared GPU.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace kb {

// ---------------------------------------------------------------------------
// Device status word (one per loaded module). Kernels write a non-zero code
// here when a bounded wait expires; the host reads it back through
// kebab_device_status(). The word is passed to every kernel as a pointer. Layout: bits 0..7 error class, bits 8..15 the wait
// site, bits 16..31 the block index (truncated).
// ---------------------------------------------------------------------------
enum : uint32_t {
  DEV_OK = 0,
  DEV_TIMEOUT = 1,
};
enum WaitSite : uint32_t {
  SITE_FULL = 1,        // MMA issuer waiting for a filled smem stage
  SITE_EMPTY = 2,       // TMA producer waiting for a free smem stage
  SITE_TMEM_FULL = 3,   // epilogue waiting for an accumulator
  SITE_TMEM_EMPTY = 4,  // MMA issuer waiting for a drained accumulator
  SITE_MMA_DONE = 5,    // single-stage kernels waiting for their MMA
  SITE_TMA_DONE = 6,    // single-stage kernels waiting for their TMA
  SITE_PROBE = 7,       // the deliberate-timeout probe kernel
  SITE_DRAIN = 8,       // teardown drain after an abort
  SITE_PARTIAL = 9,     // stream-K owner waiting for a contributor's partial
  SITE_BCHUNK = 10,     // gated GEMM producer waiting for a chunk of B to arrive
};

// Where a kernel reports a failed wait, and how long a wait may take.
// Clock probe: with a buffer given, thread 0 of every CTA records (SM cycle
// counter, global ns timer) at entry and at exit, four u64 per CTA; the host
// divides cycles by nanoseconds to get the SM clock the launch really ran at.
struct ClockProbe {
  unsigned long long c0 = 0, t0 = 0;
  __device__ __forceinline__ void begin(unsigned long long* buf) {
    if (buf && threadIdx.x == 0) {
      asm volatile("mov.u64 %0, %%clock64;" : "=l"(c0));
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    }
  }
  __device__ __forceinline__ void end(unsigned long long* buf) const {
    if (buf && threadIdx.x == 0) {
      unsigned long long c1, t1;
      asm volatile("mov.u64 %0, %%clock64;" : "=l"(c1));
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
      unsigned long long* d = buf + (size_t)blockIdx.x * 4;
      d[0] = c0;
      d[1] = t0;
      d[2] = c1;
      d[3] = t1;
    }
  }
};

struct WaitCtx {
  uint32_t* status;     // device status word (see above)
  uint64_t timeout_ns;  // budget for any single barrier wait
};

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(uint32_t* status, uint32_t cls, uint32_t site) {
  uint32_t code = cls | (site << 8) | ((blockIdx.x & 0xFFFFu) << 16);
  atomicCAS(status, 0u, code);
}

__device__ __forceinline__ bool aborted(const uint32_t* status) {
  return *reinterpret_cast<const volatile uint32_t*>(status) != 0u;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Arrive on a barrier given by its shared::cluster address (own or peer CTA).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete. Returns false
// (and records DEV_TIMEOUT) when `timeout_ns` of wall time pass, or when
// another block has already recorded an error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const WaitCtx& ctx, uint32_t site) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((it & 63u) == 0u) {
      if (aborted(ctx.status)) return false;
      if (globaltimer() - t0 > ctx.timeout_ns) {
        record_error(ctx.status, DEV_TIMEOUT, site);
        return false;
      }
    }
  }
}

// As mbar_wait, but sleeps `backoff_ns` between polls once the first few have
// failed: for waits that are expected to be long (an epilogue waiting out a
// whole main loop), where tight polling only burns issue slots and power.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, const WaitCtx& ctx, uint32_t site,
                                                  uint32_t backoff_ns) {
  if (backoff_ns == 0) return mbar_wait(bar, parity, ctx, site);
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(addr, parity)) return true;
    if (it > 4) __nanosleep(backoff_ns);
    if ((it & 15u) == 0u) {
      if (aborted(ctx.status)) return false;
      if (globaltimer() - t0 > ctx.timeout_ns) {
        record_error(ctx.status, DEV_TIMEOUT, site);
        return false;
      }
    }
  }
}

// shared::cluster address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Programmatic dependent launch. wait: block until the grids this launch
// depends on have completed and their memory is visible (a no-op when the
// launch has no such dependency). launch_dependents: allow the next
// PDL-launched grid on the stream to start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// A cluster barrier split in two: arrive early (releasing this thread's prior
// writes, e.g. mbarrier initialisation), wait later (acquiring the peers').
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 2D tiled load global -> this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// L2 eviction-priority policies for the cache-hinted loads below.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const void* tmap, uint64_t* bar, int32_t x, int32_t y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair_hint(void* smem_dst, const void* tmap, uint32_t bar_cluster_addr,
                                                      int32_t x, int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar_cluster_addr), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// 2D tiled load into this CTA's shared memory whose completion is signalled on
// a barrier of the CTA pair (`bar_cluster_addr` may be the peer's barrier).
// Used by the cta_group::2 kernels: both CTAs of a pair load their own half
// of A and B, and the transaction bytes land on the leader CTA's barrier.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* tmap, uint32_t bar_cluster_addr, int32_t x,
                                                 int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Order this thread's earlier (acquire) observations of global memory before
// its later async-proxy (TMA) reads of global memory.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Make generic-proxy shared-memory writes visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM management
// ---------------------------------------------------------------------------
template <int CG>
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
  else
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
template <int CG>
__device__ __forceinline__ void tmem_relinquish() {
  if constexpr (CG == 1)
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  else
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
template <int CG>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
  else
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05: UMMA descriptors and issue
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor (sm100 format): start address, leading and
// stride byte offsets (all >> 4), version 1 at bits 46..47, swizzle mode at
// bits 61..63 (2 = 128-byte swizzle). For a K-major operand staged by TMA with
// 128-byte swizzle, rows are 128 bytes apart and groups of 8 rows 1024 bytes
// apart (the stride byte offset); the leading byte offset is unused.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;                    // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>((1024u >> 4) & 0x3FFFu) << 32;  // SBO = 1024 bytes
  d |= static_cast<uint64_t>(1u) << 46;                    // descriptor version for sm100
  d |= static_cast<uint64_t>(2u) << 61;                    // SWIZZLE_128B
  return d;
}

// General shared-memory matrix descriptor: `layout` 0 = no swizzle,
// 2 = 128-byte swizzle; byte offsets are multiples of 16.
__device__ __forceinline__ uint64_t umma_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) | static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16 |
         static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32 | static_cast<uint64_t>(1u) << 46 |
         static_cast<uint64_t>(layout & 7u) << 61;
}

// Instruction descriptor for kind::f16 with FP32 accumulation, both operands
// K-major. `ab_bf16` selects BF16 (1) or FP16 (0) for A and B.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N, int ab_bf16) {
  return (1u << 4)                                     // D format: F32
         | (static_cast<uint32_t>(ab_bf16) << 7)       // A format
         | (static_cast<uint32_t>(ab_bf16) << 10)      // B format
         | (static_cast<uint32_t>(N >> 3) << 17)       // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);      // M / 16
}

// Sparse variant (2:4 A): bit 2 = sparse; the metadata selector (bits 0..1) is 0.
__host__ __device__ constexpr uint32_t umma_idesc_f16_sparse(int M, int N, int ab_bf16) {
  return umma_idesc_f16(M, N, ab_bf16) | (1u << 2);
}

__device__ __forceinline__ void umma_f16_cg1(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_f16_cg2(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 2:4 sparse A: logical K = 32 per instruction; metadata at TMEM `e_tmem`.
template <int CG>
__device__ __forceinline__ void umma_f16_sp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t e_tmem,
                                            uint32_t idesc, uint32_t accumulate) {
  if constexpr (CG == 1)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.sp.cta_group::1.kind::f16 [%0], %1, %2, [%3], %4, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(e_tmem), "r"(idesc), "r"(accumulate)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.sp.cta_group::2.kind::f16 [%0], %1, %2, [%3], %4, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(e_tmem), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Shared memory -> TMEM copy of 128 rows x 128 bits (4 columns), source
// described by a matrix descriptor.
template <int CG>
__device__ __forceinline__ void tmem_cp_128x128b(uint32_t taddr, uint64_t sdesc) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.cp.cta_group::1.128x128b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
  else
    asm volatile("tcgen05.cp.cta_group::2.128x128b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Signal `bar` (this CTA) once all tcgen05 ops issued so far by this thread complete.
__device__ __forceinline__ void umma_commit_cg1(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// Pair version: arrive on the barrier at the same offset in every CTA of `mask`.
__device__ __forceinline__ void umma_commit_cg2_mc(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM -> registers. 32 lanes x 32 bit, 32 consecutive columns:
// thread t of the warp receives lane (base_lane + t), columns col..col+31.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace kb
