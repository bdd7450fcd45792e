// Microbenchmark probes for the Blackwell primitives the ladder is built on —
// the sm_100a counterparts of the reference's Hopper probes
// (kebab/lib/microbench/mma_wgmma.cu: one verified op, then a throughput loop;
// copy_gmem_to_smem_2d_tma_ptx.cu: TMA bandwidth):
//   umma_once    one 128 x 256 x 64 tcgen05.mma chain on constant operands,
//                read back with tcgen05.ld and checked (every D = 64).
//   umma_bench   back-to-back tcgen05.mma from one thread per CTA (or per CTA
//                pair with cta_group::2) into TMEM: tensor-core throughput.
//   umma_latency one MMA + commit + mbarrier wait, repeated: issue-to-done
//                latency in SM cycles.
//   tmem_ld      tcgen05.ld 32x32b.x32 + wait::ld loop on 4 warps: TMEM read
//                bandwidth per SM.
//   tma_load     each CTA streams a slice of a large global buffer through a
//                shared-memory ring with 2-D TMA loads: TMA / HBM read bandwidth.
//   tma_ingest   the same loop over an L2-resident slice, several passes, with
//                a chosen ring depth: bytes one SM takes in per cycle.
// A TMA-multicast probe is not built: multicast loads are kept out of every
// source file so that the library may run on several GPUs of this pool.
// Every wait is bounded (ptx.cuh).
#include <algorithm>
#include <vector>

#include "gemm_umma.cuh"
#include "internal.h"
#include "kebab/microbench.h"

namespace kb {

namespace {

constexpr int MB_N = 256;
constexpr int A_BYTES = 128 * 64 * 2;         // 128 rows x 64 K, 128-byte rows
constexpr int B_BYTES = MB_N * 64 * 2;        // 256 rows x 64 K
constexpr int MB_SMEM = 1024 + A_BYTES + B_BYTES + 64;

__device__ void fill_const(uint8_t* p, int bytes, uint16_t bits) {
  uint32_t w = bits | ((uint32_t)bits << 16);
  for (int i = threadIdx.x; i < bytes / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(p)[i] = w;
}

// Operands, barrier and TMEM slot, shared by the MMA probes.
struct MbSmem {
  uint8_t* A;
  uint8_t* B;
  uint64_t* bar;
  uint32_t* slot;
};

__device__ MbSmem mb_layout(uint8_t* raw) {
  uint8_t* s = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  MbSmem m;
  m.A = s;
  m.B = s + A_BYTES;
  m.bar = reinterpret_cast<uint64_t*>(s + A_BYTES + B_BYTES);
  m.slot = reinterpret_cast<uint32_t*>(m.bar + 1);
  return m;
}

// SP: tcgen05.mma.sp (2:4 A, K = 32 logical per instruction) with metadata
// "keep elements 0 and 1" of every group copied into TMEM columns 256..259.
template <int CG, bool SP = false>
__global__ void __launch_bounds__(128, 1) umma_probe_kernel(int iters, int n, int bf16, float* out, long long* cycles,
                                                            WaitCtx ctx) {
  extern __shared__ uint8_t smem_raw[];
  MbSmem m = mb_layout(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  fill_const(m.A, A_BYTES, bf16 ? 0x3F80 : 0x3C00);  // 1.0
  fill_const(m.B, B_BYTES, bf16 ? 0x3F80 : 0x3C00);
  fence_proxy_async_smem();  // generic writes -> visible to the tensor core
  if (threadIdx.x == 0) {
    mbar_init(m.bar, 1);
    fence_barrier_init();
  }
  constexpr uint32_t COLS = SP ? 512 : 256;
  if constexpr (SP) {
    // Metadata block (128 rows x 16 bytes): nibble p0 | p1 << 2 = 0 | 1 << 2.
    uint8_t* e = m.B + B_BYTES - 2048;
    for (int i = threadIdx.x; i < 2048; i += blockDim.x) e[i] = 0x44;
    fence_proxy_async_smem();
  }
  if (warp == 0) {
    tmem_alloc<CG>(m.slot, COLS);
    tmem_relinquish<CG>();
  }
  tc_fence_before();
  if constexpr (CG == 2) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *m.slot;
  const uint32_t idesc = SP ? umma_idesc_f16_sparse(128 * CG, n, bf16) : umma_idesc_f16(128 * CG, n, bf16);
  if (threadIdx.x == 0 && rank == 0) {
    if constexpr (SP)
      tmem_cp_128x128b<CG>(tmem + 256, umma_desc(smem_u32(m.B + B_BYTES - 2048), 16, 128, 0));
    const long long t0 = clock64();
    for (int i = 0; i < iters; ++i) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if constexpr (SP) {
          // A: 16 packed elements (32 bytes) per instruction; B: 32 K (64 bytes).
          const uint64_t ad = umma_desc_sw128(smem_u32(m.A) + k * 32);
          const uint64_t bd = umma_desc_sw128(smem_u32(m.B) + (k & 1) * 64);
          umma_f16_sp<CG>(tmem, ad, bd, tmem + 256 + (uint32_t)(k & 2), idesc | (uint32_t)(k & 1), (i | k) != 0);
        } else {
          const uint64_t ad = umma_desc_sw128(smem_u32(m.A) + k * 32), bd = umma_desc_sw128(smem_u32(m.B) + k * 32);
          if constexpr (CG == 1) umma_f16_cg1(tmem, ad, bd, idesc, (i | k) != 0);
          else umma_f16_cg2(tmem, ad, bd, idesc, (i | k) != 0);
        }
      }
    }
    if constexpr (CG == 1) umma_commit_cg1(m.bar);
    else umma_commit_cg2_mc(m.bar, 0x3);
    mbar_wait(m.bar, 0, ctx, SITE_MMA_DONE);
    if (cycles) cycles[blockIdx.x / CG] = clock64() - t0;
  } else if (threadIdx.x == 0 && CG == 2) {
    mbar_wait(m.bar, 0, ctx, SITE_MMA_DONE);  // the peer waits for the multicast commit
  }
  __syncthreads();
  tc_fence_after();
  if (out && blockIdx.x < CG) {
    // Read back D (this CTA's 128 lanes x n columns) into out[rank][lane][col].
    for (int c = 0; c < n; c += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, v);
      tmem_ld_wait();
      for (int j = 0; j < 32; ++j)
        out[((size_t)rank * 128 + warp * 32 + lane) * n + c + j] = __uint_as_float(v[j]);
    }
  }
  tc_fence_before();
  if constexpr (CG == 2) cluster_sync(); else __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc<CG>(tmem, COLS);
  }
}

__global__ void __launch_bounds__(128, 1) umma_latency_kernel(int iters, long long* cycles, WaitCtx ctx) {
  extern __shared__ uint8_t smem_raw[];
  MbSmem m = mb_layout(smem_raw);
  const int warp = threadIdx.x >> 5;
  fill_const(m.A, A_BYTES, 0x3C00);
  fill_const(m.B, B_BYTES, 0x3C00);
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(m.bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc<1>(m.slot, 256);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *m.slot;
  if (threadIdx.x == 0) {
    const uint32_t idesc = umma_idesc_f16(128, 256, 0);
    long long total = 0;
    for (int i = 0; i < iters; ++i) {
      const long long t0 = clock64();
      umma_f16_cg1(tmem, umma_desc_sw128(smem_u32(m.A)), umma_desc_sw128(smem_u32(m.B)), idesc, 0);
      umma_commit_cg1(m.bar);
      if (!mbar_wait(m.bar, (uint32_t)(i & 1), ctx, SITE_MMA_DONE)) break;
      total += clock64() - t0;
    }
    cycles[0] = total / (iters > 0 ? iters : 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc<1>(tmem, 256);
  }
}

__global__ void __launch_bounds__(128, 1) tmem_ld_kernel(int iters, long long* cycles, float* sink) {
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5;
  if (warp == 0) {
    tmem_alloc<1>(&slot, 256);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = slot + ((uint32_t)(warp * 32) << 16);
  uint32_t acc = 0;
  const long long t0 = clock64();
  for (int i = 0; i < iters; ++i) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(tmem + (uint32_t)((i * 32) & 255), v);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) acc ^= v[j];
  }
  const long long t1 = clock64();
  if (threadIdx.x == 0) cycles[blockIdx.x] = t1 - t0;
  if (acc == 0x12345u) sink[0] = (float)acc;  // keep the loads alive
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc<1>(slot, 256);
  }
}

// Streams rows [blockIdx.x * rows_per_cta, ...) of a [rows][cols] FP16 array
// through STAGES shared-memory slots of box_rows x 64 elements, `passes`
// times over (passes > 1 with a slice that stays in L2 measures what one SM
// can take in from L2). Thread 0 of each CTA records its SM cycles from the
// first load to the last arrival in cycles[blockIdx.x] when cycles != null.
constexpr int TMA_STAGES = 8;  // slots allocated; `stages` of them are used
__global__ void __launch_bounds__(64, 1) tma_load_kernel(const __grid_constant__ CUtensorMap tm, int rows_per_cta,
                                                         int box_rows, int col_boxes, int stages, int passes,
                                                         long long* cycles, WaitCtx ctx) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* s = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stage_bytes = box_rows * 128;
  uint64_t* full = reinterpret_cast<uint64_t*>(s + stages * stage_bytes);
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) mbar_init(&full[i], 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  const int row0 = blockIdx.x * rows_per_cta;
  const int per_pass = (rows_per_cta / box_rows) * col_boxes;
  const int nboxes = per_pass * passes;
  const long long t0 = clock64();
  // Keep `stages` loads in flight; the "consumer" only waits for arrival.
  for (int i = 0; i < nboxes + stages; ++i) {
    if (i >= stages) {
      const int j = i - stages;
      if (!mbar_wait(&full[j % stages], (uint32_t)((j / stages) & 1), ctx, SITE_FULL)) return;
    }
    if (i < nboxes) {
      const int st = i % stages, b = i % per_pass;
      mbar_arrive_expect_tx(&full[st], stage_bytes);
      tma_load_2d(s + st * stage_bytes, &tm, &full[st], (b % col_boxes) * 64, row0 + (b / col_boxes) * box_rows);
    }
  }
  if (cycles) cycles[blockIdx.x] = clock64() - t0;
}

struct Events {
  cudaEvent_t a, b;
  Events() {
    cudaEventCreate(&a);
    cudaEventCreate(&b);
  }
  ~Events() {
    cudaEventDestroy(a);
    cudaEventDestroy(b);
  }
  float ms() {
    float t = 0;
    cudaEventElapsedTime(&t, a, b);
    return t;
  }
};

int finish(cudaStream_t s, const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, what);
  return kebab_device_status(reinterpret_cast<kebab_stream_t>(s), nullptr, 1);
}

template <int CG, bool SP = false>
int launch_umma_probe(int grid_ctas, int iters, int n, int bf16, float* out, long long* cycles, cudaStream_t s) {
  WaitCtx ctx;
  int rc = wait_ctx(&ctx);
  if (rc) return rc;
  auto kern = umma_probe_kernel<CG, SP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MB_SMEM);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid_ctas);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = MB_SMEM;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CG;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, iters, n, bf16, out, cycles, ctx);
  if (e != cudaSuccess) return cuda_fail(e, "umma probe launch");
  return KEBAB_OK;
}

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" {

int kebab_mbench_umma_once(int ab_bf16, int cta_group, float* host_out, int64_t host_out_len) {
  if ((cta_group != 1 && cta_group != 2) || !host_out || host_out_len < 128LL * cta_group * MB_N)
    return fail(KEBAB_EINVAL, "umma_once: cta_group 1|2 and an output of 128*cta_group*256 floats");
  float* d = nullptr;
  cudaError_t e = cudaMalloc(&d, sizeof(float) * 128 * cta_group * MB_N);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  int rc = cta_group == 1 ? launch_umma_probe<1>(1, 1, MB_N, ab_bf16, d, nullptr, nullptr)
                          : launch_umma_probe<2>(2, 1, MB_N, ab_bf16, d, nullptr, nullptr);
  if (rc == KEBAB_OK) rc = finish(nullptr, "umma_once");
  if (rc == KEBAB_OK) {
    e = cudaMemcpy(host_out, d, sizeof(float) * 128 * cta_group * MB_N, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) rc = cuda_fail(e, "cudaMemcpy");
  }
  cudaFree(d);
  return rc;
}

int kebab_mbench_umma(int cta_group, int n, int ab_bf16, int iters, double* tflops, double* cycles_per_mma) {
  if ((cta_group != 1 && cta_group != 2) || n < 16 || n > 256 || n % 16 || iters <= 0)
    return fail(KEBAB_EINVAL, "umma: cta_group 1|2, n in 16..256 step 16, iters > 0");
  DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  const int grid = (dev->sm_count / cta_group) * cta_group;
  long long* cyc = nullptr;
  cudaError_t e = cudaMalloc(&cyc, sizeof(long long) * grid);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  Events ev;
  // warm-up, then the timed launch
  rc = cta_group == 1 ? launch_umma_probe<1>(grid, std::max(1, iters / 10), n, ab_bf16, nullptr, cyc, nullptr)
                      : launch_umma_probe<2>(grid, std::max(1, iters / 10), n, ab_bf16, nullptr, cyc, nullptr);
  if (rc == KEBAB_OK) rc = finish(nullptr, "umma warm-up");
  if (rc == KEBAB_OK) {
    cudaEventRecord(ev.a);
    rc = cta_group == 1 ? launch_umma_probe<1>(grid, iters, n, ab_bf16, nullptr, cyc, nullptr)
                        : launch_umma_probe<2>(grid, iters, n, ab_bf16, nullptr, cyc, nullptr);
    cudaEventRecord(ev.b);
    if (rc == KEBAB_OK) rc = finish(nullptr, "umma bench");
  }
  if (rc == KEBAB_OK) {
    std::vector<long long> h(grid / cta_group);
    cudaMemcpy(h.data(), cyc, sizeof(long long) * h.size(), cudaMemcpyDeviceToHost);
    long long mx = *std::max_element(h.begin(), h.end());
    // 4 MMAs of (128*cg) x n x 16 per iteration, per CTA (pair)
    const double flops = 2.0 * (128.0 * cta_group) * n * 64.0 * iters * (grid / cta_group);
    if (tflops) *tflops = flops / (ev.ms() * 1e-3) / 1e12;
    if (cycles_per_mma) *cycles_per_mma = (double)mx / (4.0 * iters);
  }
  cudaFree(cyc);
  return rc;
}


int kebab_mbench_umma_sp(int cta_group, int n, int iters, double* tflops, double* cycles_per_mma) {
  if ((cta_group != 1 && cta_group != 2) || n < 16 || n > 256 || n % 16 || iters <= 0)
    return fail(KEBAB_EINVAL, "umma_sp: cta_group 1|2, n in 16..256 step 16, iters > 0");
  DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  const int grid = (dev->sm_count / cta_group) * cta_group;
  long long* cyc = nullptr;
  cudaError_t e = cudaMalloc(&cyc, sizeof(long long) * grid);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  Events ev;
  rc = cta_group == 1 ? launch_umma_probe<1, true>(grid, std::max(1, iters / 10), n, 0, nullptr, cyc, nullptr)
                      : launch_umma_probe<2, true>(grid, std::max(1, iters / 10), n, 0, nullptr, cyc, nullptr);
  if (rc == KEBAB_OK) rc = finish(nullptr, "umma_sp warm-up");
  if (rc == KEBAB_OK) {
    cudaEventRecord(ev.a);
    rc = cta_group == 1 ? launch_umma_probe<1, true>(grid, iters, n, 0, nullptr, cyc, nullptr)
                        : launch_umma_probe<2, true>(grid, iters, n, 0, nullptr, cyc, nullptr);
    cudaEventRecord(ev.b);
    if (rc == KEBAB_OK) rc = finish(nullptr, "umma_sp bench");
  }
  if (rc == KEBAB_OK) {
    std::vector<long long> h(grid / cta_group);
    cudaMemcpy(h.data(), cyc, sizeof(long long) * h.size(), cudaMemcpyDeviceToHost);
    long long mx = *std::max_element(h.begin(), h.end());
    // 4 sparse MMAs of (128*cg) x n x 32 (logical K) per iteration, dense-equivalent FLOPs
    const double flops = 2.0 * (128.0 * cta_group) * n * 128.0 * iters * (grid / cta_group);
    if (tflops) *tflops = flops / (ev.ms() * 1e-3) / 1e12;
    if (cycles_per_mma) *cycles_per_mma = (double)mx / (4.0 * iters);
  }
  cudaFree(cyc);
  return rc;
}

int kebab_mbench_umma_latency(int iters, double* cycles) {
  if (iters <= 0 || !cycles) return fail(KEBAB_EINVAL, "umma_latency: iters > 0");
  WaitCtx ctx;
  int rc = wait_ctx(&ctx);
  if (rc) return rc;
  long long* d = nullptr;
  cudaError_t e = cudaMalloc(&d, sizeof(long long));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  e = cudaFuncSetAttribute(umma_latency_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, MB_SMEM);
  if (e == cudaSuccess) {
    umma_latency_kernel<<<1, 128, MB_SMEM>>>(iters, d, ctx);
    rc = finish(nullptr, "umma latency");
  } else {
    rc = cuda_fail(e, "cudaFuncSetAttribute");
  }
  long long h = 0;
  if (rc == KEBAB_OK) cudaMemcpy(&h, d, sizeof(h), cudaMemcpyDeviceToHost);
  *cycles = (double)h;
  cudaFree(d);
  return rc;
}

int kebab_mbench_tmem_ld(int iters, double* bytes_per_clk_per_sm, double* tbps) {
  if (iters <= 0) return fail(KEBAB_EINVAL, "tmem_ld: iters > 0");
  DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  long long* cyc = nullptr;
  float* sink = nullptr;
  cudaMalloc(&cyc, sizeof(long long) * dev->sm_count);
  cudaMalloc(&sink, sizeof(float));
  Events ev;
  tmem_ld_kernel<<<dev->sm_count, 128>>>(std::max(1, iters / 10), cyc, sink);
  rc = finish(nullptr, "tmem_ld warm-up");
  if (rc == KEBAB_OK) {
    cudaEventRecord(ev.a);
    tmem_ld_kernel<<<dev->sm_count, 128>>>(iters, cyc, sink);
    cudaEventRecord(ev.b);
    rc = finish(nullptr, "tmem_ld");
  }
  if (rc == KEBAB_OK) {
    std::vector<long long> h(dev->sm_count);
    cudaMemcpy(h.data(), cyc, sizeof(long long) * h.size(), cudaMemcpyDeviceToHost);
    const double bytes_per_cta = 4.0 * 32 * 32 * 4 * (double)iters;  // 4 warps x 32 lanes x 32 cols x 4 B
    const long long mx = *std::max_element(h.begin(), h.end());
    if (bytes_per_clk_per_sm) *bytes_per_clk_per_sm = bytes_per_cta / (double)mx;
    if (tbps) *tbps = bytes_per_cta * dev->sm_count / (ev.ms() * 1e-3) / 1e12;
  }
  cudaFree(cyc);
  cudaFree(sink);
  return rc;
}

int kebab_mbench_tma_load(const void* buf, int64_t rows, int64_t cols, int box_rows, double* gbps) {
  if (!buf || rows <= 0 || cols <= 0 || cols % 64 || box_rows <= 0 || box_rows > 256 || box_rows % 8 || !gbps)
    return fail(KEBAB_EINVAL, "tma_load: cols % 64 == 0, box_rows a multiple of 8 in 8..256");
  DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  WaitCtx ctx;
  if ((rc = wait_ctx(&ctx))) return rc;
  const int grid = dev->sm_count;
  int64_t rows_per_cta = (rows / grid) / box_rows * box_rows;
  if (rows_per_cta <= 0) return fail(KEBAB_EINVAL, "tma_load: buffer too small for one box per SM");
  CUtensorMap tm;
  if ((rc = make_tmap_2d(&tm, buf, KEBAB_F16, rows, cols, cols, box_rows, 64, true))) return rc;
  // As many slots as fit in ~200 KB (at most 8): 8 x 8 KB boxes .. 6 x 32 KB boxes.
  const int stages = std::max(2, std::min(TMA_STAGES, (200 * 1024) / (box_rows * 128)));
  const int smem = 1024 + stages * box_rows * 128 + 8 * stages + 64;
  cudaError_t e = cudaFuncSetAttribute(tma_load_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  Events ev;
  tma_load_kernel<<<grid, 64, smem>>>(tm, (int)rows_per_cta, box_rows, (int)(cols / 64), stages, 1, nullptr, ctx);
  if ((rc = finish(nullptr, "tma_load warm-up"))) return rc;
  cudaEventRecord(ev.a);
  tma_load_kernel<<<grid, 64, smem>>>(tm, (int)rows_per_cta, box_rows, (int)(cols / 64), stages, 1, nullptr, ctx);
  cudaEventRecord(ev.b);
  if ((rc = finish(nullptr, "tma_load"))) return rc;
  *gbps = (double)rows_per_cta * grid * cols * 2.0 / (ev.ms() * 1e-3) / 1e9;
  return KEBAB_OK;
}

int kebab_mbench_tma_ingest(const void* buf, int64_t rows, int64_t cols, int box_rows, int stages, int passes,
                            double* gbps, double* bytes_per_clk_per_sm) {
  if (!buf || rows <= 0 || cols <= 0 || cols % 64 || box_rows <= 0 || box_rows > 256 || box_rows % 8 || !gbps ||
      !bytes_per_clk_per_sm || passes <= 0 || stages < 1 || stages > TMA_STAGES || stages * box_rows * 128 > 200 * 1024)
    return fail(KEBAB_EINVAL, "tma_ingest: cols % 64 == 0, box_rows a multiple of 8 in 8..256, 1..8 stages of at "
                              "most 200 KB in all, passes > 0");
  DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  WaitCtx ctx;
  if ((rc = wait_ctx(&ctx))) return rc;
  const int grid = dev->sm_count;
  const int64_t rows_per_cta = (rows / grid) / box_rows * box_rows;
  if (rows_per_cta <= 0) return fail(KEBAB_EINVAL, "tma_ingest: buffer too small for one box per SM");
  if ((rows_per_cta / box_rows) * (cols / 64) * passes > INT32_MAX) return fail(KEBAB_EINVAL, "tma_ingest: too many boxes");
  CUtensorMap tm;
  if ((rc = make_tmap_2d(&tm, buf, KEBAB_F16, rows, cols, cols, box_rows, 64, true))) return rc;
  const int smem = 1024 + stages * box_rows * 128 + 8 * stages + 64;
  cudaError_t e = cudaFuncSetAttribute(tma_load_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  long long* cyc = nullptr;
  if ((e = cudaMalloc(&cyc, sizeof(long long) * grid)) != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  Events ev;
  // One pass brings the slices into L2; the timed launch then reads them `passes` times.
  tma_load_kernel<<<grid, 64, smem>>>(tm, (int)rows_per_cta, box_rows, (int)(cols / 64), stages, 1, nullptr, ctx);
  rc = finish(nullptr, "tma_ingest warm-up");
  if (!rc) {
    cudaEventRecord(ev.a);
    tma_load_kernel<<<grid, 64, smem>>>(tm, (int)rows_per_cta, box_rows, (int)(cols / 64), stages, passes, cyc, ctx);
    cudaEventRecord(ev.b);
    rc = finish(nullptr, "tma_ingest");
  }
  if (!rc) {
    std::vector<long long> h(grid);
    e = cudaMemcpy(h.data(), cyc, sizeof(long long) * grid, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
      rc = cuda_fail(e, "cudaMemcpy");
    } else {
      std::sort(h.begin(), h.end());
      const double bytes_cta = (double)rows_per_cta * cols * 2.0 * passes;
      *gbps = bytes_cta * grid / (ev.ms() * 1e-3) / 1e9;
      *bytes_per_clk_per_sm = bytes_cta / (double)h[grid / 2];
    }
  }
  cudaFree(cyc);
  return rc;
}

}  // extern "C"
