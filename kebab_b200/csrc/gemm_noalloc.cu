// kebab_gemm_streamk_noalloc: the stream-K pair GEMM (rung 109) for callers
// that must not allocate device memory.
//
// Who needs it: code running where cudaMalloc is unavailable or forbidden —
// for instance inside a framework's custom allocator or memory-pool callback,
// a pre-allocated real-time serving loop with a fixed memory budget, or a
// plugin whose host forbids allocation after start-up. The regular entry
// point allocates its stream-K workspace on first use; this one does not.
//
// Instead the partial tiles and their ready flags live in a file-scope static
// device array of a fixed size, present on every GPU that loads the library
// until the process exits: kNoallocSlots slots of 128 x 256 FP32 (128 KiB
// each, one per CTA) = 20 MiB, plus kNoallocSlots * 4 flags. A device whose
// stream-K grid needs more CTAs than kNoallocSlots is rejected with
// KEBAB_ENOTSUP. Host code cannot use the array's name as a device address,
// so a per-device set-up (with that device current) looks the address up with
// cudaGetSymbolAddress and keeps it. The set-up is also the moment the CUDA
// driver loads this file's module onto the device (lazy module loading), which
// is when the 20 MiB array and the kernels' code are committed: it is the one
// step that may allocate. It runs on the first call per device, or explicitly
// with a set-up-only call (null pointers and M = N = K = 0); make that call
// before entering the code that must not allocate, and before any stream
// capture. Every call shares the one array: the flags are cleared on the
// stream at the start of each call (cudaMemsetAsync, which allocates nothing)
// and the partials are fully rewritten before they are read, so calls that
// overlap on the GPU (different streams, or concurrent host threads) race and
// must be serialised by the caller.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "gemm_umma.cuh"
#include "internal.h"
#include "kebab/kebab.h"

namespace kb {
namespace {

constexpr int kNoallocSlots = 160;                  // CTAs covered (148 on B200)
constexpr int kNoallocBN = 256, kNoallocStages = 6;  // the rung-109 configuration
constexpr size_t kSlotFloats = 128 * kNoallocBN;

struct alignas(256) NoallocScratch {
  float partials[kNoallocSlots * kSlotFloats];  // 20 MiB
  uint32_t flags[kNoallocSlots * 4];
};
static __device__ __align__(256) NoallocScratch g_noalloc_scratch;

struct NoallocDevice {
  bool ready = false;
  NoallocScratch* scratch = nullptr;
  int max_clusters = 0;
};
std::mutex g_noalloc_mu;
NoallocDevice g_noalloc_dev[64];

template <typename T>
cudaError_t opt_in(int sm_count, int* max_clusters) {
  using L = UmmaSmem<kNoallocBN, kNoallocStages, 2>;
  auto kern = gemm_umma_ws_kernel<T, kNoallocBN, kNoallocStages, 2, true, 0, true>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t qc = {};
  qc.gridDim = dim3(2 * (sm_count / 2), 1, 1);
  qc.blockDim = dim3(UmmaEpi<kNoallocBN>::THREADS, 1, 1);
  qc.dynamicSmemBytes = L::ALLOC;
  cudaLaunchAttribute qa[1];
  qa[0].id = cudaLaunchAttributeClusterDimension;
  qa[0].val.clusterDim.x = 2;
  qa[0].val.clusterDim.y = 1;
  qa[0].val.clusterDim.z = 1;
  qc.attrs = qa;
  qc.numAttrs = 1;
  int n = 0;
  e = cudaOccupancyMaxActiveClusters(&n, kern, &qc);
  (void)cudaGetLastError();
  *max_clusters = std::min(sm_count / 2, (e == cudaSuccess && n > 0) ? n : sm_count / 2);
  return cudaSuccess;
}

// Once per device, with that device current: the device address of the
// static scratch, both dtypes' shared-memory opt-in (which also loads their
// code) and the pair count. Everything a later call needs, so later calls
// allocate nothing.
int setup_device(NoallocDevice** out) {
  DeviceInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  if (dev->device >= 64) return fail(KEBAB_ENOTSUP, "no-alloc GEMM supports device ids below 64");
  NoallocDevice& nd = g_noalloc_dev[dev->device];
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!nd.ready) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    int c16 = 0, c_bf16 = 0;
    if ((e = opt_in<__half>(dev->sm_count, &c16)) != cudaSuccess ||
        (e = opt_in<__nv_bfloat16>(dev->sm_count, &c_bf16)) != cudaSuccess)
      return cuda_fail(e, "cudaFuncSetAttribute(no-alloc stream-K kernel)");
    nd.max_clusters = std::min(c16, c_bf16);
    nd.scratch = static_cast<NoallocScratch*>(ptr);
    nd.ready = true;
  }
  *out = &nd;
  return KEBAB_OK;
}

template <typename T>
int launch_noalloc(const GemmProblem& p) {
  using L = UmmaSmem<kNoallocBN, kNoallocStages, 2>;
  auto kern = gemm_umma_ws_kernel<T, kNoallocBN, kNoallocStages, 2, true, 0, true>;
  NoallocDevice* ndp = nullptr;
  int rc = setup_device(&ndp);
  if (rc) return rc;
  NoallocDevice& nd = *ndp;
  const int clusters = nd.max_clusters;
  if (2 * clusters > kNoallocSlots)
    return fail(KEBAB_ENOTSUP, "no-alloc GEMM: this device needs " + std::to_string(2 * clusters) +
                                   " stream-K slots, the static scratch holds " + std::to_string(kNoallocSlots));

  UmmaArgs args;
  if ((rc = wait_ctx(&args.ctx))) return rc;
  CUtensorMap tA, tB, tC;
  if ((rc = make_tmap_2d(&tA, p.A, p.dtype, p.M, p.K, p.K, 128, 64, true))) return rc;
  if ((rc = make_tmap_2d(&tB, p.B, p.dtype, p.N, p.K, p.K, kNoallocBN / 2, 64, true))) return rc;
  if ((rc = make_tmap_2d(&tC, p.C, p.dtype, p.N, p.M, p.M, 32, 32, false))) return rc;
  args.M = (int)p.M;
  args.N = (int)p.N;
  args.K = (int)p.K;
  args.tiles_m = (int)((p.M + 255) / 256);
  args.tiles_n = (int)((p.N + kNoallocBN - 1) / kNoallocBN);
  args.epi_backoff_ns = 0;
  args.l2_hint = 0;
  const long long tiles = (long long)args.tiles_m * args.tiles_n;
  if (tiles > INT32_MAX / 2) return fail(KEBAB_EINVAL, "too many tiles");
  {
    const double target = std::sqrt((double)clusters * kNoallocBN / 256.0);
    int best = 1;
    double best_err = 1e30;
    for (int d = 1; d <= args.tiles_m; ++d)
      if (args.tiles_m % d == 0 && std::fabs(std::log(d / target)) <= best_err + 1e-9) {
        best = d;
        best_err = std::fabs(std::log(d / target));
      }
    args.group_m = best;
  }
  // Same split as rung 109: whole tiles round robin, then the last partial
  // wave plus one full wave by K-iterations.
  const long long waves = tiles / clusters, rem = tiles % clusters;
  args.sk_tiles = rem ? (int)(waves >= 1 ? rem + clusters : rem) : 0;
  args.dp_tiles = (int)(tiles - args.sk_tiles);
  args.ws = nd.scratch->partials;
  args.flags = nd.scratch->flags;
  args.epoch = 1;
  // The scratch keeps the previous call's contents: clear the flags first.
  cudaError_t e = cudaMemsetAsync(nd.scratch->flags, 0, sizeof(nd.scratch->flags), p.stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(no-alloc flags)");

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.blockDim = dim3(UmmaEpi<kNoallocBN>::THREADS, 1, 1);
  cfg.dynamicSmemBytes = L::ALLOC;
  cfg.stream = p.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tA, tB, tC, args);
  if (e != cudaSuccess) return cuda_fail(e, "no-alloc stream-K launch");
  return KEBAB_OK;
}

}  // namespace

// Called by kebab_shutdown(): forget every device's set-up, so a call after a
// device reset looks the address up and opts in again.
void noalloc_reset() {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  for (auto& d : g_noalloc_dev) d = NoallocDevice();
}

}  // namespace kb

using namespace kb;

extern "C" int kebab_gemm_streamk_noalloc(kebab_dtype dtype, const void* A, const void* B, void* C, int64_t M,
                                          int64_t N, int64_t K, kebab_stream_t stream) {
  if (!A && !B && !C && M == 0 && N == 0 && K == 0) {
    // Set-up only: the per-device step that may allocate (see above).
    NoallocDevice* nd = nullptr;
    (void)stream;
    return setup_device(&nd);
  }
  if (!A || !B || !C) return fail(KEBAB_EINVAL, "null pointer passed to kebab_gemm_streamk_noalloc");
  if (M <= 0 || N <= 0 || K <= 0) return fail(KEBAB_EINVAL, "invalid dimensions");
  if (dtype != KEBAB_F16 && dtype != KEBAB_BF16) return fail(KEBAB_EINVAL, "no-alloc GEMM supports F16 and BF16");
  GemmProblem p{(int)dtype, A, B, C, M, N, K, 'R', 'C', false, reinterpret_cast<cudaStream_t>(stream)};
  int rc = check_tma_shapes(p);
  if (rc) return rc;
  return dtype == KEBAB_F16 ? launch_noalloc<__half>(p) : launch_noalloc<__nv_bfloat16>(p);
}
