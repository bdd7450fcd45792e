// Host runtime of libkebab_b200.so: error plumbing, per-device state (SM
// count, the device status word), TMA descriptor encoding, the wait-timeout
// probe kernel.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "internal.h"

namespace kb {

// Status word that kernels set when a bounded wait expires. One per device
// (a __device__ variable is instantiated in every context that loads the
// module); kernels receive its address as a parameter.
__device__ uint32_t g_device_status_word;

namespace {
thread_local std::string t_last_error;
std::mutex g_mu;
std::vector<DeviceInfo*> g_devices;
uint64_t g_timeout_ns = 0;  // 0 = not yet initialised
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

uint64_t default_timeout_ns() {
  const char* e = std::getenv("KEBAB_WAIT_TIMEOUT_MS");
  if (e && *e) {
    long long ms = std::atoll(e);
    if (ms > 0) return (uint64_t)ms * 1000000ull;
  }
  return 2000ull * 1000000ull;
}
}  // namespace

void set_error(const std::string& msg) { t_last_error = msg; }

namespace {
thread_local unsigned long long* t_probe = nullptr;
thread_local int64_t t_probe_ctas = 0;
}  // namespace

unsigned long long* take_clock_probe(int ctas) {
  unsigned long long* p = t_probe;
  if (!p || ctas > t_probe_ctas) return nullptr;
  t_probe = nullptr;
  t_probe_ctas = 0;
  return p;
}

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(KEBAB_ECUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

int device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lk(g_mu);
  if ((int)g_devices.size() <= dev) g_devices.resize(dev + 1, nullptr);
  if (!g_devices[dev]) {
    auto* d = new DeviceInfo();
    d->device = dev;
    if ((e = cudaDeviceGetAttribute(&d->sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d->cc_major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&d->cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess) {
      delete d;
      return cuda_fail(e, "cudaDeviceGetAttribute");
    }
    void* p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, g_device_status_word)) != cudaSuccess) {
      delete d;
      return cuda_fail(e, "cudaGetSymbolAddress(status word)");
    }
    d->status = static_cast<uint32_t*>(p);
    g_devices[dev] = d;
  }
  *out = g_devices[dev];
  if ((*out)->cc_major != 10) {
    return fail(KEBAB_ENOTSUP, "kebab-b200 kernels are built for sm_100a only; device " + std::to_string(dev) +
                                   " is sm_" + std::to_string((*out)->cc_major) + std::to_string((*out)->cc_minor));
  }
  return KEBAB_OK;
}

int wait_ctx(WaitCtx* out) {
  DeviceInfo* d = nullptr;
  int rc = device_info(&d);
  if (rc) return rc;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_timeout_ns == 0) g_timeout_ns = default_timeout_ns();
    out->timeout_ns = g_timeout_ns;
  }
  out->status = d->status;
  return KEBAB_OK;
}

int kps_env(int dflt) {
  const char* e = std::getenv("KEBAB_KPS");
  if (e && e[0] == '1') return 1;
  if (e && e[0] == '2') return 2;
  return dflt;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("KEBAB_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

static int get_encoder() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_encode) return KEBAB_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return fail(KEBAB_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return KEBAB_OK;
}


namespace {
// Tensor maps are cached per (device, base pointer, dtype, shape, pitch, box,
// swizzle): encoding one costs about a microsecond of host time, and a GEMM
// needs three. Bounded: the map is cleared when it reaches kTmapCap entries
// (callers cycling through many buffers re-encode), and by kebab_shutdown().
struct TmapKey {
  int dev, dtype, swizzle;
  const void* base;
  uint64_t rows, cols, ld;
  uint32_t box_rows, box_cols;
  bool operator==(const TmapKey& o) const {
    return dev == o.dev && dtype == o.dtype && swizzle == o.swizzle && base == o.base && rows == o.rows &&
           cols == o.cols && ld == o.ld && box_rows == o.box_rows && box_cols == o.box_cols;
  }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    uint64_t h = reinterpret_cast<uintptr_t>(k.base) * 0x9E3779B97F4A7C15ull;
    for (uint64_t v : {(uint64_t)k.dev, (uint64_t)k.dtype, (uint64_t)k.swizzle, k.rows, k.cols, k.ld,
                       (uint64_t)k.box_rows << 32 | k.box_cols})
      h = (h ^ v) * 0x100000001B3ull;
    return (size_t)h;
  }
};
constexpr size_t kTmapCap = 4096;
std::mutex g_tmap_mu;
std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> g_tmaps;
}  // namespace

int make_tmap_2d_sw(CUtensorMap* out, const void* base, int dtype, uint64_t rows, uint64_t cols, uint64_t ld,
                    uint32_t box_rows, uint32_t box_cols, int swizzle_bytes) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(KEBAB_EINVAL, "TMA operand base address is not 16-byte aligned");
  if ((ld * 2) % 16 != 0) return fail(KEBAB_EINVAL, "TMA operand row pitch is not a multiple of 16 bytes");
  int dev = 0;
  (void)cudaGetDevice(&dev);
  const TmapKey key{dev, dtype, swizzle_bytes, base, rows, cols, ld, box_rows, box_cols};
  {
    std::lock_guard<std::mutex> lk(g_tmap_mu);
    auto it = g_tmaps.find(key);
    if (it != g_tmaps.end()) {
      *out = it->second;
      return KEBAB_OK;
    }
  }
  int rc = get_encoder();
  if (rc) return rc;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapDataType t = dtype == KEBAB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = g_encode(out, t, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                        : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                        : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                              : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KEBAB_EINVAL, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(r));
  std::lock_guard<std::mutex> lk(g_tmap_mu);
  if (g_tmaps.size() >= kTmapCap) g_tmaps.clear();
  g_tmaps.emplace(key, *out);
  return KEBAB_OK;
}

int make_tmap_2d(CUtensorMap* out, const void* base, int dtype, uint64_t rows, uint64_t cols, uint64_t ld,
                 uint32_t box_rows, uint32_t box_cols, bool swizzle128) {
  return make_tmap_2d_sw(out, base, dtype, rows, cols, ld, box_rows, box_cols, swizzle128 ? 128 : 0);
}

int check_tma_shapes(const GemmProblem& p) {
  if ((reinterpret_cast<uintptr_t>(p.A) | reinterpret_cast<uintptr_t>(p.B) | reinterpret_cast<uintptr_t>(p.C)) & 15u)
    return fail(KEBAB_EINVAL, "A, B and C must be 16-byte aligned for the TMA rungs");
  const bool needK = p.lhs == 'R' || p.rhs == 'C';
  const bool needM = p.lhs == 'C' || !p.c_row;
  const bool needN = p.rhs == 'R' || p.c_row;
  if (needK && p.K % 8 != 0)
    return fail(KEBAB_EINVAL, "K must be a multiple of 8 (16-byte rows of A / B) for the TMA rungs");
  if (needM && p.M % 8 != 0)
    return fail(KEBAB_EINVAL, "M must be a multiple of 8 (16-byte pitch of A or C) for the TMA rungs");
  if (needN && p.N % 8 != 0)
    return fail(KEBAB_EINVAL, "N must be a multiple of 8 (16-byte pitch of B or C) for the TMA rungs");
  if (p.M > INT32_MAX || p.N > INT32_MAX || p.K > INT32_MAX)
    return fail(KEBAB_EINVAL, "each of M, N, K must fit in int32 for the TMA rungs");
  return KEBAB_OK;
}

namespace {
struct SkWorkspace {
  void* base = nullptr;
  size_t ws_bytes = 0, flags = 0;
  uint32_t epoch = 0;
};
std::map<std::pair<int, cudaStream_t>, SkWorkspace> g_sk;
}  // namespace

int sk_workspace(cudaStream_t stream, size_t ws_bytes, size_t flags, float** ws, uint32_t** flag_ptr,
                 uint32_t* epoch) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lk(g_mu);
  SkWorkspace& w = g_sk[{dev, stream}];
  if (w.ws_bytes < ws_bytes || w.flags < flags) {
    if (w.base) {
      cudaStreamSynchronize(stream);
      cudaFree(w.base);
      w.base = nullptr;
    }
    const size_t ws_round = (ws_bytes + 255) & ~size_t(255);
    if ((e = cudaMalloc(&w.base, ws_round + flags * sizeof(uint32_t))) != cudaSuccess)
      return cuda_fail(e, "cudaMalloc(stream-K workspace)");
    if ((e = cudaMemset(static_cast<uint8_t*>(w.base) + ws_round, 0, flags * sizeof(uint32_t))) != cudaSuccess)
      return cuda_fail(e, "cudaMemset(stream-K flags)");
    w.ws_bytes = ws_round;
    w.flags = flags;
    w.epoch = 0;
  }
  *ws = static_cast<float*>(w.base);
  *flag_ptr = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(w.base) + w.ws_bytes);
  if (++w.epoch == 0) ++w.epoch;  // 0 is the value of never-written flags
  *epoch = w.epoch;
  return KEBAB_OK;
}

// ---------------------------------------------------------------------------
// Deliberate-timeout probe: one warp waits on an mbarrier that nothing will
// ever arrive at; the bounded wait expires, records the error and returns.
// ---------------------------------------------------------------------------
__global__ void probe_wait_kernel(WaitCtx ctx) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, ctx, SITE_PROBE);
  __syncthreads();
}

}  // namespace kb

using namespace kb;

extern "C" {

const char* kebab_last_error(void) { return t_last_error.c_str(); }

int kebab_clock_probe(void* buf, int64_t max_ctas) {
  if ((buf == nullptr) != (max_ctas == 0) || max_ctas < 0 || (reinterpret_cast<uintptr_t>(buf) & 7u))
    return fail(KEBAB_EINVAL, "clock probe: need an 8-byte aligned buffer and a positive CTA count, or null and 0");
  t_probe = static_cast<unsigned long long*>(buf);
  t_probe_ctas = max_ctas;
  return KEBAB_OK;
}

int kebab_set_wait_timeout_us(uint64_t timeout_us) {
  if (timeout_us == 0) return fail(KEBAB_EINVAL, "timeout must be positive");
  std::lock_guard<std::mutex> lk(g_mu);
  g_timeout_ns = timeout_us * 1000ull;
  return KEBAB_OK;
}

int kebab_device_status(kebab_stream_t stream, uint32_t* code, int clear) {
  DeviceInfo* d = nullptr;
  int rc = device_info(&d);
  if (rc) return rc;
  cudaError_t e = cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  uint32_t w = 0;
  if ((e = cudaMemcpy(&w, d->status, sizeof(w), cudaMemcpyDeviceToHost)) != cudaSuccess)
    return cuda_fail(e, "reading the device status word");
  if (code) *code = w;
  if (clear && w) {
    uint32_t z = 0;
    if ((e = cudaMemcpy(d->status, &z, sizeof(z), cudaMemcpyHostToDevice)) != cudaSuccess)
      return cuda_fail(e, "clearing the device status word");
  }
  if (w) {
    char buf[160];
    std::snprintf(buf, sizeof(buf), "device wait timed out: class %u, site %u, block %u", w & 0xFFu, (w >> 8) & 0xFFu,
                  w >> 16);
    return fail(KEBAB_ETIMEOUT, buf);
  }
  return KEBAB_OK;
}

int kebab_probe_wait_timeout(kebab_stream_t stream, uint64_t timeout_us) {
  WaitCtx ctx;
  int rc = wait_ctx(&ctx);
  if (rc) return rc;
  // Start from a clean word so the result reflects this probe only.
  rc = kebab_device_status(stream, nullptr, 1);
  if (rc != KEBAB_OK && rc != KEBAB_ETIMEOUT) return rc;
  ctx.timeout_ns = timeout_us * 1000ull;
  probe_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(ctx);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "probe launch");
  return kebab_device_status(stream, nullptr, 1);
}

void kebab_shutdown(void) {
  noalloc_reset();
  {
    std::lock_guard<std::mutex> lk(g_tmap_mu);
    g_tmaps.clear();
  }
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto& kv : g_sk)
    if (kv.second.base) cudaFree(kv.second.base);
  g_sk.clear();
  for (auto* d : g_devices) delete d;
  g_devices.clear();
}

}  // extern "C"
