// Broadcast of B overlapped with the GEMM that consumes it, without SMs.
//
// The M-sharded GEMM (every rank owns a row block of A and needs all of B)
// starts with a broadcast of B from rank 0. Here that broadcast is a chain of
// copy-engine pulls over NVLink: rank r copies B chunk by chunk from rank
// r - 1's buffer (mapped into this process with CUDA IPC), each chunk as soon
// as rank r - 1 holds it. After each chunk's copy a stream memory operation
// raises a device flag, and the GEMM (kebab_gemm_gated, launched first on
// another stream) makes its TMA producer wait, bounded, on the flag of the
// chunk a tile needs. Copy engines and stream memory operations use no SMs,
// so the persistent GEMM keeps every SM while B streams in, and its TMA
// loads only ever read this GPU's own memory.
//
// Which rank holds which chunk is published through a small block of host
// shared memory (one uint32 per rank and chunk, holding the call's epoch):
// every rank's host thread polls its own copy events and publishes, and
// polls its predecessor's slots before issuing the next pull. Every wait is
// bounded.
//
// No counterpart in the reference, which has no multi-GPU code.
#include <cudaTypedefs.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <map>
#include <mutex>
#include <thread>
#include <vector>

#include "internal.h"
#include "kebab/peer.h"

namespace kb {
namespace {

std::mutex g_peer_mu;
PFN_cuMemGetAddressRange_v3020 g_addr_range = nullptr;
PFN_cuStreamWriteValue32_v11070 g_write_value = nullptr;

int driver_fn(const char* name, int version, void** out) {
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPointByVersion(name, out, version, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !*out)
    return fail(KEBAB_ECUDA, std::string(name) + " entry point unavailable");
  return KEBAB_OK;
}

int peer_fns() {
  std::lock_guard<std::mutex> lk(g_peer_mu);
  int rc;
  if (!g_addr_range && (rc = driver_fn("cuMemGetAddressRange", 3020, reinterpret_cast<void**>(&g_addr_range))))
    return rc;
  if (!g_write_value && (rc = driver_fn("cuStreamWriteValue32", 11070, reinterpret_cast<void**>(&g_write_value))))
    return rc;
  return KEBAB_OK;
}

// Opened IPC mappings by allocation base in this process (one open per
// exported allocation, reference counted).
struct Mapping {
  void* base;
  int refs;
};
std::map<std::string, Mapping> g_maps;

std::string handle_key(const cudaIpcMemHandle_t& h) { return std::string(h.reserved, sizeof(h.reserved)); }

// Copy-completion events, reused across calls on this host thread.
thread_local std::vector<cudaEvent_t> t_events;

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" {

int kebab_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  if (!ptr || !handle || !offset) return fail(KEBAB_EINVAL, "null pointer passed to kebab_ipc_export");
  int rc = peer_fns();
  if (rc) return rc;
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = g_addr_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(KEBAB_EINVAL, "cuMemGetAddressRange failed: not a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
  return KEBAB_OK;
}

int kebab_ipc_open(const void* handle, int64_t offset, void** ptr) {
  if (!handle || !ptr || offset < 0) return fail(KEBAB_EINVAL, "bad arguments to kebab_ipc_open");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  std::lock_guard<std::mutex> lk(g_peer_mu);
  auto it = g_maps.find(handle_key(h));
  if (it == g_maps.end()) {
    void* base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    it = g_maps.emplace(handle_key(h), Mapping{base, 0}).first;
  }
  ++it->second.refs;
  *ptr = static_cast<uint8_t*>(it->second.base) + offset;
  return KEBAB_OK;
}

int kebab_ipc_close(const void* handle) {
  if (!handle) return fail(KEBAB_EINVAL, "null handle passed to kebab_ipc_close");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  std::lock_guard<std::mutex> lk(g_peer_mu);
  auto it = g_maps.find(handle_key(h));
  if (it == g_maps.end()) return fail(KEBAB_EINVAL, "kebab_ipc_close: handle is not open");
  if (--it->second.refs == 0) {
    cudaError_t e = cudaIpcCloseMemHandle(it->second.base);
    g_maps.erase(it);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  }
  return KEBAB_OK;
}

int kebab_flag_write(uint32_t* flag, uint32_t value, kebab_stream_t stream) {
  if (!flag) return fail(KEBAB_EINVAL, "null flag passed to kebab_flag_write");
  int rc = peer_fns();
  if (rc) return rc;
  CUresult r = g_write_value(reinterpret_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(flag), value, 0);
  if (r != CUDA_SUCCESS) return fail(KEBAB_ECUDA, "cuStreamWriteValue32 failed with CUresult " + std::to_string(r));
  return KEBAB_OK;
}

int kebab_ring_pull(void* dst, const void* src, int64_t chunk_bytes, int64_t total_bytes, uint32_t* ready,
                    uint32_t epoch, const uint32_t* have_src, uint32_t* have_mine, kebab_stream_t stream,
                    kebab_stream_t stream2, uint64_t timeout_us) {
  if (!dst || !have_mine || chunk_bytes <= 0 || total_bytes <= 0 || (src && (!have_src || !ready)))
    return fail(KEBAB_EINVAL, "bad arguments to kebab_ring_pull");
  if (epoch == 0) return fail(KEBAB_EINVAL, "kebab_ring_pull: epoch 0 is the value of never-written slots");
  int rc = peer_fns();
  if (rc) return rc;
  const int64_t nchunks = (total_bytes + chunk_bytes - 1) / chunk_bytes;
  auto* mine = reinterpret_cast<std::atomic<uint32_t>*>(have_mine);
  if (!src) {
    // The source rank holds every chunk already.
    for (int64_t j = 0; j < nchunks; ++j) mine[j].store(epoch, std::memory_order_release);
    return KEBAB_OK;
  }
  const auto* prev = reinterpret_cast<const std::atomic<uint32_t>*>(have_src);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaStream_t s2 = reinterpret_cast<cudaStream_t>(stream2);
  while ((int64_t)t_events.size() < 2 * nchunks) {
    cudaEvent_t ev;
    cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
    t_events.push_back(ev);
  }
  auto deadline = std::chrono::steady_clock::now() + std::chrono::microseconds(timeout_us);
  int64_t issued = 0, published = 0;
  // Publish every chunk whose copy has completed, in order.
  auto publish = [&]() -> int {
    while (published < issued) {
      cudaError_t e = cudaEventQuery(t_events[published]);
      if (e == cudaErrorNotReady) break;
      if (e != cudaSuccess) return cuda_fail(e, "cudaEventQuery(chunk copy)");
      mine[published].store(epoch, std::memory_order_release);
      ++published;
    }
    return KEBAB_OK;
  };
  while (published < nchunks) {
    bool progressed = false;
    if (issued < nchunks && prev[issued].load(std::memory_order_acquire) == epoch) {
      const int64_t off = issued * chunk_bytes;
      const int64_t n = std::min(chunk_bytes, total_bytes - off);
      // With a second stream the chunk is split in two copies that can run
      // on two copy engines; the flag waits for both.
      const int64_t n1 = s2 ? std::min(n, ((n / 2) + 255) / 256 * 256) : n;
      uint8_t* d = static_cast<uint8_t*>(dst) + off;
      const uint8_t* sp = static_cast<const uint8_t*>(src) + off;
      cudaError_t e = cudaMemcpyAsync(d, sp, (size_t)n1, cudaMemcpyDeviceToDevice, s);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(chunk from the previous rank)");
      if (s2 && n > n1) {
        cudaEvent_t half = t_events[nchunks + issued];
        if ((e = cudaMemcpyAsync(d + n1, sp + n1, (size_t)(n - n1), cudaMemcpyDeviceToDevice, s2)) != cudaSuccess)
          return cuda_fail(e, "cudaMemcpyAsync(second half of a chunk)");
        if ((e = cudaEventRecord(half, s2)) != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
        if ((e = cudaStreamWaitEvent(s, half, 0)) != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent");
      }
      CUresult r = g_write_value(reinterpret_cast<CUstream>(s), reinterpret_cast<CUdeviceptr>(ready + issued), epoch, 0);
      if (r != CUDA_SUCCESS) return fail(KEBAB_ECUDA, "cuStreamWriteValue32 failed with CUresult " + std::to_string(r));
      if ((e = cudaEventRecord(t_events[issued], s)) != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
      ++issued;
      progressed = true;
    }
    const int64_t before = published;
    if ((rc = publish())) return rc;
    if (published != before) progressed = true;
    if (progressed) {
      deadline = std::chrono::steady_clock::now() + std::chrono::microseconds(timeout_us);
    } else {
      if (std::chrono::steady_clock::now() > deadline)
        return fail(KEBAB_ETIMEOUT, "kebab_ring_pull: timed out with " + std::to_string(issued) + " of " +
                                        std::to_string(nchunks) + " chunks issued and " + std::to_string(published) +
                                        " published");
      std::this_thread::yield();
    }
  }
  return KEBAB_OK;
}

int kebab_chain_push(const void* src, void* dst_next, int64_t chunk_bytes, int64_t total_bytes, uint32_t* ready_next,
                     uint32_t epoch, const uint32_t* have_mine, uint32_t* have_next, kebab_stream_t stream,
                     kebab_stream_t stream2, uint64_t timeout_us) {
  if (!src || chunk_bytes <= 0 || total_bytes <= 0 || (dst_next && (!ready_next || !have_next)) ||
      (!dst_next && !have_mine))
    return fail(KEBAB_EINVAL, "bad arguments to kebab_chain_push");
  if (epoch == 0) return fail(KEBAB_EINVAL, "kebab_chain_push: epoch 0 is the value of never-written slots");
  int rc = peer_fns();
  if (rc) return rc;
  const int64_t nchunks = (total_bytes + chunk_bytes - 1) / chunk_bytes;
  const auto* mine = reinterpret_cast<const std::atomic<uint32_t>*>(have_mine);
  auto* next = reinterpret_cast<std::atomic<uint32_t>*>(have_next);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaStream_t s2 = reinterpret_cast<cudaStream_t>(stream2);
  while ((int64_t)t_events.size() < 2 * nchunks) {
    cudaEvent_t ev;
    cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
    t_events.push_back(ev);
  }
  auto deadline = std::chrono::steady_clock::now() + std::chrono::microseconds(timeout_us);
  int64_t issued = 0, published = 0;
  const int64_t goal = dst_next ? nchunks : 0;  // the last rank forwards nothing
  int64_t arrived = 0;                          // last rank: chunks seen landed
  while (published < goal || (!dst_next && arrived < nchunks)) {
    bool progressed = false;
    if (!dst_next) {
      while (arrived < nchunks && mine[arrived].load(std::memory_order_acquire) == epoch) {
        ++arrived;
        progressed = true;
      }
    } else {
      if (issued < nchunks && (!have_mine || mine[issued].load(std::memory_order_acquire) == epoch)) {
        const int64_t off = issued * chunk_bytes;
        const int64_t n = std::min(chunk_bytes, total_bytes - off);
        const int64_t n1 = s2 ? std::min(n, ((n / 2) + 255) / 256 * 256) : n;
        uint8_t* d = static_cast<uint8_t*>(dst_next) + off;
        const uint8_t* sp = static_cast<const uint8_t*>(src) + off;
        cudaError_t e = cudaMemcpyAsync(d, sp, (size_t)n1, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(chunk to the next rank)");
        if (s2 && n > n1) {
          cudaEvent_t half = t_events[nchunks + issued];
          if ((e = cudaMemcpyAsync(d + n1, sp + n1, (size_t)(n - n1), cudaMemcpyDeviceToDevice, s2)) != cudaSuccess)
            return cuda_fail(e, "cudaMemcpyAsync(second half of a chunk)");
          if ((e = cudaEventRecord(half, s2)) != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
          if ((e = cudaStreamWaitEvent(s, half, 0)) != cudaSuccess) return cuda_fail(e, "cudaStreamWaitEvent");
        }
        // The next rank's device flag, written over NVLink after the chunk.
        CUresult r = g_write_value(reinterpret_cast<CUstream>(s), reinterpret_cast<CUdeviceptr>(ready_next + issued),
                                   epoch, 0);
        if (r != CUDA_SUCCESS)
          return fail(KEBAB_ECUDA, "cuStreamWriteValue32 (peer flag) failed with CUresult " + std::to_string(r));
        if ((e = cudaEventRecord(t_events[issued], s)) != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
        ++issued;
        progressed = true;
      }
      while (published < issued) {
        cudaError_t e = cudaEventQuery(t_events[published]);
        if (e == cudaErrorNotReady) break;
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventQuery(chunk copy)");
        next[published].store(epoch, std::memory_order_release);
        ++published;
        progressed = true;
      }
    }
    if (progressed) {
      deadline = std::chrono::steady_clock::now() + std::chrono::microseconds(timeout_us);
    } else {
      if (std::chrono::steady_clock::now() > deadline)
        return fail(KEBAB_ETIMEOUT, "kebab_chain_push: timed out with " + std::to_string(issued) + " of " +
                                        std::to_string(nchunks) + " chunks pushed, " + std::to_string(published) +
                                        " landed, " + std::to_string(arrived) + " received");
      std::this_thread::yield();
    }
  }
  return KEBAB_OK;
}

}  // extern "C"
