// Internal host-side declarations shared by the translation units of
// libkebab_b200.so (not part of the public interface in include/).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "kebab/kebab.h"
#include "ptx.cuh"

namespace kb {

// Thread-local last-error message behind kebab_last_error().
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

// Per-device runtime facts, queried once per device.
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  uint32_t* status = nullptr;  // device address of the status word
};
int device_info(DeviceInfo** out);  // for the current device

// Wait context for kernels launched now (status word + current timeout).
int wait_ctx(WaitCtx* out);

// Whether launches that support it use programmatic dependent launch (their
// prologue overlaps the previous kernel on the stream). On unless the
// environment sets KEBAB_PDL=0.
bool pdl_enabled();

// 2D tensor map over a row-major [rows][cols] array of 2-byte elements
// (cols contiguous, row pitch `ld` elements), box {box_cols, box_rows}.
// swizzle128: 128-byte swizzle (box_cols * 2 must be 128).
int make_tmap_2d(CUtensorMap* out, const void* base, int dtype, uint64_t rows, uint64_t cols, uint64_t ld,
                 uint32_t box_rows, uint32_t box_cols, bool swizzle128);
// Same with the swizzle given in bytes: 0 (none), 32, 64 or 128.
int make_tmap_2d_sw(CUtensorMap* out, const void* base, int dtype, uint64_t rows, uint64_t cols, uint64_t ld,
                    uint32_t box_rows, uint32_t box_cols, int swizzle_bytes);

// Stream-K workspace of the calling (device, stream): `ws_bytes` of FP32
// partials and `flags` uint32 flags (zeroed once, when allocated), plus the
// epoch this launch must write into the flags (one more than the last).
// Allocated on first use and grown as needed; freed by kebab_shutdown().
int sk_workspace(cudaStream_t stream, size_t ws_bytes, size_t flags, float** ws, uint32_t** flag_ptr,
                 uint32_t* epoch);

// Problem description passed to every launcher.
struct GemmProblem {
  int dtype;  // KEBAB_F16 / KEBAB_BF16
  const void* A;
  const void* B;
  void* C;
  int64_t M, N, K;
  char lhs, rhs;  // 'R'/'C' storage of A and B
  bool c_row = false;  // C row-major (ldC = N) instead of column-major (ldC = M)
  cudaStream_t stream;
  // Gated B (persistent tcgen05 rungs 104, 105, 107 only): B's columns arrive
  // in chunks of b_chunk_cols while the GEMM runs; chunk j is readable once
  // the device flag b_ready[j] equals b_epoch (see UmmaArgs).
  const uint32_t* b_ready = nullptr;
  int64_t b_chunk_cols = 0;
  uint32_t b_epoch = 0;
};

// Launchers of the ladder rungs (return KEBAB_* status).
int launch_v1_simt(const GemmProblem& p);
int launch_v101_tma_mmasync(const GemmProblem& p);
int launch_v102_umma(const GemmProblem& p);
int launch_v103_ws(const GemmProblem& p);
int launch_v104_persistent(const GemmProblem& p);
int launch_v105_pair(const GemmProblem& p);
int launch_v106_skinny(const GemmProblem& p);
int launch_v107_pair_wide(const GemmProblem& p);
int launch_v108_streamk(const GemmProblem& p);
int launch_v109_pair_streamk(const GemmProblem& p);
int launch_v110_persistent_n128(const GemmProblem& p);
int launch_v111_persistent_n64(const GemmProblem& p);
int launch_v112_pair_384(const GemmProblem& p);
// K-blocks per ring stage: KEBAB_KPS=1 or 2 (read per call), else `dflt`.
int kps_env(int dflt);
int launch_v106_skinny_splits(const GemmProblem& p, int splits);  // splits <= 0: heuristic

// Clock probe armed by kebab_clock_probe() on this host thread for the next
// tcgen05 GEMM launch: returns the buffer (and disarms it) when it holds at
// least `ctas` CTAs' records, else null.
unsigned long long* take_clock_probe(int ctas);

// Forgets the no-alloc GEMM's per-device set-up (kebab_shutdown()).
void noalloc_reset();

// Validation shared by the TMA-based rungs: 16-byte aligned pointers and
// 16-byte row pitches of A, B and C in their storage layouts (RC: K % 8 and
// M % 8; a column-major A needs M % 8, a row-major B or C needs N % 8).
int check_tma_shapes(const GemmProblem& p);

}  // namespace kb
