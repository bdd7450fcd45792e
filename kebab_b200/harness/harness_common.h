// Shared pieces of the C++ harness (bench_gemm, runonce_gemm): host matrix
// initialisation, device buffers, event timing, the cuBLAS comparator, result
// checking and CSV output.
#pragma once

#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <random>
#include <sstream>
#include <string>
#include <utility>
#include <vector>

#include "kebab/kebab.h"

#define CHECK_CUDA(x)                                                                                    \
  do {                                                                                                   \
    cudaError_t e_ = (x);                                                                                \
    if (e_ != cudaSuccess) {                                                                             \
      std::fprintf(stderr, "CUDA error %s at %s:%d: %s\n", cudaGetErrorName(e_), __FILE__, __LINE__,     \
                   cudaGetErrorString(e_));                                                              \
      std::exit(1);                                                                                      \
    }                                                                                                    \
  } while (0)
#define CHECK_CUBLAS(x)                                                                 \
  do {                                                                                  \
    cublasStatus_t s_ = (x);                                                            \
    if (s_ != CUBLAS_STATUS_SUCCESS) {                                                  \
      std::fprintf(stderr, "cuBLAS error %d at %s:%d\n", (int)s_, __FILE__, __LINE__);  \
      std::exit(1);                                                                     \
    }                                                                                   \
  } while (0)

namespace kebab {
namespace harness {

template <typename T>
struct TypeInfo;
template <>
struct TypeInfo<__half> {
  static constexpr const char* name = "float16";
  static constexpr kebab_dtype dtype = KEBAB_F16;
  static constexpr cudaDataType_t cuda = CUDA_R_16F;
  static constexpr double rel_fro_tol = 1e-3;
  static float to_f(__half v) { return __half2float(v); }
  static __half from_f(float v) { return __float2half(v); }
};
template <>
struct TypeInfo<__nv_bfloat16> {
  static constexpr const char* name = "bfloat16";
  static constexpr kebab_dtype dtype = KEBAB_BF16;
  static constexpr cudaDataType_t cuda = CUDA_R_16BF;
  // Two independently rounded BF16 results differ by ~2^-8 relative.
  static constexpr double rel_fro_tol = 4e-3;
  static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __nv_bfloat16 from_f(float v) { return __float2bfloat16(v); }
};

inline std::string upper(std::string s) {
  std::transform(s.begin(), s.end(), s.begin(), [](unsigned char c) { return (char)std::toupper(c); });
  return s;
}
inline std::string sci(double v) {
  std::ostringstream o;
  o << std::scientific << std::setprecision(2) << v;
  return o.str();
}

// Initialisation modes of the reference (kebab/include/kebab/utils/
// matrix_init.h:20-113): ONE, RAND (uniform_real_distribution<float>(-1, 1)
// over the caller's mt19937, in storage order), RANGE (storage index), ROW,
// COL (logical row / column index at the storage position of `fmt`).
enum class InitMode { ONE, RAND, RANGE, ROW, COL };

inline InitMode parse_init(const std::string& s) {
  if (s == "one") return InitMode::ONE;
  if (s == "range") return InitMode::RANGE;
  if (s == "row") return InitMode::ROW;
  if (s == "col") return InitMode::COL;
  return InitMode::RAND;
}
inline std::pair<InitMode, InitMode> parse_binary_init(const std::string& m) {
  size_t d = m.find('-');
  if (d == std::string::npos) return {parse_init(m), parse_init(m)};
  return {parse_init(m.substr(0, d)), parse_init(m.substr(d + 1))};
}

template <typename T>
void init_matrix(T* data, long long rows, long long cols, InitMode mode, std::mt19937& gen, char fmt) {
  const long long n = rows * cols;
  switch (mode) {
    case InitMode::ONE:
      for (long long i = 0; i < n; ++i) data[i] = TypeInfo<T>::from_f(1.0f);
      break;
    case InitMode::RAND: {
      std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
      for (long long i = 0; i < n; ++i) data[i] = TypeInfo<T>::from_f(dist(gen));
      break;
    }
    case InitMode::RANGE:
      for (long long i = 0; i < n; ++i) data[i] = TypeInfo<T>::from_f((float)i);
      break;
    case InitMode::ROW:
    case InitMode::COL:
      for (long long i = 0; i < rows; ++i)
        for (long long j = 0; j < cols; ++j) {
          long long idx = (fmt == 'R') ? i * cols + j : j * rows + i;
          data[idx] = TypeInfo<T>::from_f((float)(mode == InitMode::ROW ? i : j));
        }
      break;
  }
}

template <typename T>
struct DeviceBuffer {
  T* p = nullptr;
  long long n = 0;
  explicit DeviceBuffer(long long count) : n(count) { CHECK_CUDA(cudaMalloc(&p, sizeof(T) * (size_t)n)); }
  ~DeviceBuffer() { cudaFree(p); }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  void upload(const std::vector<T>& h) { CHECK_CUDA(cudaMemcpy(p, h.data(), sizeof(T) * h.size(), cudaMemcpyHostToDevice)); }
  std::vector<T> download() const {
    std::vector<T> h((size_t)n);
    CHECK_CUDA(cudaMemcpy(h.data(), p, sizeof(T) * (size_t)n, cudaMemcpyDeviceToHost));
    return h;
  }
};

// Warm-up launches, then `runs` launches between one event pair; returns the
// mean milliseconds per launch (the reference's measureLatency).
struct Timer {
  int warmup, runs;
  Timer(int w, int r) : warmup(w), runs(std::max(1, r)) {}
  template <class F>
  float measure(F&& f) {
    for (int i = 0; i < warmup; ++i) f();
    CHECK_CUDA(cudaDeviceSynchronize());
    cudaEvent_t a, b;
    CHECK_CUDA(cudaEventCreate(&a));
    CHECK_CUDA(cudaEventCreate(&b));
    CHECK_CUDA(cudaEventRecord(a));
    for (int i = 0; i < runs; ++i) f();
    CHECK_CUDA(cudaEventRecord(b));
    CHECK_CUDA(cudaEventSynchronize(b));
    float ms = 0.f;
    CHECK_CUDA(cudaEventElapsedTime(&ms, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return ms / runs;
  }
};

// cuBLAS with the reference's RC/RR mapping (getCublasGemmConfig,
// kebab/include/kebab/utils/cublas_reference.h:36-120): C column-major, ldC = M.
template <typename T>
void cublas_gemm(cublasHandle_t h, char lhs, char rhs, const T* A, const T* B, T* C, long long M, long long N,
                 long long K) {
  const float one = 1.0f, zero = 0.0f;
  cublasOperation_t opA = (lhs == 'R') ? CUBLAS_OP_T : CUBLAS_OP_N;
  cublasOperation_t opB = (rhs == 'R') ? CUBLAS_OP_T : CUBLAS_OP_N;
  long long lda = (lhs == 'R') ? K : M;
  long long ldb = (rhs == 'R') ? N : K;
  CHECK_CUBLAS(cublasGemmEx(h, opA, opB, (int)M, (int)N, (int)K, &one, A, TypeInfo<T>::cuda, (int)lda, B,
                            TypeInfo<T>::cuda, (int)ldb, &zero, C, TypeInfo<T>::cuda, (int)M, CUBLAS_COMPUTE_32F,
                            CUBLAS_GEMM_DEFAULT));
}

// The reference's own half comparator (cublas_reference.h:136): cublasHgemm,
// FP16 accumulation. Reported beside the FP32-accumulate one above, which is
// the fair comparator for this library's FP32-accumulate kernels.
inline void cublas_hgemm(cublasHandle_t h, char lhs, char rhs, const __half* A, const __half* B, __half* C,
                         long long M, long long N, long long K) {
  const __half one = __float2half(1.0f), zero = __float2half(0.0f);
  cublasOperation_t opA = (lhs == 'R') ? CUBLAS_OP_T : CUBLAS_OP_N;
  cublasOperation_t opB = (rhs == 'R') ? CUBLAS_OP_T : CUBLAS_OP_N;
  long long lda = (lhs == 'R') ? K : M;
  long long ldb = (rhs == 'R') ? N : K;
  CHECK_CUBLAS(cublasHgemm(h, opA, opB, (int)M, (int)N, (int)K, &one, A, (int)lda, B, (int)ldb, &zero, C, (int)M));
}

struct Check {
  bool ok;
  double rel_fro, worst;
};

// Relative Frobenius distance <= rel_tol and |d - r| <= 1e-2 (1 + |r|) per element.
template <typename T>
Check compare(const std::vector<T>& dev, const std::vector<T>& ref, double rel_tol) {
  double num = 0, den = 0, worst = 0;
  bool finite = true;
  for (size_t i = 0; i < dev.size(); ++i) {
    const double d = TypeInfo<T>::to_f(dev[i]), r = TypeInfo<T>::to_f(ref[i]);
    if (!std::isfinite(d)) finite = false;
    num += (d - r) * (d - r);
    den += r * r;
    worst = std::max(worst, std::fabs(d - r) / (1e-2 * (1.0 + std::fabs(r))));
  }
  const double rel = den > 0 ? std::sqrt(num / den) : std::sqrt(num);
  return {finite && rel <= rel_tol && worst <= 1.0, rel, worst};
}

// The reference's CSV columns (kebab/lib/benchmark/benchmark_runner.cpp:90-106).
class CsvWriter {
 public:
  explicit CsvWriter(const std::string& path) : f_(path, std::ios::out | std::ios::trunc) {
    if (f_) f_ << "Operator,Variant,BatchSize,Latency(ms),Throughput(GFLOPS),Speedup\n";
  }
  bool ok() const { return (bool)f_; }
  void row(const std::string& op, const std::string& variant, long long size, double ms, double gflops,
           double speedup) {
    f_ << op << "," << variant << "," << size << "," << std::fixed << std::setprecision(6) << ms << ","
       << std::setprecision(2) << gflops << "," << std::setprecision(3) << speedup << "\n";
    f_.flush();
  }

 private:
  std::ofstream f_;
};

// gpu_id >= device count falls back to GPU 0; a negative id keeps the current
// device (the reference's behaviour, bench_gemm.cu:360-376).
inline void select_gpu(int gpu_id) {
  int count = 0;
  CHECK_CUDA(cudaGetDeviceCount(&count));
  if (gpu_id >= 0 && gpu_id < count) {
    CHECK_CUDA(cudaSetDevice(gpu_id));
  } else if (gpu_id >= count) {
    std::cerr << "Warning: GPU " << gpu_id << " not available (" << count << " GPUs); using GPU 0" << std::endl;
    CHECK_CUDA(cudaSetDevice(0));
  }
}

}  // namespace harness
}  // namespace kebab
