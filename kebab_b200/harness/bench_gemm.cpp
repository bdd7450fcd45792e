// bench_gemm — the config.yaml-driven GEMM benchmark of the reference
// (kebab/lib/benchmark/bench_gemm.cu:87-435), over the B200 ladder.
//
// For every precision, problem (operators.gemm.matrix_sizes as squares, plus
// operators.gemm.shapes) and mode it: initialises A and B on the host from one
// mt19937(seed) stream (the reference's initializeMatrix modes), times cuBLAS
// (cublasGemmEx, FP32 compute — a reported comparator), then for every
// implementation and version verifies kebab_gemm against cuBLAS and times it
// (warm-up runs, then measurement runs between one CUDA event pair, like
// BenchmarkRunner::measureLatency, kebab/include/kebab/utils/benchmark.h:80-99),
// prints a table and writes bench_results/gemm_results_<type>_<impls>.csv with
// the reference's columns (Operator,Variant,BatchSize,Latency(ms),
// Throughput(GFLOPS),Speedup), so the reference's report / autotune scripts
// read it unchanged.
//
// Usage: bench_gemm [--config config.yaml] [--out-dir bench_results] [--dump-config]
#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <iomanip>
#include <iostream>
#include <random>
#include <sstream>
#include <string>
#include <sys/stat.h>
#include <type_traits>
#include <vector>

#include "config_parser.h"
#include "harness_common.h"
#include "kebab/kebab.h"

using kebab::config::ConfigParser;
using namespace kebab::harness;

namespace {

void dump_config(const ConfigParser& c) {
  auto ivec = [](const std::vector<int>& v) {
    std::string s = "[";
    for (size_t i = 0; i < v.size(); ++i) s += (i ? ", " : "") + std::to_string(v[i]);
    return s + "]";
  };
  auto svec = [](const std::vector<std::string>& v) {
    std::string s = "[";
    for (size_t i = 0; i < v.size(); ++i) s += std::string(i ? ", " : "") + "\"" + v[i] + "\"";
    return s + "]";
  };
  std::string shapes = "[";
  auto sh = c.getOperatorShapes("gemm");
  for (size_t i = 0; i < sh.size(); ++i)
    shapes += std::string(i ? ", " : "") + "[" + std::to_string(sh[i][0]) + ", " + std::to_string(sh[i][1]) + ", " +
              std::to_string(sh[i][2]) + "]";
  shapes += "]";
  std::cout << "{\"warmup_runs\": " << c.getWarmupRuns() << ", \"measurement_runs\": " << c.getMeasurementRuns()
            << ", \"impls\": " << svec(c.getOperatorImpls("gemm")) << ", \"versions\": "
            << ivec(c.getOperatorVersions("gemm")) << ", \"matrix_sizes\": " << ivec(c.getOperatorMatrixSizes("gemm"))
            << ", \"modes\": " << svec(c.getOperatorModes("gemm")) << ", \"precisions\": "
            << svec(c.getOperatorPrecisions("gemm")) << ", \"init_method\": \"" << c.getOperatorInitMethod("gemm")
            << "\", \"gpu_id\": " << c.getOperatorGpuId("gemm") << ", \"verbose\": "
            << (c.getOperatorVerbose("gemm") ? "true" : "false") << ", \"seed\": " << c.getOperatorSeed("gemm")
            << ", \"shapes\": " << shapes << ", \"enabled\": " << (c.isOperatorEnabled("gemm") ? "true" : "false")
            << ", \"build_mode\": \"" << c.getBuildMode() << "\"}" << std::endl;
}

template <typename T>
int bench_precision(const ConfigParser& cfg, const std::string& out_dir) {
  const std::string type_name = TypeInfo<T>::name;
  const auto impls = cfg.getOperatorImpls("gemm");
  const auto versions = cfg.getOperatorVersions("gemm");
  const auto modes = cfg.getOperatorModes("gemm");
  const auto init = parse_binary_init(cfg.getOperatorInitMethod("gemm"));
  const int warmup = cfg.getWarmupRuns(), runs = cfg.getMeasurementRuns();
  std::vector<std::vector<long long>> problems;
  for (int s : cfg.getOperatorMatrixSizes("gemm")) problems.push_back({s, s, s});
  for (auto& s : cfg.getOperatorShapes("gemm")) problems.push_back(s);

  std::string impl_str;
  for (size_t i = 0; i < impls.size(); ++i) impl_str += (i ? "_" : "") + impls[i];
  mkdir(out_dir.c_str(), 0755);
  const std::string csv_path = out_dir + "/gemm_results_" + type_name + "_" + impl_str + ".csv";
  CsvWriter csv(csv_path);
  if (!csv.ok()) {
    std::cerr << "ERROR: cannot create " << csv_path << std::endl;
    return 1;
  }
  std::mt19937 gen(cfg.getOperatorSeed("gemm"));
  cublasHandle_t handle;
  CHECK_CUBLAS(cublasCreate(&handle));
  int failures = 0;

  std::cout << "\n== GEMM benchmark: " << type_name << " | versions:";
  for (int v : versions) std::cout << " v" << v << "(" << kebab_version_name(v) << ")";
  std::cout << std::endl;

  for (const auto& pr : problems) {
    const long long M = pr[0], N = pr[1], K = pr[2];
    for (const auto& mode_in : modes) {
      std::string mode = upper(mode_in);
      const char lhs = mode.size() > 0 ? mode[0] : 'R', rhs = mode.size() > 1 ? mode[1] : 'R';
      std::vector<T> hA((size_t)(M * K)), hB((size_t)(K * N));
      init_matrix(hA.data(), M, K, init.first, gen, lhs);
      init_matrix(hB.data(), K, N, init.second, gen, rhs);
      DeviceBuffer<T> dA(M * K), dB(K * N), dC(M * N), dRef(M * N);
      dA.upload(hA);
      dB.upload(hB);
      const double flops = 2.0 * (double)M * (double)N * (double)K;
      Timer timer(warmup, runs);
      const float cublas_ms = timer.measure([&] { cublas_gemm<T>(handle, lhs, rhs, dA.p, dB.p, dRef.p, M, N, K); });
      const double cublas_tflops = flops / (cublas_ms * 1e-3) / 1e12;
      std::vector<T> ref = dRef.download();
      std::cout << "  " << M << "x" << N << "x" << K << " " << mode << "  cuBLAS " << std::fixed
                << std::setprecision(1) << cublas_tflops << " TFLOP/s (FP32 accumulate)";
      if constexpr (std::is_same<T, __half>::value) {
        DeviceBuffer<T> dH(M * N);
        const float h_ms = timer.measure([&] { cublas_hgemm(handle, lhs, rhs, dA.p, dB.p, dH.p, M, N, K); });
        std::cout << ", cublasHgemm " << flops / (h_ms * 1e-3) / 1e12 << " TFLOP/s (FP16 accumulate, the reference's)";
      }
      std::cout << std::endl;
      for (const auto& impl : impls) {
        if (impl != "cuda") {
          std::cout << "    impl " << impl << ": skipped (only the cuda ladder is built for sm_100a)" << std::endl;
          continue;
        }
        for (int v : versions) {
          CHECK_CUDA(cudaMemset(dC.p, 0, sizeof(T) * (size_t)(M * N)));
          int rc = kebab_gemm(TypeInfo<T>::dtype, dA.p, dB.p, dC.p, M, N, K, mode.c_str(), v, nullptr);
          if (rc == KEBAB_OK) rc = kebab_device_status(nullptr, nullptr, 1);
          std::string status;
          double tflops = 0.0, ms = 0.0;
          if (rc != KEBAB_OK) {
            status = std::string("ERROR ") + kebab_last_error();
          } else {
            Check chk = compare(dC.download(), ref, TypeInfo<T>::rel_fro_tol);
            if (!chk.ok) {
              status = "FAIL (rel_fro " + sci(chk.rel_fro) + ", worst " + sci(chk.worst) + ")";
              ++failures;
            } else {
              ms = timer.measure([&] { kebab_gemm(TypeInfo<T>::dtype, dA.p, dB.p, dC.p, M, N, K, mode.c_str(), v,
                                                  nullptr); });
              tflops = flops / (ms * 1e-3) / 1e12;
              status = "PASS";
              csv.row("GEMM", "cuda_v" + std::to_string(v) + "_" + kebab_version_name(v), M,
                      ms, tflops * 1000.0, cublas_tflops > 0 ? tflops / cublas_tflops : 0.0);
            }
          }
          std::cout << "    v" << std::setw(3) << v << " " << std::left << std::setw(48) << kebab_version_name(v)
                    << std::right << std::setw(9) << std::setprecision(1) << tflops << " TFLOP/s ("
                    << std::setw(5) << std::setprecision(1) << (cublas_tflops > 0 ? 100.0 * tflops / cublas_tflops : 0)
                    << "% of cuBLAS)  " << status << std::endl;
        }
      }
    }
  }
  cublasDestroy(handle);
  std::cout << "Results saved to: " << csv_path << std::endl;
  return failures ? 2 : 0;
}

}  // namespace

int main(int argc, char** argv) {
  std::string config_path = "config.yaml", out_dir = "bench_results";
  bool dump = false;
  for (int i = 1; i < argc; ++i) {
    if (!std::strcmp(argv[i], "--config") && i + 1 < argc) config_path = argv[++i];
    else if (!std::strcmp(argv[i], "--out-dir") && i + 1 < argc) out_dir = argv[++i];
    else if (!std::strcmp(argv[i], "--dump-config")) dump = true;
    else {
      std::cerr << "usage: bench_gemm [--config config.yaml] [--out-dir bench_results] [--dump-config]" << std::endl;
      return 1;
    }
  }
  try {
    ConfigParser cfg(config_path);
    if (dump) {
      dump_config(cfg);
      return 0;
    }
    if (!cfg.isOperatorEnabled("gemm")) {
      std::cout << "operators.gemm.enabled is false; nothing to do" << std::endl;
      return 0;
    }
    select_gpu(cfg.getOperatorGpuId("gemm"));
    int rc = 0;
    for (const auto& p : cfg.getOperatorPrecisions("gemm")) {
      if (p == "float16" || p == "half") rc |= bench_precision<__half>(cfg, out_dir);
      else if (p == "bfloat16" || p == "bf16") rc |= bench_precision<__nv_bfloat16>(cfg, out_dir);
      else if (p == "float32" || p == "float")
        std::cout << "\nSkipping float32: not implemented (use half or bfloat16), as in the reference" << std::endl;
      else std::cout << "\nSkipping unknown precision " << p << std::endl;
    }
    return rc;
  } catch (const std::exception& e) {
    std::cerr << "ERROR: " << e.what() << std::endl;
    return 1;
  }
}
