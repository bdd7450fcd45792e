// runonce_gemm — one launch of one rung, for Nsight Compute, then a check
// against cuBLAS: the role of the reference's runonce_gemm_cuda
// (kebab/lib/benchmark/runonce_gemm_cuda.cu:30-117). By default it takes the
// first size, mode, precision and version from the config, like the reference.
//
// Usage: runonce_gemm [--config config.yaml] [--version V] [--m M --n N --k K]
//                     [--mode RC] [--precision float16|bfloat16]
#include <cstring>
#include <iostream>
#include <random>

#include "config_parser.h"
#include "harness_common.h"

using kebab::config::ConfigParser;
using namespace kebab::harness;

template <typename T>
int run(long long M, long long N, long long K, const std::string& mode, int version, unsigned seed) {
  std::mt19937 gen(seed);
  const char lhs = mode.size() > 0 ? mode[0] : 'R', rhs = mode.size() > 1 ? mode[1] : 'R';
  std::vector<T> hA((size_t)(M * K)), hB((size_t)(K * N));
  init_matrix(hA.data(), M, K, InitMode::RAND, gen, lhs);
  init_matrix(hB.data(), K, N, InitMode::RAND, gen, rhs);
  DeviceBuffer<T> dA(M * K), dB(K * N), dC(M * N), dRef(M * N);
  dA.upload(hA);
  dB.upload(hB);
  int rc = kebab_gemm(TypeInfo<T>::dtype, dA.p, dB.p, dC.p, M, N, K, mode.c_str(), version, nullptr);
  if (rc == KEBAB_OK) rc = kebab_device_status(nullptr, nullptr, 1);
  if (rc != KEBAB_OK) {
    std::cerr << "kebab_gemm failed (" << rc << "): " << kebab_last_error() << std::endl;
    return 1;
  }
  cublasHandle_t h;
  CHECK_CUBLAS(cublasCreate(&h));
  cublas_gemm<T>(h, lhs, rhs, dA.p, dB.p, dRef.p, M, N, K);
  CHECK_CUDA(cudaDeviceSynchronize());
  cublasDestroy(h);
  Check c = compare(dC.download(), dRef.download(), TypeInfo<T>::rel_fro_tol);
  std::cout << "v" << version << " (" << kebab_version_name(version) << ") " << TypeInfo<T>::name << " " << M << "x"
            << N << "x" << K << " " << mode << ": " << (c.ok ? "PASS" : "FAIL") << " rel_fro=" << sci(c.rel_fro)
            << " worst=" << sci(c.worst) << std::endl;
  return c.ok ? 0 : 2;
}

int main(int argc, char** argv) {
  std::string config_path = "config.yaml", mode, precision;
  long long M = 0, N = 0, K = 0;
  int version = -1;
  for (int i = 1; i + 1 < argc; i += 2) {
    std::string a = argv[i];
    if (a == "--config") config_path = argv[i + 1];
    else if (a == "--version") version = std::atoi(argv[i + 1]);
    else if (a == "--m") M = std::atoll(argv[i + 1]);
    else if (a == "--n") N = std::atoll(argv[i + 1]);
    else if (a == "--k") K = std::atoll(argv[i + 1]);
    else if (a == "--mode") mode = argv[i + 1];
    else if (a == "--precision") precision = argv[i + 1];
    else {
      std::cerr << "unknown option " << a << std::endl;
      return 1;
    }
  }
  try {
    ConfigParser cfg(config_path);
    auto sizes = cfg.getOperatorMatrixSizes("gemm");
    long long s = sizes.empty() ? 1024 : sizes[0];
    if (!M) M = s;
    if (!N) N = s;
    if (!K) K = s;
    if (mode.empty()) mode = upper(cfg.getOperatorModes("gemm")[0]);
    if (precision.empty()) precision = cfg.getOperatorPrecisions("gemm")[0];
    if (version < 0) version = cfg.getOperatorVersion("gemm");
    select_gpu(cfg.getOperatorGpuId("gemm"));
    if (precision == "bfloat16" || precision == "bf16")
      return run<__nv_bfloat16>(M, N, K, mode, version, cfg.getOperatorSeed("gemm"));
    return run<__half>(M, N, K, mode, version, cfg.getOperatorSeed("gemm"));
  } catch (const std::exception& e) {
    std::cerr << "ERROR: " << e.what() << std::endl;
    return 1;
  }
}
