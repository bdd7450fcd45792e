// Compiles the reference's OWN CPU GEMM and matrix initialiser (header-only,
// kebab/include/kebab/utils/reference_gemm.h and matrix_init.h, included
// unmodified from the reference tree) into oracle/_ref/libkebab_ref.so, so
// that tests can pin the restatement in kebab_oracle.cpp against them and
// bench.py can time the reference routine itself. Test infrastructure only.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <cstring>
#include <random>

#include "kebab/utils/matrix_init.h"
#include "kebab/utils/reference_gemm.h"

extern "C" {

// referenceGemmCpp<float>(A, B, C, M, N, K, 'R', 'C'): the reference CPU GEMM
// in RC mode (A row-major, B column-major, C column-major).
void kbr_gemm_f32(const float* A, const float* B, float* C, int M, int N, int K) {
  kebab::utils::referenceGemmCpp<float>(A, B, C, M, N, K, 'R', 'C');
}

// referenceGemmCpp<__half>: FP16 accumulation (exported for the record).
void kbr_gemm_f16acc(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K) {
  kebab::utils::referenceGemmCpp<__half>(reinterpret_cast<const __half*>(A), reinterpret_cast<const __half*>(B),
                                         reinterpret_cast<__half*>(C), M, N, K, 'R', 'C');
}

// initializeMatrix RAND for A (rowsA x colsA, 'R') then B (rowsB x colsB,
// 'C') from one mt19937(seed), as the reference benchmark does.
void kbr_init_rand_f16(uint16_t* A, int rowsA, int colsA, uint16_t* B, int rowsB, int colsB, uint32_t seed) {
  std::mt19937 gen(seed);
  kebab::utils::initializeMatrix<__half>(reinterpret_cast<__half*>(A), rowsA, colsA, kebab::utils::InitMode::RAND,
                                         gen, 'R');
  kebab::utils::initializeMatrix<__half>(reinterpret_cast<__half*>(B), rowsB, colsB, kebab::utils::InitMode::RAND,
                                         gen, 'C');
}

void kbr_init_rand_bf16(uint16_t* A, int rowsA, int colsA, uint16_t* B, int rowsB, int colsB, uint32_t seed) {
  std::mt19937 gen(seed);
  kebab::utils::initializeMatrix<__nv_bfloat16>(reinterpret_cast<__nv_bfloat16*>(A), rowsA, colsA,
                                                kebab::utils::InitMode::RAND, gen, 'R');
  kebab::utils::initializeMatrix<__nv_bfloat16>(reinterpret_cast<__nv_bfloat16*>(B), rowsB, colsB,
                                                kebab::utils::InitMode::RAND, gen, 'C');
}

uint16_t kbr_float2half(float f) {
  __half h = __float2half(f);
  uint16_t r;
  std::memcpy(&r, &h, 2);
  return r;
}

uint16_t kbr_float2bf16(float f) {
  __nv_bfloat16 h = __float2bfloat16(f);
  uint16_t r;
  std::memcpy(&r, &h, 2);
  return r;
}

}  // extern "C"
