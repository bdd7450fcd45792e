// C++ mirror of the reference operator interface
// (kebab/include/kebab/cuda/cuda_gemm.h:10-33 and the per-version launchers
// declared at :43-257), implemented over the B200 ladder by libkebab_b200.so.
// Callers written against the reference compile unchanged: the same
// baseline::gemm overloads with the same defaults, and the same
// gemm_cuda_version_feature_name. Like the reference these print an error
// and return; the status-returning C ABI is in kebab/kebab.h.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kebab/kebab.h"

namespace baseline {

// Replaces gemm_cuda_version_feature_name (kebab/lib/cuda/cuda_gemm.cu:81-106).
const char* gemm_cuda_version_feature_name(int version);

// Replace the three overloads at kebab/lib/cuda/cuda_gemm.cu:112, :246, :259.
// A: M x K, B: K x N, C: M x N column-major; opmode "RC" (A row-major, B
// column-major). version: a B200 rung (1, 101..106, 120) or a reference id.
void gemm(const float* A, const float* B, float* C, int M, int N, int K, const char* opmode = "RC",
          int version = 1, cudaStream_t stream = 0);
void gemm(const __half* A, const __half* B, __half* C, int M, int N, int K, const char* opmode = "RC",
          int version = 1, cudaStream_t stream = 0);
void gemm(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C, int M, int N, int K,
          const char* opmode = "RC", int version = 1, cudaStream_t stream = 0);

// Per-rung launchers, same argument convention as the reference's
// gemm_vN_<feature>_fp16(A, B, C, M, N, K, lhs_format, rhs_format, stream).
#define KEBAB_DECLARE_RUNG(NAME)                                                                          \
  void NAME##_fp16(const __half* A, const __half* B, __half* C, int M, int N, int K, char lhs_format,    \
                   char rhs_format, cudaStream_t stream);                                                \
  void NAME##_bf16(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C, int M, int N, int K, \
                   char lhs_format, char rhs_format, cudaStream_t stream);
KEBAB_DECLARE_RUNG(gemm_v1_simt_warptiling)                                   // CUDA cores (reference v1)
KEBAB_DECLARE_RUNG(gemm_v101_tma_mmasync)                                     // TMA staging + mma.sync
KEBAB_DECLARE_RUNG(gemm_v102_tma_umma_tmem)                                   // + tcgen05.mma, TMEM
KEBAB_DECLARE_RUNG(gemm_v103_tma_umma_tmem_warpspecialized)                   // + producer/MMA/epilogue warps
KEBAB_DECLARE_RUNG(gemm_v104_tma_umma_tmem_warpspecialized_persistent)        // + persistent scheduler
KEBAB_DECLARE_RUNG(gemm_v105_tma_umma_tmem_warpspecialized_persistent_2cta)   // + cta_group::2 pairs
KEBAB_DECLARE_RUNG(gemm_v106_tma_umma_tmem_swapab_splitk_cluster_skinny)      // M <= 256: swap-AB, cluster split-K
KEBAB_DECLARE_RUNG(gemm_v107_tma_umma_tmem_warpspecialized_persistent_2cta_256x512)  // pairs, 256 x 512 tiles
KEBAB_DECLARE_RUNG(gemm_v108_tma_umma_tmem_warpspecialized_persistent_streamk)  // v104 + stream-K
KEBAB_DECLARE_RUNG(gemm_v109_tma_umma_tmem_warpspecialized_persistent_2cta_streamk)  // v105 + stream-K
KEBAB_DECLARE_RUNG(gemm_v110_tma_umma_tmem_warpspecialized_persistent_128x128)  // v104, 128 x 128 tiles
KEBAB_DECLARE_RUNG(gemm_v111_tma_umma_tmem_warpspecialized_persistent_128x64)   // v104, 128 x 64 tiles
KEBAB_DECLARE_RUNG(gemm_v112_tma_umma_tmem_warpspecialized_persistent_2cta_256x384)  // pairs, 256 x 384 tiles
KEBAB_DECLARE_RUNG(gemm_v141_tma_umma_tmem_warpspecialized_persistent_2cta_rowmajor_c)  // v105, row-major C
#undef KEBAB_DECLARE_RUNG

// The reference's own launcher names (kebab/include/kebab/cuda/cuda_gemm.h:43-257,
// every non-template fp16 / bf16 launcher except the v8..v12 names, whose
// feature strings name the cluster load this build never issues; those ids
// still reach their rung through baseline::gemm; the gemm_v2 template is
// left out too),
// each forwarding to the B200 rung its version id maps to (kebab_version_name()
// tells which), with the same (A, B, C, M, N, K, lhs_format, rhs_format,
// stream) arguments.
#define KEBAB_REFERENCE_ALIAS_F16(NAME, ID)                                                              \
  void NAME(const __half* A, const __half* B, __half* C, int M, int N, int K, char lhs_format,          \
            char rhs_format, cudaStream_t stream);
#define KEBAB_REFERENCE_ALIAS_BF16(NAME, ID)                                                             \
  void NAME(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C, int M, int N, int K,       \
            char lhs_format, char rhs_format, cudaStream_t stream);
#define KEBAB_REFERENCE_ALIASES \
  KEBAB_REFERENCE_ALIAS_BF16(gemm_v1_warptiling_bf16_baseline, 1) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v1_warptiling_fp16_baseline, 1) \
  KEBAB_REFERENCE_ALIAS_BF16(gemm_v3_wgmma_tma_warpgroup_bf16, 3) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v3_wgmma_tma_warpgroup_fp16, 3) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v4_wgmma_tma_warpgroup_warpspecialized_fp16, 4) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v5_wgmma_tma_warpgroup_warpspecialized_persistent_fp16, 5) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v6_wgmma_tma_warpgroup_warpspecialized_persistent_tilescheduler_fp16, 6) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v7_wgmma_tma_warpgroup_warpspecialized_persistent_tilescheduler_ptxbarrier_tma5d_fp16, 7) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v13_wgmma_tma_warpspecialized_persistent_tilescheduler_ptxbarrier_tma2d_fp16, 13) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v14_wgmma_tma_warpspecialized_persistent_ptxbarrier_tmastore_hilbert_stmatrix_padded_nocluster_fp16, 14) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v15_wgmma_tma_warpspecialized_ptxbarrier_tmastore_hilbert_stmatrix_padded_nocluster_nopersistent_fp16, 15) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v16_wgmma_tma_warpspecialized_persistent_ptxbarrier_tmastore_hilbert_stmatrix_padded_nocluster_linearschedule_fp16, 16) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v17_wgmma_tma_warpgroup_ptxbarrier_fp16, 17) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v18_wgmma_tma_warpgroup_warpspecialized_persistent_stmatrix_fp16, 18) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v19_wgmma_tma_warpgroup_warpspecialized_persistent_hilbert_fp16, 19) \
  KEBAB_REFERENCE_ALIAS_F16(gemm_v41_wgmma_tma_warpgroup_warpspecialized_fp16, 41)
KEBAB_REFERENCE_ALIASES
#undef KEBAB_REFERENCE_ALIAS_F16
#undef KEBAB_REFERENCE_ALIAS_BF16

}  // namespace baseline
