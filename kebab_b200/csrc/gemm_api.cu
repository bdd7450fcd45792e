// Operator surface: the C ABI (kebab_gemm & co.) and the C++ mirror of the
// reference's baseline:: interface, both dispatching over the B200 ladder.
//
// Reference behaviour kept (kebab/lib/cuda/cuda_gemm.cu):
//   - null pointers / non-positive dims are rejected (:115-122);
//   - opmode is upper-cased; lhs = opmode[0] or 'R', rhs = opmode[1] or 'C'
//     (:125-129);
//   - float inputs are "not implemented" (:246-253);
//   - unknown versions are rejected (:235-238).
// Differences: a status code is returned (the C++ overloads still print and
// return void, like the reference), indices are int64, and reference version
// ids map onto the B200 rung that carries the same idea.
#include <algorithm>
#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "internal.h"
#include "kebab/cuda/cuda_gemm.h"
#include "kebab/peer.h"

namespace kb {
namespace {

struct Rung {
  int id;
  const char* name;
  int (*launch)(const GemmProblem&);
};

const Rung kRungs[] = {
    {1, "simt_warptiling", launch_v1_simt},
    {101, "tma_mmasync", launch_v101_tma_mmasync},
    {102, "tma_umma_tmem", launch_v102_umma},
    {103, "tma_umma_tmem_warpspecialized", launch_v103_ws},
    {104, "tma_umma_tmem_warpspecialized_persistent", launch_v104_persistent},
    {105, "tma_umma_tmem_warpspecialized_persistent_2cta", launch_v105_pair},
    {106, "tma_umma_tmem_swapab_splitk_cluster_skinny", launch_v106_skinny},
    {107, "tma_umma_tmem_warpspecialized_persistent_2cta_256x512", launch_v107_pair_wide},
    {108, "tma_umma_tmem_warpspecialized_persistent_streamk", launch_v108_streamk},
    {109, "tma_umma_tmem_warpspecialized_persistent_2cta_streamk", launch_v109_pair_streamk},
    {110, "tma_umma_tmem_warpspecialized_persistent_128x128", launch_v110_persistent_n128},
    {111, "tma_umma_tmem_warpspecialized_persistent_128x64", launch_v111_persistent_n64},
    {112, "tma_umma_tmem_warpspecialized_persistent_2cta_256x384", launch_v112_pair_384},
    {141, "tma_umma_tmem_warpspecialized_persistent_2cta_rowmajor_c", launch_v105_pair},
};

const Rung* find_rung(int id) {
  for (const auto& r : kRungs)
    if (r.id == id) return &r;
  return nullptr;
}

// Reference version id -> B200 rung with the same idea (see the table in
// kebab_version_name's documentation).
int map_reference_id(int v) {
  switch (v) {
    case 2: case 3: case 17: return 102;             // TMA + one MMA stream per CTA
    case 4: case 15: return 103;                     // warp specialised, one tile per CTA
    case 5: case 6: case 7: case 13: case 14:
    case 16: case 18: case 19: return 104;           // persistent scheduler
    case 8: case 9: case 10: case 11: case 12: return 105;  // cluster pairs
    case 20: return 120;                             // decomposition heuristic
    case 41: return 141;                             // row-major C
    default: return v;
  }
}

// The role of the reference's v20 heuristic (cuda_gemm.cu:25-77): choose a
// decomposition from the tile count against the QUERIED SM count.
// KEBAB_V120_MODE = dp | persistent | pair | wide | streamk (pairs) | streamk1
// (1-CTA) | n128 | n64 | skinny | heuristic (default).
int choose_v120(int64_t M, int64_t N, int64_t K, int sm_count, bool rc_colc, bool allow_384) {
  const char* env = std::getenv("KEBAB_V120_MODE");
  if (env && *env) {
    std::string m(env);
    std::transform(m.begin(), m.end(), m.begin(), [](unsigned char c) { return (char)std::toupper(c); });
    if (m == "DP" || m == "DATAPARALLEL") return 103;
    if (m == "PERSISTENT") return 104;
    if (m == "PAIR" || m == "2CTA") return 105;
    if (m == "WIDE" || m == "PAIRWIDE") return 107;
    if (m == "PAIR384" || m == "FIT") return 112;
    if (m == "STREAMK" || m == "PAIRSTREAMK") return 109;
    if (m == "STREAMK1") return 108;
    if (m == "N128" || m == "NARROW") return 110;
    if (m == "N64") return 111;
    if ((m == "SKINNY" || m == "SPLITK") && rc_colc) return 106;
  }
  // Decode-like shapes: too few 128-row tiles to occupy the GPU, and enough
  // of B (N x K >= 4 Mi elements) that streaming it dominates: the swap-AB
  // split-K rung. Below that (256 x 1024 x 1024: 27 TFLOP/s on 106 against 67
  // on 111) the small-problem tiles below win.
  if (M <= 256 && rc_colc && N * K >= (int64_t)4 * 1024 * 1024) return 106;
  const int64_t pairs = sm_count / 2;
  const int64_t pair_tiles = ((M + 255) / 256) * ((N + 255) / 256);
  // Pair tiles halve B traffic per CTA; worth it once they fill the pairs.
  // Among the pair widths 256 (105), 512 (107, N a multiple of 512) and 384
  // (112, column-major B only) take the least cost = waves x tile width x a
  // per-FLOP factor: wider tiles stage fewer operand bytes per FLOP (lower
  // power, higher clock under the cap). Fitted factors from the measurements
  // below: 256 wide 1.05-1.11 (the upper end in power-capped loops), 384
  // 0.99-1.06, against 512 = 1. Measured (TFLOP/s, 105 / 107 / 112):
  // 4096^3 1326 / 1397 / 1251, 3072^3 1319 / 1363 / 1057, 3072 x 2048 x 2048
  // 913 / 896 / 1101, 2048 x 3072 x 4096 1063 / 1097 / 1269, 2560 x 8192 x
  // 4096 1349 / 1268 / 1411, 2048 x 28672 x 8192 (config 4a on 8 GPUs) 1272
  // / 1315 / 1296. The stream-K rungs (108, 109) are not chosen here:
  // measured against 105 they tie at 4096^3, lose at 3072 x 2048 x 2048 (828
  // vs 953) and at 2048 x 28672 x 8192 (1261 vs 1272).
  if (pair_tiles >= pairs) {
    auto cost = [&](int bn, double per_flop) {
      const int64_t t = ((M + 255) / 256) * ((N + bn - 1) / bn);
      return (double)((t + pairs - 1) / pairs) * bn * per_flop;
    };
    int best = 105;
    double c = cost(256, 1.08);
    if (N % 512 == 0 && cost(512, 1.0) <= c) best = 107, c = cost(512, 1.0);
    if (allow_384 && cost(384, 1.03) < 0.97 * c) best = 112;
    return best;
  }
  // Small problems: the widest 128-row tiles that still occupy the SMs.
  // 128 x 256 (v104) at 2048^3 and 4096 x 1024 x 1024; 128 x 128 (v110) at
  // 1280^3 .. 1536^3 and 2048 x 1024 x 4096; 128 x 64 (v111, latency-bound
  // sizes) up to 1024^3, where it beats cuBLAS below 1024^3.
  const int64_t tm = (M + 127) / 128;
  const int64_t t256 = tm * ((N + 255) / 256), t128 = tm * ((N + 127) / 128), t64 = tm * ((N + 63) / 64);
  if (t256 * 10 >= (int64_t)sm_count * 8) return 104;
  // Too few tiles and a deep K: split K over a cluster (rung 106 tiles M in
  // 256-row blocks and reduces through distributed shared memory):
  // 1024 x 1024 x 8192 672 vs 391 TFLOP/s, 2048 x 1024 x 4096 898 vs 666,
  // 1536 x 1536 x 3072 819 vs 682. At K = 1536 (1536^3: 533 vs 569) and
  // 1280 the 128 x 128 tiles still win.
  if (rc_colc && K >= 3072) return 106;
  if (t128 <= sm_count && t128 * 10 >= (int64_t)sm_count * 6) return 110;
  if (t64 <= sm_count) return 111;
  return 110;
}

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" {

const char* kebab_version_name(int version) {
  if (version == 120) return "decomposition_heuristic";
  const int id = map_reference_id(version);
  if (id == 120) return "decomposition_heuristic";
  const Rung* r = find_rung(id);
  return r ? r->name : "unknown";
}

int kebab_list_versions(int* out, int cap) {
  int n = 0;
  for (const auto& r : kRungs)
    if (out && n < cap) out[n++] = r.id; else if (!out) ++n;
  if (out && n < cap) out[n++] = 120;
  else if (!out) ++n;
  return n;
}

// allow_384: rung 112 may be chosen (column-major B, no 512-column chunking).
static int resolve(int version, int64_t M, int64_t N, int64_t K, bool rc_colc, bool allow_384 = true) {
  int id = map_reference_id(version);
  if (id == 120) {
    DeviceInfo* d = nullptr;
    int rc = device_info(&d);
    int sms = rc == KEBAB_OK ? d->sm_count : 148;
    id = choose_v120(M, N, K, sms, rc_colc, allow_384);
  }
  if (!find_rung(id)) {
    fail(KEBAB_EINVAL, "unsupported version " + std::to_string(version));
    return -KEBAB_EINVAL;
  }
  return id;
}

int kebab_resolve_version(int version, kebab_dtype dtype, int64_t M, int64_t N, int64_t K) {
  (void)dtype;
  return resolve(version, M, N, K, true);
}

int kebab_gemm(kebab_dtype dtype, const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
               const char* opmode, int version, kebab_stream_t stream) {
  if (!A || !B || !C) return fail(KEBAB_EINVAL, "null pointer passed to kebab_gemm");
  if (M <= 0 || N <= 0 || K <= 0)
    return fail(KEBAB_EINVAL, "invalid dimensions: M=" + std::to_string(M) + ", N=" + std::to_string(N) +
                                  ", K=" + std::to_string(K));
  if (dtype == KEBAB_F32) return fail(KEBAB_ENOTSUP, "float precision not implemented; use half or bfloat16");
  if (dtype != KEBAB_F16 && dtype != KEBAB_BF16) return fail(KEBAB_EINVAL, "unknown dtype");
  std::string mode(opmode ? opmode : "RC");
  std::transform(mode.begin(), mode.end(), mode.begin(), [](unsigned char c) { return (char)std::toupper(c); });
  const char lhs = mode.size() >= 1 ? mode[0] : 'R';
  const char rhs = mode.size() >= 2 ? mode[1] : 'C';
  const char cl = mode.size() >= 3 ? mode[2] : 'C';
  if ((lhs != 'R' && lhs != 'C') || (rhs != 'R' && rhs != 'C') || (cl != 'R' && cl != 'C') || mode.size() > 3)
    return fail(KEBAB_EINVAL, "opmode must be two (or three, with C's layout) of R/C, got \"" + mode + "\"");
  const bool c_row = (cl == 'R') || map_reference_id(version) == 141;
  const int id = resolve(version, M, N, K, lhs == 'R' && rhs == 'C' && !c_row, rhs == 'C');
  if (id < 0) return -id;
  const Rung* r = find_rung(id);
  GemmProblem p{(int)dtype, A, B, C, M, N, K, lhs, rhs, c_row, reinterpret_cast<cudaStream_t>(stream)};
  return r->launch(p);
}

int kebab_gemm_gated(kebab_dtype dtype, const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                     int version, const uint32_t* b_ready, int64_t chunk_cols, uint32_t epoch,
                     kebab_stream_t stream) {
  if (!A || !B || !C || !b_ready) return fail(KEBAB_EINVAL, "null pointer passed to kebab_gemm_gated");
  if (M <= 0 || N <= 0 || K <= 0) return fail(KEBAB_EINVAL, "invalid dimensions");
  if (dtype != KEBAB_F16 && dtype != KEBAB_BF16) return fail(KEBAB_EINVAL, "gated GEMM supports F16 and BF16");
  // The heuristic keeps to widths that divide the 512-aligned chunks callers use.
  const int id = resolve(version, M, N, K, true, false);
  if (id < 0) return -id;
  if (id != 104 && id != 105 && id != 107 && id != 112)
    return fail(KEBAB_ENOTSUP, "gated B runs on the persistent rungs 104, 105, 107 and 112; version " +
                                   std::to_string(version) + " resolves to " + std::to_string(id));
  GemmProblem p{(int)dtype, A, B, C, M, N, K, 'R', 'C', false, reinterpret_cast<cudaStream_t>(stream)};
  p.b_ready = b_ready;
  p.b_chunk_cols = chunk_cols;
  p.b_epoch = epoch;
  return find_rung(id)->launch(p);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// C++ mirror of the reference interface (kebab/include/kebab/cuda/cuda_gemm.h)
// ---------------------------------------------------------------------------
namespace baseline {

const char* gemm_cuda_version_feature_name(int version) { return kebab_version_name(version); }

static void report(int rc, const char* what) {
  if (rc != KEBAB_OK) std::fprintf(stderr, "ERROR: %s: %s\n", what, kebab_last_error());
}

void gemm(const float* A, const float* B, float* C, int M, int N, int K, const char* opmode, int version,
          cudaStream_t stream) {
  report(kebab_gemm(KEBAB_F32, A, B, C, M, N, K, opmode, version, stream), "baseline::gemm (float)");
}
void gemm(const __half* A, const __half* B, __half* C, int M, int N, int K, const char* opmode, int version,
          cudaStream_t stream) {
  report(kebab_gemm(KEBAB_F16, A, B, C, M, N, K, opmode, version, stream), "baseline::gemm (half)");
}
void gemm(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C, int M, int N, int K,
          const char* opmode, int version, cudaStream_t stream) {
  report(kebab_gemm(KEBAB_BF16, A, B, C, M, N, K, opmode, version, stream), "baseline::gemm (bfloat16)");
}

#define KEBAB_RUNG_LAUNCHER(NAME, ID)                                                                            \
  void NAME##_fp16(const __half* A, const __half* B, __half* C, int M, int N, int K, char lhs_format,          \
                   char rhs_format, cudaStream_t stream) {                                                     \
    const char mode[3] = {lhs_format, rhs_format, 0};                                                          \
    report(kebab_gemm(KEBAB_F16, A, B, C, M, N, K, mode, ID, stream), #NAME "_fp16");                         \
  }                                                                                                            \
  void NAME##_bf16(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C, int M, int N, int K,      \
                   char lhs_format, char rhs_format, cudaStream_t stream) {                                    \
    const char mode[3] = {lhs_format, rhs_format, 0};                                                          \
    report(kebab_gemm(KEBAB_BF16, A, B, C, M, N, K, mode, ID, stream), #NAME "_bf16");                        \
  }

KEBAB_RUNG_LAUNCHER(gemm_v1_simt_warptiling, 1)
KEBAB_RUNG_LAUNCHER(gemm_v101_tma_mmasync, 101)
KEBAB_RUNG_LAUNCHER(gemm_v102_tma_umma_tmem, 102)
KEBAB_RUNG_LAUNCHER(gemm_v103_tma_umma_tmem_warpspecialized, 103)
KEBAB_RUNG_LAUNCHER(gemm_v104_tma_umma_tmem_warpspecialized_persistent, 104)
KEBAB_RUNG_LAUNCHER(gemm_v105_tma_umma_tmem_warpspecialized_persistent_2cta, 105)
KEBAB_RUNG_LAUNCHER(gemm_v106_tma_umma_tmem_swapab_splitk_cluster_skinny, 106)
KEBAB_RUNG_LAUNCHER(gemm_v107_tma_umma_tmem_warpspecialized_persistent_2cta_256x512, 107)
KEBAB_RUNG_LAUNCHER(gemm_v108_tma_umma_tmem_warpspecialized_persistent_streamk, 108)
KEBAB_RUNG_LAUNCHER(gemm_v109_tma_umma_tmem_warpspecialized_persistent_2cta_streamk, 109)
KEBAB_RUNG_LAUNCHER(gemm_v110_tma_umma_tmem_warpspecialized_persistent_128x128, 110)
KEBAB_RUNG_LAUNCHER(gemm_v111_tma_umma_tmem_warpspecialized_persistent_128x64, 111)
KEBAB_RUNG_LAUNCHER(gemm_v112_tma_umma_tmem_warpspecialized_persistent_2cta_256x384, 112)
KEBAB_RUNG_LAUNCHER(gemm_v141_tma_umma_tmem_warpspecialized_persistent_2cta_rowmajor_c, 141)
#undef KEBAB_RUNG_LAUNCHER

// The reference's launcher names, forwarding to the rung their id maps to.
#define KEBAB_REFERENCE_ALIAS_F16(NAME, ID)                                                              \
  void NAME(const __half* A, const __half* B, __half* C, int M, int N, int K, char lhs_format,          \
            char rhs_format, cudaStream_t stream) {                                                     \
    const char mode[3] = {lhs_format, rhs_format, 0};                                                   \
    report(kebab_gemm(KEBAB_F16, A, B, C, M, N, K, mode, ID, stream), #NAME);                           \
  }
#define KEBAB_REFERENCE_ALIAS_BF16(NAME, ID)                                                             \
  void NAME(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C, int M, int N, int K,       \
            char lhs_format, char rhs_format, cudaStream_t stream) {                                    \
    const char mode[3] = {lhs_format, rhs_format, 0};                                                   \
    report(kebab_gemm(KEBAB_BF16, A, B, C, M, N, K, mode, ID, stream), #NAME);                          \
  }
KEBAB_REFERENCE_ALIASES
#undef KEBAB_REFERENCE_ALIAS_F16
#undef KEBAB_REFERENCE_ALIAS_BF16

}  // namespace baseline

// ---------------------------------------------------------------------------
// CuTe-API alias (kebab/include/kebab/cute/gemm.h)
// ---------------------------------------------------------------------------
#include "kebab/cute/gemm.h"

namespace kebab {
namespace cute {

namespace {
std::string cute_mode(const char* opmode) {
  std::string m(opmode ? opmode : "default");
  std::transform(m.begin(), m.end(), m.begin(), [](unsigned char c) { return (char)std::toupper(c); });
  if (m == "DEFAULT" || m.empty()) return "RR";
  if (m.size() == 1) m += 'R';  // the CuTe path's default rhs
  return m;
}
template <typename T>
int dtype_of();
template <>
int dtype_of<__half>() { return KEBAB_F16; }
template <>
int dtype_of<__nv_bfloat16>() { return KEBAB_BF16; }
template <>
int dtype_of<float>() { return KEBAB_F32; }
}  // namespace

template <typename T>
void gemm(const T* A, const T* B, T* C, int M, int N, int K, const char* opmode, int version, cudaStream_t stream) {
  (void)version;  // every CuTe version resolves to the decomposition heuristic
  const std::string mode = cute_mode(opmode);
  const int rc = kebab_gemm((kebab_dtype)dtype_of<T>(), A, B, C, M, N, K, mode.c_str(), 120, stream);
  if (rc != KEBAB_OK) std::fprintf(stderr, "ERROR: kebab::cute::gemm: %s\n", kebab_last_error());
}

template void gemm<__half>(const __half*, const __half*, __half*, int, int, int, const char*, int, cudaStream_t);
template void gemm<__nv_bfloat16>(const __nv_bfloat16*, const __nv_bfloat16*, __nv_bfloat16*, int, int, int,
                                  const char*, int, cudaStream_t);
template void gemm<float>(const float*, const float*, float*, int, int, int, const char*, int, cudaStream_t);

}  // namespace cute
}  // namespace kebab
