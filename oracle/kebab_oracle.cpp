// kebab_oracle — CPU restatement of the reference's GEMM path. TEST
// INFRASTRUCTURE ONLY: only tests/, __graft_entry__.smoke() and bench.py's
// cpu_baseline / reference legs load this library, as the checker. The GPU
// product path never calls it.
//
// Parity is pinned: tests/test_oracle_pin.py checks every function here
// bit-for-bit against the reference's own code compiled from its sources into
// oracle/_ref (oracle/build_oracle.py), and against the committed fixtures in
// tests/golden/ (which that script generated from the compiled reference).
//
// What each function restates (paths within LancerLab/kebab):
//   kbo_gemm*            kebab/include/kebab/utils/reference_gemm.h:41-92
//                        (referenceGemmCpp<float>, RC: getA 'R' A[i*K+k],
//                        getB 'C' B[j*K+k], column-major C[j*M+i], per-element
//                        sequential k sum starting at 0.0f, `sum += a*b`).
//   kbo_fill_pair        kebab/include/kebab/utils/matrix_init.h:64-73 (RAND:
//                        mt19937 + uniform_real_distribution<float>(-1,1) in
//                        storage order, A then B from one generator, then
//                        round-to-nearest-even to FP16/BF16). The normal
//                        distribution is new (the reference has none): a
//                        Box-Muller transform over the same mt19937 stream.
//   kbo_prune_2of4       kebab/lib/microbench/sparse_mma.cu:63-85
//   kbo_pack_2of4        kebab/lib/microbench/sparse_mma.cu:88-119
//   kbo_encode_2of4      kebab/lib/microbench/sparse_mma.cu:38-48
//   kbo_meta_cutlass_il2 kebab/lib/microbench/cutlass_meta_probe.cu:43-77
//   kbo_meta_rowpair /   kebab/lib/microbench/sparse_mma.cu:122-166
//   kbo_meta_il2_ordered
//
// Build flags matter: -O3 -ffp-contract=off -fno-fast-math, so that every
// `sum += a*b` is a float multiply rounded to float followed by a float add,
// exactly like the reference compiled the same way. Vectorising across
// output columns keeps each element's summation order intact.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

namespace {

enum Dtype : int { DT_F16 = 0, DT_BF16 = 1 };

// --- exact conversions ------------------------------------------------------
float half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: renormalise
      int e = -1;
      do {
        man <<= 1;
        ++e;
      } while ((man & 0x400u) == 0);
      bits = sign | (uint32_t)(127 - 15 - e) << 23 | (man & 0x3FFu) << 13;
    }
  } else if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | (exp + 127 - 15) << 23 | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

float bf16_to_float(uint16_t b) {
  uint32_t bits = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// IEEE binary32 -> binary16, round to nearest even (what __float2half does).
uint16_t float_to_half(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) {  // inf or nan
    return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  }
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to inf
  if (ax < 0x38800000u) {                                      // result subnormal or zero
    // value = ax as float; half subnormal unit is 2^-24.
    uint32_t e = ax >> 23;
    if (e < 102) return (uint16_t)sign;  // < 2^-25: rounds to zero
    uint32_t man = (ax & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126 - e;  // so that result = man >> shift (in units of 2^-24)
    uint32_t res = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1u);
    uint32_t half_ulp = 1u << (shift - 1);
    if (rem > half_ulp || (rem == half_ulp && (res & 1u))) ++res;
    return (uint16_t)(sign | res);
  }
  uint32_t res = ((ax >> 13) - (112u << 10));
  uint32_t rem = ax & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (res & 1u))) ++res;
  return (uint16_t)(sign | res);
}

uint16_t float_to_bf16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40u);
  uint32_t lsb = (x >> 16) & 1u;
  x += 0x7FFFu + lsb;
  return (uint16_t)(x >> 16);
}

inline float to_float(uint16_t v, int dt) { return dt == DT_BF16 ? bf16_to_float(v) : half_to_float(v); }
inline uint16_t from_float(float v, int dt) { return dt == DT_BF16 ? float_to_bf16(v) : float_to_half(v); }

int resolve_threads(int threads) {
  if (threads > 0) return threads;
  unsigned hc = std::thread::hardware_concurrency();
  return hc ? (int)hc : 1;
}

template <class F>
void parallel_for(int64_t n, int threads, F&& f) {
  threads = (int)std::min<int64_t>(std::max(1, threads), std::max<int64_t>(1, n));
  if (threads <= 1) {
    f(0, n);
    return;
  }
  std::vector<std::thread> ts;
  int64_t chunk = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    int64_t b = t * chunk, e = std::min(n, b + chunk);
    if (b >= e) break;
    ts.emplace_back([&, b, e] { f(b, e); });
  }
  for (auto& t : ts) t.join();
}

// Core: rows [r0, r1) of C for the column block [j0, j1), from a float A
// (row-major M x K) and a transposed float B (row-major K x N, Bt[k*N + j]).
// For each (i, j) the sum runs k = 0..K-1 in order from 0.0f: identical
// arithmetic to referenceGemmCpp<float>; vectorisation is across j only.
constexpr int JB = 128;
constexpr int IB = 4;

__attribute__((target_clones("avx2", "default"))) void gemm_block(const float* A, const float* Bt, int64_t N,
                                                                    int64_t K, int64_t i0, int64_t ni, int64_t j0,
                                                                    int64_t nj, float* out /* ni x JB */) {
  float acc[IB][JB];
  for (int64_t ii = 0; ii < IB; ++ii)
    for (int64_t jj = 0; jj < JB; ++jj) acc[ii][jj] = 0.0f;
  for (int64_t k = 0; k < K; ++k) {
    const float* b = Bt + k * N + j0;
    for (int64_t ii = 0; ii < ni; ++ii) {
      const float a = A[(i0 + ii) * K + k];
      float* acc_row = acc[ii];
      if (nj == JB) {
        for (int64_t jj = 0; jj < JB; ++jj) acc_row[jj] += a * b[jj];
      } else {
        for (int64_t jj = 0; jj < nj; ++jj) acc_row[jj] += a * b[jj];
      }
    }
  }
  for (int64_t ii = 0; ii < ni; ++ii)
    for (int64_t jj = 0; jj < nj; ++jj) out[ii * JB + jj] = acc[ii][jj];
}

void widen(const uint16_t* src, float* dst, int64_t n, int dt, int threads) {
  parallel_for(n, threads, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) dst[i] = to_float(src[i], dt);
  });
}

// B is column-major K x N (B[j*K + k]); produce Bt[k*N + j] as float.
void widen_transpose_b(const uint16_t* B, float* Bt, int64_t K, int64_t N, int dt, int threads) {
  parallel_for(K, threads, [&](int64_t k0, int64_t k1) {
    for (int64_t j = 0; j < N; ++j)
      for (int64_t k = k0; k < k1; ++k) Bt[k * N + j] = to_float(B[j * K + k], dt);
  });
}

}  // namespace

extern "C" {

int kbo_version() { return 1; }

uint16_t kbo_float_to_half(float f) { return float_to_half(f); }
uint16_t kbo_float_to_bf16(float f) { return float_to_bf16(f); }
float kbo_half_to_float(uint16_t h) { return half_to_float(h); }
float kbo_bf16_to_float(uint16_t h) { return bf16_to_float(h); }

// Fills A (nA elements) then B (nB elements) from ONE mt19937(seed) stream.
// dist 0: uniform_real_distribution<float>(-1, 1), times `scale` when scale
//         != 1 (scale 1 reproduces matrix_init.h RAND exactly).
// dist 1: normal N(0, scale^2) by Box-Muller: u1 = (g() + 0.5) / 2^32,
//         u2 = (g() + 0.5) / 2^32 (double), r = sqrt(-2 ln u1),
//         z0 = r cos(2 pi u2), z1 = r sin(2 pi u2); values are taken in pairs
//         (z0 then z1), each times `scale`, rounded to float, then to the
//         storage type. A and B share the stream; a trailing odd value's
//         partner is discarded, never carried into B.
void kbo_fill_pair(uint16_t* A, int64_t nA, int distA, double scaleA, uint16_t* B, int64_t nB, int distB,
                   double scaleB, uint32_t seed, int dtype) {
  std::mt19937 gen(seed);
  auto fill = [&](uint16_t* dst, int64_t n, int dist, double scale) {
    if (dist == 0) {
      std::uniform_real_distribution<float> u(-1.0f, 1.0f);
      const bool unit = (scale == 1.0);
      for (int64_t i = 0; i < n; ++i) {
        float v = u(gen);
        if (!unit) v = (float)((double)v * scale);
        dst[i] = from_float(v, dtype);
      }
    } else {
      const double two_pi = 6.283185307179586476925286766559;
      for (int64_t i = 0; i < n; i += 2) {
        double u1 = ((double)gen() + 0.5) / 4294967296.0;
        double u2 = ((double)gen() + 0.5) / 4294967296.0;
        double r = std::sqrt(-2.0 * std::log(u1));
        dst[i] = from_float((float)(r * std::cos(two_pi * u2) * scale), dtype);
        if (i + 1 < n) dst[i + 1] = from_float((float)(r * std::sin(two_pi * u2) * scale), dtype);
      }
    }
  };
  if (A && nA > 0) fill(A, nA, distA, scaleA);
  if (B && nB > 0) fill(B, nB, distB, scaleB);
}

// Full C = A * B (RC), FP32 column-major C (ldC = M). threads <= 0: all cores.
int kbo_gemm(const uint16_t* A, const uint16_t* B, float* C, int64_t M, int64_t N, int64_t K, int dtype,
             int threads) {
  if (M <= 0 || N <= 0 || K <= 0) return 22;
  threads = resolve_threads(threads);
  std::vector<float> Af((size_t)(M * K)), Bt((size_t)(K * N));
  widen(A, Af.data(), M * K, dtype, threads);
  widen_transpose_b(B, Bt.data(), K, N, dtype, threads);
  const int64_t nib = (M + IB - 1) / IB, njb = (N + JB - 1) / JB;
  parallel_for(nib * njb, threads, [&](int64_t b, int64_t e) {
    std::vector<float> out(IB * JB);
    for (int64_t t = b; t < e; ++t) {
      int64_t ib = t / njb, jb = t % njb;
      int64_t i0 = ib * IB, ni = std::min<int64_t>(IB, M - i0);
      int64_t j0 = jb * JB, nj = std::min<int64_t>(JB, N - j0);
      gemm_block(Af.data(), Bt.data(), N, K, i0, ni, j0, nj, out.data());
      for (int64_t ii = 0; ii < ni; ++ii)
        for (int64_t jj = 0; jj < nj; ++jj) C[(j0 + jj) * M + (i0 + ii)] = out[ii * JB + jj];
    }
  });
  return 0;
}

// Rows `rows[0..nrows)` of C, written row by row: out[r*N + j] = C[rows[r], j].
// Same arithmetic as kbo_gemm; B is widened/transposed once.
int kbo_gemm_rows(const uint16_t* A, const uint16_t* B, const int64_t* rows, int64_t nrows, float* out, int64_t M,
                  int64_t N, int64_t K, int dtype, int threads) {
  if (M <= 0 || N <= 0 || K <= 0) return 22;
  threads = resolve_threads(threads);
  std::vector<float> Af((size_t)(nrows * K)), Bt((size_t)(K * N));
  for (int64_t r = 0; r < nrows; ++r) {
    if (rows[r] < 0 || rows[r] >= M) return 22;
    for (int64_t k = 0; k < K; ++k) Af[r * K + k] = to_float(A[rows[r] * K + k], dtype);
  }
  widen_transpose_b(B, Bt.data(), K, N, dtype, threads);
  const int64_t nib = (nrows + IB - 1) / IB, njb = (N + JB - 1) / JB;
  parallel_for(nib * njb, threads, [&](int64_t b, int64_t e) {
    std::vector<float> blk(IB * JB);
    for (int64_t t = b; t < e; ++t) {
      int64_t ib = t / njb, jb = t % njb;
      int64_t i0 = ib * IB, ni = std::min<int64_t>(IB, nrows - i0);
      int64_t j0 = jb * JB, nj = std::min<int64_t>(JB, N - j0);
      gemm_block(Af.data(), Bt.data(), N, K, i0, ni, j0, nj, blk.data());
      for (int64_t ii = 0; ii < ni; ++ii)
        for (int64_t jj = 0; jj < nj; ++jj) out[(i0 + ii) * N + j0 + jj] = blk[ii * JB + jj];
    }
  });
  return 0;
}

// Individual elements C[ii[e], jj[e]] (scalar sequential-k sums).
int kbo_gemm_elems(const uint16_t* A, const uint16_t* B, const int64_t* ii, const int64_t* jj, int64_t n, float* out,
                   int64_t M, int64_t N, int64_t K, int dtype, int threads) {
  threads = resolve_threads(threads);
  for (int64_t e = 0; e < n; ++e)
    if (ii[e] < 0 || ii[e] >= M || jj[e] < 0 || jj[e] >= N) return 22;
  parallel_for(n, threads, [&](int64_t b, int64_t e1) {
    for (int64_t e = b; e < e1; ++e) {
      const uint16_t* a = A + ii[e] * K;
      const uint16_t* bb = B + jj[e] * K;
      float sum = 0.0f;
      for (int64_t k = 0; k < K; ++k) sum += to_float(a[k], dtype) * to_float(bb[k], dtype);
      out[e] = sum;
    }
  });
  return 0;
}

// ----------------------------------------------------------------------------
// 2:4 structured sparsity (FP16 A, row-major M x K, K % 4 == 0)
// ----------------------------------------------------------------------------

// Keep the two largest |a| of every group of 4 along K; zero the other two.
// The pair kept under ties is the one std::partial_sort(idx, idx+2, idx+4,
// greater-by-|a|) selects, which is what the reference calls.
int kbo_prune_2of4(const uint16_t* A, uint16_t* out, int64_t M, int64_t K) {
  if (M <= 0 || K <= 0 || K % 4) return 22;
  if (out != A) std::memcpy(out, A, sizeof(uint16_t) * (size_t)(M * K));
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t g = 0; g < K / 4; ++g) {
      uint16_t* grp = out + m * K + g * 4;
      float vals[4];
      int idx[4] = {0, 1, 2, 3};
      for (int i = 0; i < 4; ++i) vals[i] = std::fabs(half_to_float(grp[i]));
      std::partial_sort(idx, idx + 2, idx + 4, [&](int a, int b) { return vals[a] > vals[b]; });
      for (int i = 0; i < 4; ++i)
        if (i != idx[0] && i != idx[1]) grp[i] = 0;  // +0.0 in FP16
    }
  }
  return 0;
}

// Pack a pruned A: per group, the two non-zero entries (ascending position)
// go to packed[m*K/2 + 2g + {0,1}] and their positions (0..3) to
// meta[same]. Returns 0, or 1 when any group does not have exactly 2
// non-zeros (the reference's `return false`); outputs are then unspecified.
int kbo_pack_2of4(const uint16_t* As, uint16_t* packed, uint32_t* meta, int64_t M, int64_t K) {
  if (M <= 0 || K <= 0 || K % 4) return 22;
  const int64_t PK = K / 2;
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t g = 0; g < K / 4; ++g) {
      int nz[2] = {-1, -1}, found = 0;
      for (int i = 0; i < 4; ++i) {
        if (half_to_float(As[m * K + g * 4 + i]) != 0.0f) {
          if (found < 2) nz[found] = i;
          ++found;
        }
      }
      if (found != 2) return 1;
      packed[m * PK + 2 * g + 0] = As[m * K + g * 4 + nz[0]];
      packed[m * PK + 2 * g + 1] = As[m * K + g * 4 + nz[1]];
      meta[m * PK + 2 * g + 0] = (uint32_t)nz[0];
      meta[m * PK + 2 * g + 1] = (uint32_t)nz[1];
    }
  }
  return 0;
}

// Pair of kept positions -> code 0..5 ((0,1)->0 ... (2,3)->5); others -> 0.
uint32_t kbo_encode_2of4(int i0, int i1) {
  static const int table[4][4] = {{0, 0, 1, 2}, {0, 0, 3, 4}, {0, 0, 0, 5}, {0, 0, 0, 0}};
  if (i0 < 0 || i0 > 3 || i1 < 0 || i1 > 3 || i0 >= i1) return 0;
  return (uint32_t)table[i0][i1];
}

// CUTLASS ColumnMajorInterleaved<2> metadata, generalised tile by tile: the
// matrix is cut into 16-row x 32-column tiles of A (16 x 16 packed entries),
// tiles in row-major tile order, 64 u32 slots per tile. In a tile, row pair
// rp (rows 2rp, 2rp+1) gives word0 = (2-bit positions of packed entries 0..7
// of row 2rp) | (same of row 2rp+1) << 16 and word1 = the same for entries
// 8..15; word0 goes to slot 2*(2rp) and word1 to slot 2*(2rp+1) (the
// ColumnMajorInterleaved<2> offset of logical rows 2rp and 2rp+1 of a {32,1}
// extent); the other slots are zero. Requires M % 16 == 0, K % 32 == 0.
int kbo_meta_cutlass_il2(const uint32_t* meta, int64_t M, int64_t K, uint32_t* out) {
  if (M <= 0 || K <= 0 || M % 16 || K % 32) return 22;
  const int64_t PK = K / 2, tiles_k = K / 32;
  for (int64_t tm = 0; tm < M / 16; ++tm) {
    for (int64_t tk = 0; tk < tiles_k; ++tk) {
      uint32_t* t = out + (tm * tiles_k + tk) * 64;
      std::memset(t, 0, 64 * sizeof(uint32_t));
      for (int rp = 0; rp < 8; ++rp) {
        const uint32_t* r0 = meta + (tm * 16 + 2 * rp) * PK + tk * 16;
        const uint32_t* r1 = r0 + PK;
        uint32_t c0r0 = 0, c1r0 = 0, c0r1 = 0, c1r1 = 0;
        for (int i = 0; i < 8; ++i) {
          c0r0 |= (r0[i] & 3u) << (2 * i);
          c1r0 |= (r0[i + 8] & 3u) << (2 * i);
          c0r1 |= (r1[i] & 3u) << (2 * i);
          c1r1 |= (r1[i + 8] & 3u) << (2 * i);
        }
        t[2 * (2 * rp)] = c0r0 | (c0r1 << 16);
        t[2 * (2 * rp + 1)] = c1r0 | (c1r1 << 16);
      }
    }
  }
  return 0;
}

// Group codes: codes[m*(K/4) + g] = encode(meta pair of group g of row m).
int kbo_group_codes(const uint32_t* meta, int64_t M, int64_t K, uint32_t* codes) {
  if (M <= 0 || K <= 0 || K % 4) return 22;
  const int64_t PK = K / 2, G = K / 4;
  for (int64_t m = 0; m < M; ++m)
    for (int64_t g = 0; g < G; ++g)
      codes[m * G + g] = kbo_encode_2of4((int)meta[m * PK + 2 * g], (int)meta[m * PK + 2 * g + 1]);
  return 0;
}

// Ordered-metadata layouts of the reference's single 16x32 tile, generalised
// tile by tile (16 rows x 32 columns of A, 8 group codes per tile row, 32 u32
// per tile, tiles in row-major tile order). Row-pair layout: for rp in 0..7,
// rows rp and rp+8; word0 = codes g=0..3 of row rp at 4g | of row rp+8 at
// 16+4g, word1 the same for g=4..7, stored at 2rp, 2rp+1.
int kbo_meta_rowpair(const uint32_t* codes, int64_t M, int64_t K, uint32_t* out) {
  if (M <= 0 || K <= 0 || M % 16 || K % 32) return 22;
  const int64_t G = K / 4, tiles_k = K / 32;
  for (int64_t tm = 0; tm < M / 16; ++tm)
    for (int64_t tk = 0; tk < tiles_k; ++tk) {
      uint32_t* t = out + (tm * tiles_k + tk) * 32;
      for (int rp = 0; rp < 8; ++rp) {
        const uint32_t* c0 = codes + (tm * 16 + rp) * G + tk * 8;
        const uint32_t* c1 = codes + (tm * 16 + rp + 8) * G + tk * 8;
        uint32_t w0 = 0, w1 = 0;
        for (int g = 0; g < 4; ++g) {
          w0 |= (c0[g] & 0xFu) << (4 * g);
          w0 |= (c1[g] & 0xFu) << (16 + 4 * g);
          w1 |= (c0[g + 4] & 0xFu) << (4 * g);
          w1 |= (c1[g + 4] & 0xFu) << (16 + 4 * g);
        }
        t[2 * rp] = w0;
        t[2 * rp + 1] = w1;
      }
      for (int s = 16; s < 32; ++s) t[s] = 0;
    }
  return 0;
}

// Interleaved-2 ordered layout: per row m of the tile, e0 = codes g=0..3 at
// 4g, e1 = codes g=4..7 at 4g, stored at 2m, 2m+1.
int kbo_meta_il2_ordered(const uint32_t* codes, int64_t M, int64_t K, uint32_t* out) {
  if (M <= 0 || K <= 0 || M % 16 || K % 32) return 22;
  const int64_t G = K / 4, tiles_k = K / 32;
  for (int64_t tm = 0; tm < M / 16; ++tm)
    for (int64_t tk = 0; tk < tiles_k; ++tk) {
      uint32_t* t = out + (tm * tiles_k + tk) * 32;
      for (int r = 0; r < 16; ++r) {
        const uint32_t* c = codes + (tm * 16 + r) * G + tk * 8;
        uint32_t e0 = 0, e1 = 0;
        for (int g = 0; g < 4; ++g) {
          e0 |= (c[g] & 0xFu) << (4 * g);
          e1 |= (c[g + 4] & 0xFu) << (4 * g);
        }
        t[2 * r] = e0;
        t[2 * r + 1] = e1;
      }
    }
  return 0;
}

}  // extern "C"
