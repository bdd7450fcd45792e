// 2:4 structured sparsity on the GPU: prune, pack, metadata encoders, and the
// compression into the operand layout of tcgen05.mma.sp.
//
// The reference does all of this on the host, for one 16 x 32 tile
// (kebab/lib/microbench/sparse_mma.cu:38-166, cutlass_meta_probe.cu:43-173).
// These kernels produce bit-identical results for whole matrices:
//   prune  : keep the 2 largest |a| of each group of 4 along K, with exactly
//            the tie order of std::partial_sort(idx, idx+2, idx+4, greater)
//            as libstdc++ implements it (heap-select of 2 then sort-heap),
//            which is what the reference calls; zero the rest (+0.0).
//   pack   : the two non-zeros of each group in ascending position, and their
//            positions as one uint32 per packed entry; fails (status) when a
//            group does not hold exactly two non-zeros.
//   codes / cutlass-il2 / rowpair / il2-ordered: the reference's metadata
//            encoders, generalised tile by tile (16 x 32 tiles of A in
//            row-major tile order).
//   compress: pruned A -> (packed A, metadata in the tcgen05 sparse layout)
//            for kebab_gemm_sparse24; see kSparseETile below.
// All kernels are HBM-bound integer work: one thread per group (or per
// 16-wide K chunk), coalesced 8/16-byte accesses, grid-stride loops sized to
// the SM count.
#include <algorithm>

#include "gemm_umma.cuh"
#include "internal.h"
#include "kebab/sparse24.h"

namespace kb {

namespace {

__device__ __forceinline__ float h2f(uint16_t v, int bf16) {
  if (bf16) return __uint_as_float((uint32_t)v << 16);
  return __half2float(__ushort_as_half(v));
}

// The pair of positions std::partial_sort(idx, idx+2, idx+4, cmp) keeps, with
// cmp(a, b) = v[a] > v[b]: make_heap on {0,1}, then for i = 2, 3 replace the
// heap top when cmp(i, top), re-heapifying the two-element heap.
__device__ __forceinline__ void partial_sort_top2(const float v[4], int& a, int& b) {
  // make_heap([0,1]): top is 0 iff v1 > v0
  int h0, h1;
  if (v[1] > v[0]) {
    h0 = 0;
    h1 = 1;
  } else {
    h0 = 1;
    h1 = 0;
  }
#pragma unroll
  for (int i = 2; i < 4; ++i) {
    if (v[i] > v[h0]) {
      // pop_heap(first, middle, i) with value i: adjust the 2-heap {h1, i}
      if (v[h1] > v[i]) {
        h0 = i;  // heap = [i, h1]
      } else {
        h0 = h1;  // heap = [h1, i]
        h1 = i;
      }
    }
  }
  a = h0;
  b = h1;
}

__device__ __forceinline__ uint2 prune_group(uint2 raw, int bf16) {
  uint16_t e[4] = {(uint16_t)(raw.x & 0xFFFF), (uint16_t)(raw.x >> 16), (uint16_t)(raw.y & 0xFFFF),
                   (uint16_t)(raw.y >> 16)};
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = fabsf(h2f(e[i], bf16));
  int a, b;
  partial_sort_top2(v, a, b);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (i != a && i != b) e[i] = 0;
  return make_uint2(e[0] | ((uint32_t)e[1] << 16), e[2] | ((uint32_t)e[3] << 16));
}

// Four groups (two 16-byte loads) per thread and iteration: enough bytes in
// flight per thread to stream at HBM rate.
__global__ void prune_kernel(const uint16_t* __restrict__ A, uint16_t* __restrict__ out, int64_t groups, int bf16) {
  const int64_t quads = groups / 4;
  const uint4* src = reinterpret_cast<const uint4*>(A);
  uint4* dst = reinterpret_cast<uint4*>(out);
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < quads; q += (int64_t)gridDim.x * blockDim.x) {
    const uint4 x = src[2 * q], y = src[2 * q + 1];
    const uint2 a0 = prune_group(make_uint2(x.x, x.y), bf16), a1 = prune_group(make_uint2(x.z, x.w), bf16);
    const uint2 b0 = prune_group(make_uint2(y.x, y.y), bf16), b1 = prune_group(make_uint2(y.z, y.w), bf16);
    dst[2 * q] = make_uint4(a0.x, a0.y, a1.x, a1.y);
    dst[2 * q + 1] = make_uint4(b0.x, b0.y, b1.x, b1.y);
  }
  // Tail (groups % 4), handled by the first threads of block 0.
  if (blockIdx.x == 0 && threadIdx.x < groups % 4) {
    const int64_t g = quads * 4 + threadIdx.x;
    reinterpret_cast<uint2*>(out)[g] = prune_group(reinterpret_cast<const uint2*>(A)[g], bf16);
  }
}

// Positions of the two non-zeros (ascending); returns false unless exactly two.
__device__ __forceinline__ bool find_pair(const uint16_t e[4], int bf16, int& p0, int& p1) {
  int found = 0;
  p0 = p1 = -1;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (h2f(e[i], bf16) != 0.0f) {
      if (found == 0) p0 = i;
      else if (found == 1) p1 = i;
      ++found;
    }
  }
  return found == 2;
}

__global__ void pack_kernel(const uint16_t* __restrict__ As, uint16_t* __restrict__ packed, uint32_t* __restrict__ meta,
                            int64_t groups, int bf16, uint32_t* fail_count) {
  uint32_t bad = 0;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups; g += (int64_t)gridDim.x * blockDim.x) {
    const uint2 raw = reinterpret_cast<const uint2*>(As)[g];
    const uint16_t e[4] = {(uint16_t)(raw.x & 0xFFFF), (uint16_t)(raw.x >> 16), (uint16_t)(raw.y & 0xFFFF),
                           (uint16_t)(raw.y >> 16)};
    int p0, p1;
    if (!find_pair(e, bf16, p0, p1)) {
      ++bad;
      continue;
    }
    reinterpret_cast<uint32_t*>(packed)[g] = e[p0] | ((uint32_t)e[p1] << 16);
    reinterpret_cast<uint2*>(meta)[g] = make_uint2((uint32_t)p0, (uint32_t)p1);
  }
  if (bad) atomicAdd(fail_count, bad);
}

__device__ __forceinline__ uint32_t encode_pair(uint32_t i0, uint32_t i1) {
  // (0,1)->0 (0,2)->1 (0,3)->2 (1,2)->3 (1,3)->4 (2,3)->5, anything else -> 0
  if (i0 >= i1 || i1 > 3) return 0;
  if (i0 == 0) return i1 - 1;
  if (i0 == 1) return i1 + 1;
  return 5;
}

__global__ void codes_kernel(const uint32_t* __restrict__ meta, uint32_t* __restrict__ codes, int64_t groups) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups; g += (int64_t)gridDim.x * blockDim.x) {
    const uint2 p = reinterpret_cast<const uint2*>(meta)[g];
    codes[g] = encode_pair(p.x, p.y);
  }
}

// One thread per (16x32 tile, row pair): CUTLASS ColumnMajorInterleaved<2>.
__global__ void meta_cutlass_kernel(const uint32_t* __restrict__ meta, uint32_t* __restrict__ out, int64_t M,
                                    int64_t K) {
  const int64_t PK = K / 2, tiles_k = K / 32, work = (M / 16) * tiles_k * 8;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < work; w += (int64_t)gridDim.x * blockDim.x) {
    const int rp = (int)(w & 7);
    const int64_t tile = w >> 3, tm = tile / tiles_k, tk = tile % tiles_k;
    const uint32_t* r0 = meta + (tm * 16 + 2 * rp) * PK + tk * 16;
    const uint32_t* r1 = r0 + PK;
    uint32_t c0r0 = 0, c1r0 = 0, c0r1 = 0, c1r1 = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      c0r0 |= (r0[i] & 3u) << (2 * i);
      c1r0 |= (r0[i + 8] & 3u) << (2 * i);
      c0r1 |= (r1[i] & 3u) << (2 * i);
      c1r1 |= (r1[i + 8] & 3u) << (2 * i);
    }
    uint32_t* t = out + tile * 64;
    // slots 4rp..4rp+3: word0, 0, word1, 0 ; slots 32..63 of the tile are zero
    reinterpret_cast<uint4*>(t)[rp] = make_uint4(c0r0 | (c0r1 << 16), 0u, c1r0 | (c1r1 << 16), 0u);
    reinterpret_cast<uint4*>(t)[8 + rp] = make_uint4(0u, 0u, 0u, 0u);
  }
}

// Ordered 4-bit group codes, 16x32 tiles, 32 u32 per tile.
__global__ void meta_ordered_kernel(const uint32_t* __restrict__ codes, uint32_t* __restrict__ out, int64_t M,
                                    int64_t K, int rowpair) {
  const int64_t G = K / 4, tiles_k = K / 32, work = (M / 16) * tiles_k * 16;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < work; w += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(w & 15);
    const int64_t tile = w >> 4, tm = tile / tiles_k, tk = tile % tiles_k;
    uint32_t* t = out + tile * 32;
    if (rowpair) {
      if (r < 8) {
        const uint32_t* c0 = codes + (tm * 16 + r) * G + tk * 8;
        const uint32_t* c1 = codes + (tm * 16 + r + 8) * G + tk * 8;
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          w0 |= (c0[g] & 0xFu) << (4 * g);
          w0 |= (c1[g] & 0xFu) << (16 + 4 * g);
          w1 |= (c0[g + 4] & 0xFu) << (4 * g);
          w1 |= (c1[g + 4] & 0xFu) << (16 + 4 * g);
        }
        t[2 * r] = w0;
        t[2 * r + 1] = w1;
      } else {
        t[2 * r] = 0;
        t[2 * r + 1] = 0;
      }
    } else {
      const uint32_t* c = codes + (tm * 16 + r) * G + tk * 8;
      uint32_t e0 = 0, e1 = 0;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        e0 |= (c[g] & 0xFu) << (4 * g);
        e1 |= (c[g + 4] & 0xFu) << (4 * g);
      }
      t[2 * r] = e0;
      t[2 * r + 1] = e1;
    }
  }
}

// Pruned A -> packed A + tcgen05 sparse metadata. One thread per 16-wide K
// chunk of one row (4 groups: 32 bytes in, 16 bytes packed out, 16 metadata
// bits out). Metadata nibble of a group = p0 | p1 << 2 (p0 < p1).
__global__ void compress_kernel(const uint16_t* __restrict__ As, uint16_t* __restrict__ packed,
                                uint16_t* __restrict__ E, int64_t M, int64_t K, int bf16, uint32_t* fail_count) {
  const int64_t chunks_per_row = K / 16, work = M * chunks_per_row, tiles_k = K / 128;
  uint32_t bad = 0;
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < work; w += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = w / chunks_per_row, kc = w % chunks_per_row;
    const uint4* src = reinterpret_cast<const uint4*>(As + m * K + kc * 16);
    const uint4 x = src[0], y = src[1];
    const uint32_t words[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
    uint32_t outw[4];
    uint32_t bits = 0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint16_t e[4] = {(uint16_t)(words[2 * g] & 0xFFFF), (uint16_t)(words[2 * g] >> 16),
                             (uint16_t)(words[2 * g + 1] & 0xFFFF), (uint16_t)(words[2 * g + 1] >> 16)};
      int p0, p1;
      if (!find_pair(e, bf16, p0, p1)) {
        ++bad;
        p0 = 0;
        p1 = 1;
      }
      outw[g] = e[p0] | ((uint32_t)e[p1] << 16);
      bits |= (uint32_t)(p0 | (p1 << 2)) << (4 * g);
    }
    *reinterpret_cast<uint4*>(packed + m * (K / 2) + kc * 8) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
    // Tile (m / 128, k / 128), 2048 bytes; inside: m = m0 + 8 m1 + 16 m2,
    // k = 16 k1 + 32 k2 (+ k0 inside the 16-bit chunk):
    // byte = 16 m0 + 2 m1 + 256 m2 + 128 k1 + 4 k2.
    const int64_t k = kc * 16;
    const int64_t tile = (m / 128) * tiles_k + k / 128;
    const int mi = (int)(m % 128), ki = (int)(k % 128);
    const int m0 = mi & 7, m1 = (mi >> 3) & 1, m2 = mi >> 4, k1 = (ki >> 4) & 1, k2 = ki >> 5;
    const int byte = 16 * m0 + 2 * m1 + 256 * m2 + 128 * k1 + 4 * k2;
    E[(tile * 2048 + byte) / 2] = (uint16_t)bits;
  }
  if (bad) atomicAdd(fail_count, bad);
}

int grid_for(int64_t work, int threads) {
  DeviceInfo* d = nullptr;
  int sms = (device_info(&d) == KEBAB_OK) ? d->sm_count : 148;
  int64_t blocks = (work + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sms * 8));
}

int check_common(int dtype, const void* a, const void* b, int64_t M, int64_t K, int64_t m_align, int64_t k_align) {
  if (!a || !b) return fail(KEBAB_EINVAL, "null pointer");
  if (dtype != KEBAB_F16 && dtype != KEBAB_BF16) return fail(KEBAB_EINVAL, "2:4 path supports F16 and BF16");
  if (M <= 0 || K <= 0 || M % m_align || K % k_align)
    return fail(KEBAB_EINVAL, "2:4 shapes need M % " + std::to_string(m_align) + " == 0 and K % " +
                                  std::to_string(k_align) + " == 0");
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15u)
    return fail(KEBAB_EINVAL, "2:4 buffers must be 16-byte aligned");
  return KEBAB_OK;
}

int launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KEBAB_OK : cuda_fail(e, what);
}

// Per-device failure counter used by pack / compress. It is a __device__
// variable (no allocation); the call reads it back synchronously.
__device__ uint32_t g_sparse_fail;

int reset_fail(uint32_t** ptr, cudaStream_t s) {
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(ptr), g_sparse_fail);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(fail counter)");
  e = cudaMemsetAsync(*ptr, 0, sizeof(uint32_t), s);
  return e == cudaSuccess ? KEBAB_OK : cuda_fail(e, "cudaMemsetAsync");
}

int read_fail(uint32_t* ptr, cudaStream_t s, uint32_t* n) {
  cudaError_t e = cudaMemcpyAsync(n, ptr, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "reading the 2:4 failure counter");
  if (*n) return fail(KEBAB_ESPARSE, std::to_string(*n) + " groups do not hold exactly two non-zeros");
  return KEBAB_OK;
}

}  // namespace
}  // namespace kb

using namespace kb;

extern "C" {

int kebab_sparse24_prune(kebab_dtype dtype, const void* A, void* A_pruned, int64_t M, int64_t K,
                         kebab_stream_t stream) {
  int rc = check_common(dtype, A, A_pruned, M, K, 1, 4);
  if (rc) return rc;
  const int64_t groups = M * K / 4;
  prune_kernel<<<grid_for(groups / 4 + 1, 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint16_t*)A, (uint16_t*)A_pruned, groups, dtype == KEBAB_BF16);
  return launched("prune_kernel");
}

int kebab_sparse24_pack(kebab_dtype dtype, const void* A_pruned, void* A_packed, uint32_t* meta, int64_t M,
                        int64_t K, kebab_stream_t stream) {
  int rc = check_common(dtype, A_pruned, A_packed, M, K, 1, 4);
  if (rc) return rc;
  if (!meta) return fail(KEBAB_EINVAL, "null metadata pointer");
  cudaStream_t s = (cudaStream_t)stream;
  uint32_t* fc = nullptr;
  if ((rc = reset_fail(&fc, s))) return rc;
  const int64_t groups = M * K / 4;
  pack_kernel<<<grid_for(groups, 256), 256, 0, s>>>((const uint16_t*)A_pruned, (uint16_t*)A_packed, meta, groups,
                                                    dtype == KEBAB_BF16, fc);
  if ((rc = launched("pack_kernel"))) return rc;
  uint32_t n = 0;
  return read_fail(fc, s, &n);
}

int kebab_sparse24_group_codes(const uint32_t* meta, uint32_t* codes, int64_t M, int64_t K, kebab_stream_t stream) {
  int rc = check_common(KEBAB_F16, meta, codes, M, K, 1, 4);
  if (rc) return rc;
  const int64_t groups = M * K / 4;
  codes_kernel<<<grid_for(groups, 256), 256, 0, (cudaStream_t)stream>>>(meta, codes, groups);
  return launched("codes_kernel");
}

int kebab_sparse24_meta_cutlass(const uint32_t* meta, uint32_t* out, int64_t M, int64_t K, kebab_stream_t stream) {
  int rc = check_common(KEBAB_F16, meta, out, M, K, 16, 32);
  if (rc) return rc;
  const int64_t work = (M / 16) * (K / 32) * 8;
  meta_cutlass_kernel<<<grid_for(work, 256), 256, 0, (cudaStream_t)stream>>>(meta, out, M, K);
  return launched("meta_cutlass_kernel");
}

int kebab_sparse24_meta_ordered(const uint32_t* codes, uint32_t* out, int64_t M, int64_t K, int rowpair,
                                kebab_stream_t stream) {
  int rc = check_common(KEBAB_F16, codes, out, M, K, 16, 32);
  if (rc) return rc;
  const int64_t work = (M / 16) * (K / 32) * 16;
  meta_ordered_kernel<<<grid_for(work, 256), 256, 0, (cudaStream_t)stream>>>(codes, out, M, K, rowpair ? 1 : 0);
  return launched("meta_ordered_kernel");
}

int kebab_sparse24_compress(kebab_dtype dtype, const void* A_pruned, void* A_packed, void* E, int64_t M, int64_t K,
                            kebab_stream_t stream) {
  int rc = check_common(dtype, A_pruned, A_packed, M, K, 128, 128);
  if (rc) return rc;
  if (!E || (reinterpret_cast<uintptr_t>(E) & 15u)) return fail(KEBAB_EINVAL, "E must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  uint32_t* fc = nullptr;
  if ((rc = reset_fail(&fc, s))) return rc;
  const int64_t work = M * (K / 16);
  compress_kernel<<<grid_for(work, 256), 256, 0, s>>>((const uint16_t*)A_pruned, (uint16_t*)A_packed, (uint16_t*)E, M,
                                                      K, dtype == KEBAB_BF16, fc);
  if ((rc = launched("compress_kernel"))) return rc;
  uint32_t n = 0;
  return read_fail(fc, s, &n);
}

int64_t kebab_sparse24_e_bytes(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0 || M % 128 || K % 128) return -KEBAB_EINVAL;
  return (M / 128) * (K / 128) * 2048;
}

}  // extern "C"
