/*
 * kebab-b200 C ABI — 2:4 structured sparsity (FP16/BF16 A, row-major M x K).
 *
 * The reference has only host-side packers for one 16 x 32 tile, used by its
 * mma.sp microbenchmark (kebab/lib/microbench/sparse_mma.cu:38-166,
 * cutlass_meta_probe.cu:43-173). These entry points run the same algorithms
 * on the GPU for whole matrices, bit-exact, plus the compression into the
 * tcgen05.mma.sp operand layout and the sparse GEMM itself. All pointers are
 * device pointers, 16-byte aligned; calls are asynchronous on `stream` unless
 * documented as synchronous.
 */
#ifndef KEBAB_SPARSE24_H_
#define KEBAB_SPARSE24_H_

#include "kebab/kebab.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Keep the two largest |a| of every group of 4 along K, zero the others
 * (+0.0), breaking ties exactly as std::partial_sort(idx, idx+2, idx+4,
 * greater) does in libstdc++. Replaces prune_dense_to_sparse_2of4
 * (sparse_mma.cu:63-85; cutlass_meta_probe.cu:116-138). K % 4 == 0;
 * A_pruned may equal A. */
int kebab_sparse24_prune(kebab_dtype dtype, const void* A, void* A_pruned, int64_t M, int64_t K,
                         kebab_stream_t stream);

/* Pack a pruned A: A_packed (M x K/2) holds each group's two non-zeros in
 * ascending position, meta (M x K/2 uint32) their positions 0..3. Returns
 * KEBAB_ESPARSE if any group does not hold exactly two non-zeros (the
 * reference returns false). Synchronous (reads the failure count back).
 * Replaces encode_sparse_to_packed_and_meta (sparse_mma.cu:88-119). */
int kebab_sparse24_pack(kebab_dtype dtype, const void* A_pruned, void* A_packed, uint32_t* meta, int64_t M,
                        int64_t K, kebab_stream_t stream);

/* Group codes 0..5 ((0,1)->0 ... (2,3)->5) from the position pairs, one
 * uint32 per group (M x K/4). Replaces encode_2of4 (sparse_mma.cu:38-48). */
int kebab_sparse24_group_codes(const uint32_t* meta, uint32_t* codes, int64_t M, int64_t K, kebab_stream_t stream);

/* CUTLASS ColumnMajorInterleaved<2> metadata, 64 uint32 per 16 x 32 tile of
 * A, tiles in row-major tile order. M % 16 == 0, K % 32 == 0. Replaces
 * encode_cutlass_metadata_interleaved2 (cutlass_meta_probe.cu:43-77). */
int kebab_sparse24_meta_cutlass(const uint32_t* meta, uint32_t* out, int64_t M, int64_t K, kebab_stream_t stream);

/* Ordered 4-bit code layouts, 32 uint32 per 16 x 32 tile: rowpair != 0 gives
 * encode_ordered_metadata_rowpair, 0 gives encode_ordered_metadata_
 * interleaved2 (sparse_mma.cu:122-166). */
int kebab_sparse24_meta_ordered(const uint32_t* codes, uint32_t* out, int64_t M, int64_t K, int rowpair,
                                kebab_stream_t stream);

/* Bytes of the tcgen05 metadata buffer for an M x K sparse A (2048 per
 * 128 x 128 block), or a negative KEBAB_* code. M % 128 == 0, K % 128 == 0.
 * No reference counterpart. */
int64_t kebab_sparse24_e_bytes(int64_t M, int64_t K);

/* Pruned A -> A_packed (M x K/2) + E (kebab_sparse24_e_bytes bytes): the
 * operands of kebab_gemm_sparse24. Synchronous; KEBAB_ESPARSE as for pack.
 * No reference counterpart (the reference's sparse path stops at one mma.sp
 * tile, sparse_mma.cu:347-428). */
int kebab_sparse24_compress(kebab_dtype dtype, const void* A_pruned, void* A_packed, void* E, int64_t M, int64_t K,
                            kebab_stream_t stream);

/* C = A * B with A 2:4 sparse, given as (A_packed, E) from
 * kebab_sparse24_compress; B dense K x N column-major; C M x N column-major,
 * FP32 accumulation (tcgen05.mma.sp). M % 128 == 0, K % 128 == 0.
 * No reference counterpart (see above). */
int kebab_gemm_sparse24(kebab_dtype dtype, const void* A_packed, const void* E, const void* B, void* C, int64_t M,
                        int64_t N, int64_t K, kebab_stream_t stream);

/* Tile of the CTA-pair kernel kebab_gemm_sparse24 launches for an M x N
 * output on the current device: writes its rows (512, or 256 / 128 when
 * KEBAB_SPARSE_CG selects the older tiles) and columns. Returns KEBAB_OK or
 * a KEBAB_* code. No reference counterpart. */
int kebab_sparse24_tile(int64_t M, int64_t N, int* tile_m, int* tile_n);

#ifdef __cplusplus
}
#endif
#endif /* KEBAB_SPARSE24_H_ */
