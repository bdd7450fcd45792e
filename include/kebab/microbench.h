/*
 * kebab-b200 microbenchmark probes (sm_100a), the counterparts of the
 * reference's Hopper probes in kebab/lib/microbench (mma_wgmma.cu:390-470,
 * 740-826: one verified op + a throughput loop; copy_gmem_to_smem_2d_tma_ptx.cu:
 * 129-181: TMA bandwidth). All calls synchronize the device and return a
 * KEBAB_* status. No TMA-multicast probe is built: multicast loads are kept
 * out of every source file that multi-GPU runs use.
 */
#ifndef KEBAB_MICROBENCH_H_
#define KEBAB_MICROBENCH_H_

#include "kebab/kebab.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One chain of four (128*cta_group) x 256 x 16 tcgen05.mma on operands that
 * are all 1.0 (FP16, or BF16 when ab_bf16), read back from TMEM with
 * tcgen05.ld into host_out [cta_group*128][256] (every value must be 64). */
int kebab_mbench_umma_once(int ab_bf16, int cta_group, float* host_out, int64_t host_out_len);

/* Back-to-back tcgen05.mma (M = 128*cta_group, N = n, K = 16) from one thread
 * per CTA (pair) on every SM, `iters` x 4 instructions each: TFLOP/s of the
 * whole GPU and SM cycles per instruction. */
int kebab_mbench_umma(int cta_group, int n, int ab_bf16, int iters, double* tflops, double* cycles_per_mma);

/* As kebab_mbench_umma for tcgen05.mma.sp (2:4 sparse A, FP16, K = 32
 * logical per instruction): dense-equivalent TFLOP/s (2 * M * N * K_logical)
 * and SM cycles per instruction. No reference counterpart (the reference's
 * 2:4 probe is one mma.sp tile, kebab/lib/microbench/sparse_mma.cu). */
int kebab_mbench_umma_sp(int cta_group, int n, int iters, double* tflops, double* cycles_per_mma);

/* Issue-to-completion latency of one 128 x 256 x 16 MMA + commit + mbarrier
 * wait, averaged over `iters`, in SM cycles. */
int kebab_mbench_umma_latency(int iters, double* cycles);

/* tcgen05.ld 32x32b.x32 + wait::ld loop on 4 warps per SM: bytes per SM
 * cycle and aggregate TB/s. */
int kebab_mbench_tmem_ld(int iters, double* bytes_per_clk_per_sm, double* tbps);

/* 2-D TMA loads (box box_rows x 64 FP16, 128-byte swizzle, 8-deep ring) of a
 * device buffer [rows][cols] FP16 split across all SMs: GB/s. */
int kebab_mbench_tma_load(const void* buf, int64_t rows, int64_t cols, int box_rows, double* gbps);

/* The tma_load loop over a buffer small enough to stay in L2 (first read by
 * an untimed pass), read `passes` times with `stages` boxes of box_rows x 64
 * FP16 in flight per SM (1..8, at most 200 KB): aggregate GB/s and bytes per
 * SM cycle (median CTA). Shows how much operand data one SM can take in per
 * cycle, and how that depends on the bytes it keeps in flight. Variant of
 * the reference's TMA bandwidth probe (copy_gmem_to_smem_2d_tma_ptx.cu). */
int kebab_mbench_tma_ingest(const void* buf, int64_t rows, int64_t cols, int box_rows, int stages, int passes,
                            double* gbps, double* bytes_per_clk_per_sm);

#ifdef __cplusplus
}
#endif
#endif /* KEBAB_MICROBENCH_H_ */
