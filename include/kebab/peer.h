/*
 * kebab-b200 C ABI — multi-GPU support for the M-sharded GEMM: the broadcast
 * of B overlapped with the GEMM that consumes it.
 *
 * The reference has no multi-GPU code (no NCCL, MPI or peer access anywhere
 * in kebab/); these entry points have no reference counterpart. They serve
 * the north star's sharded configuration: rank r of P owns rows
 * [r M/P, (r+1) M/P) of A, B is replicated from rank 0 over NVLink, C stays
 * sharded. One process per GPU; the caller exchanges IPC handles and
 * provides a block of host shared memory (any mechanism: a file in /dev/shm,
 * shm_open) visible to all ranks of the node.
 *
 * Flow per call, with `epoch` one more than the previous call's (never 0):
 *   rank 0:  kebab_gemm(...) on its B; kebab_ring_pull(src = NULL) publishes
 *            every chunk.
 *   rank r:  kebab_gemm_gated(...) on the compute stream (B still arriving),
 *            then kebab_ring_pull(src = rank r-1's B, mapped with
 *            kebab_ipc_open) on a copy stream: copy-engine pulls chunk by
 *            chunk, a device flag per chunk, host slots published for rank
 *            r+1. Returns once every chunk has landed.
 * Ranks must not start the next call that rewrites B before every rank has
 * returned from this one (a barrier).
 */
#ifndef KEBAB_PEER_H_
#define KEBAB_PEER_H_

#include "kebab/kebab.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Size of an exported IPC handle (bytes). */
#define KEBAB_IPC_HANDLE_BYTES 64

/* Exports the device allocation holding `ptr`: writes a 64-byte handle and
 * the offset of `ptr` inside that allocation. */
int kebab_ipc_export(const void* ptr, void* handle, int64_t* offset);

/* Maps another process's allocation (its handle) into this process on the
 * current device and returns base + offset. Opening one handle again only
 * counts a reference. */
int kebab_ipc_open(const void* handle, int64_t offset, void** ptr);

/* Drops one reference to a mapping opened by kebab_ipc_open; the last one
 * unmaps it. */
int kebab_ipc_close(const void* handle);

/* Writes `value` to the device word `flag` in stream order, without a
 * kernel (a stream memory operation), after all earlier work on `stream`. */
int kebab_flag_write(uint32_t* flag, uint32_t value, kebab_stream_t stream);

/* GEMM (RC, column-major C; same arguments as kebab_gemm, and the same rung
 * choice except that the heuristic never picks rung 112 here) whose B is
 * still arriving: B's columns come in chunks of `chunk_cols` (a multiple of
 * the rung's tile width: 512 for rung 107, 384 for 112, 256 for 104 and
 * 105), and a tile needing chunk j waits (bounded, the kernel wait budget)
 * until b_ready[j] == epoch. Flags must be raised in chunk order. The
 * version must resolve to a persistent rung (104, 105, 107, 112), else
 * KEBAB_ENOTSUP. */
int kebab_gemm_gated(kebab_dtype dtype, const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                     int version, const uint32_t* b_ready, int64_t chunk_cols, uint32_t epoch,
                     kebab_stream_t stream);

/* One link of the broadcast chain. `have_mine` / `have_src` are this rank's
 * and the source rank's host-shared slots, one uint32 per chunk.
 * src == NULL: this rank is the source; marks every chunk held and returns.
 * Otherwise, for each chunk j of `chunk_bytes` (the last may be shorter):
 * waits until have_src[j] == epoch, then on `stream` copies the chunk from
 * src to dst (copy engine, peer memory), raises the device flag ready[j] to
 * epoch (stream memory operation) and records an event; as the events
 * complete, sets have_mine[j] = epoch. With a non-NULL `stream2` each chunk
 * is copied as two halves, the second on stream2 (two copy engines), and the
 * flag waits for both; stream2 must already be ordered after earlier users of
 * dst, like `stream`. Returns once every chunk has landed, or KEBAB_ETIMEOUT
 * when no progress is made for `timeout_us`. */
int kebab_ring_pull(void* dst, const void* src, int64_t chunk_bytes, int64_t total_bytes, uint32_t* ready,
                    uint32_t epoch, const uint32_t* have_src, uint32_t* have_mine, kebab_stream_t stream,
                    kebab_stream_t stream2, uint64_t timeout_us);

/* One link of the broadcast chain, push direction: this rank writes each
 * chunk into the next rank's buffer. `have_mine` / `have_next` are the
 * host-shared slots of this rank and of the next one.
 * For each chunk j: waits until this rank holds it (have_mine[j] == epoch;
 * have_mine NULL = the source rank, which holds every chunk), then on
 * `stream` copies it from src to dst_next (copy engine, peer memory; split
 * over stream2 as in kebab_ring_pull), writes the next rank's device flag
 * ready_next[j] = epoch (a stream memory operation on peer memory, ordered
 * after the copy) and, once the copy has completed, sets have_next[j] =
 * epoch. The last rank passes dst_next = NULL and only waits until every
 * have_mine[j] == epoch. Returns once done, or KEBAB_ETIMEOUT when no
 * progress is made for `timeout_us`. */
int kebab_chain_push(const void* src, void* dst_next, int64_t chunk_bytes, int64_t total_bytes, uint32_t* ready_next,
                     uint32_t epoch, const uint32_t* have_mine, uint32_t* have_next, kebab_stream_t stream,
                     kebab_stream_t stream2, uint64_t timeout_us);

#ifdef __cplusplus
}
#endif
#endif /* KEBAB_PEER_H_ */
