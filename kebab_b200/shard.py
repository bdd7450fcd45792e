"""M-row-block sharding of one GEMM across the GPUs of a node.

Rank r of P owns rows [r*M/P, (r+1)*M/P) of A — a contiguous slab of the
row-major A — and computes its own column-major C shard (ldC = M/P) through
kebab_gemm. B is replicated once by a broadcast from rank 0 (NCCL over
NVLink on GPUs). C stays sharded unless gather_c() is called. The reference
has no multi-GPU path; this is the layout the north star asks for.

The collectives go through torch.distributed, so the same host logic runs
on `gloo` ranks on CPU (tests/test_shard.py) with a stand-in GEMM.
"""
import os
from dataclasses import dataclass

TMA_ALIGN = 8  # rows of a shard: C's column pitch must stay 16-byte aligned


class ShardError(ValueError):
    pass


@dataclass(frozen=True)
class RowBlock:
    rank: int
    world: int
    start: int
    rows: int


def row_block(M, world, rank, align=TMA_ALIGN):
    """The contiguous row block of rank `rank`. Rejects remainders: every
    rank gets exactly M/world rows, a multiple of `align`."""
    if world <= 0 or not (0 <= rank < world):
        raise ShardError("bad rank %d of world %d" % (rank, world))
    if M <= 0 or M % world:
        raise ShardError("M=%d is not divisible by %d ranks" % (M, world))
    rows = M // world
    if rows % align:
        raise ShardError("shard of %d rows is not a multiple of %d" % (rows, align))
    return RowBlock(rank, world, rank * rows, rows)


def shard_a(A_global, block):
    """Rank's slab of a row-major [M, K] A (a view, no copy)."""
    return A_global[block.start:block.start + block.rows]


def broadcast_b(B, src=0, group=None):
    """Replicates B ([N, K], column-major K x N) from `src` to every rank."""
    import torch.distributed as dist
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.broadcast(B, src=src, group=group)
    return B


def sharded_gemm(A_shard, B, C_shard=None, version=120, gemm_fn=None, stream=None):
    """C_shard = A_shard * B on this rank ([N, rows] column-major result).
    `gemm_fn(A, B, C)` replaces kebab_gemm (tests use a CPU stand-in)."""
    if gemm_fn is None:
        import kebab_b200
        return kebab_b200.gemm(A_shard, B, C_shard, version=version, stream=stream)
    return gemm_fn(A_shard, B, C_shard)


def chunk_bounds(N, chunks, align=256):
    """Column ranges [n0, n1) of `chunks` N-chunks of B, each a multiple of
    `align` columns (the widest tile) except the last; fewer chunks when N
    is small."""
    if N <= 0 or chunks <= 0:
        raise ShardError("bad N=%d or chunks=%d" % (N, chunks))
    step = -(-N // chunks)
    step = -(-step // align) * align
    return [(n0, min(N, n0 + step)) for n0 in range(0, N, step)]


def broadcast_gemm_pipelined(A_shard, B, C_shard=None, chunks=4, src=0, version=120, gemm_fn=None, stream=None,
                             group=None):
    """Broadcast of B overlapped with this rank's GEMM: B ([N, K], column-
    major K x N, so an N-chunk is a contiguous slab) is broadcast from `src`
    in `chunks` pieces, all issued at once; the GEMM of chunk i (columns
    [n0, n1) of the [N, rows] C shard, also contiguous) starts as soon as
    chunk i has arrived, while later chunks are still in flight. On NCCL
    ranks the wait on a chunk is a stream dependency, not a host block.
    Each element of C is computed from the same A row and B column as by
    sharded_gemm; with the serpentine K order off (KEBAB_SERPENTINE=0) also
    in the same K order, so the results match it bit for bit (by default
    within tolerance). Returns C_shard.

    Measured on two B200s it is slower than broadcast-then-GEMM (32768^3
    BF16, 4 chunks: 37.4 ms against 29.1; 8192^3 FP16: 1.12 against 1.05):
    the persistent rungs size their grid to every SM, so NCCL's broadcast
    kernels and the chunk GEMMs contend for SMs instead of overlapping, and
    over NVLink the broadcast is a small share of the serial time (32768^3:
    ~3.6 of 29.1 ms)."""
    import torch
    import torch.distributed as dist
    N = B.shape[0]
    rows = A_shard.shape[0]
    if C_shard is None:
        C_shard = torch.empty((N, rows), dtype=B.dtype, device=B.device)
    bounds = chunk_bounds(N, chunks)
    multi = dist.is_initialized() and dist.get_world_size(group) > 1
    works = [dist.broadcast(B[n0:n1], src=src, group=group, async_op=True) if multi else None
             for n0, n1 in bounds]
    run_stream = stream if stream is not None else (torch.cuda.current_stream() if B.is_cuda else None)
    for (n0, n1), w in zip(bounds, works):
        if w is not None:
            # Work.wait() orders only the current stream after the broadcast;
            # the chunk's GEMM runs on `run_stream`, so make that one wait.
            if run_stream is not None:
                with torch.cuda.stream(run_stream):
                    w.wait()
            else:
                w.wait()
        out = sharded_gemm(A_shard, B[n0:n1], C_shard[n0:n1], version=version, gemm_fn=gemm_fn, stream=stream)
        if out is not None and out.data_ptr() != C_shard[n0:n1].data_ptr():
            C_shard[n0:n1].copy_(out)
    return C_shard


def gather_c(C_shard, world, group=None):
    """All-gathers the [N, rows] shards into the global column-major C
    ([N, rows*world]): column j of C is the concatenation of every rank's
    column j, so the gathered [P, N, rows] staging is re-laid out."""
    import torch
    import torch.distributed as dist
    N, rows = C_shard.shape
    if world == 1:
        return C_shard
    staging = torch.empty((world * N, rows), dtype=C_shard.dtype, device=C_shard.device)
    dist.all_gather_into_tensor(staging, C_shard.contiguous(), group=group)
    return staging.view(world, N, rows).permute(1, 0, 2).reshape(N, world * rows)


def chain_chunk_cols(N, K, elem_bytes=2, target_bytes=64 << 20, align=512):
    """Columns per chunk of the chained broadcast: about `target_bytes` of B
    per chunk, a multiple of `align` (the widest tile), at most N rounded up."""
    cols = max(align, (target_bytes // (K * elem_bytes)) // align * align)
    return min(cols, -(-N // align) * align)


class ChainBroadcastGemm:
    """Broadcast of B from rank 0 overlapped with every rank's GEMM on its
    row block, with the copies on copy engines instead of SMs.

    B moves down the rank chain 0 -> 1 -> ... -> P-1 in chunks over NVLink
    (CUDA IPC mappings of the neighbours' buffers), each chunk forwarded as
    soon as it has landed, while every rank's GEMM (kebab_gemm_gated on ranks
    >= 1, all SMs) already runs and waits per tile, bounded, for the chunk the
    tile needs. mode "push": rank r writes chunk j into rank r+1's B and then
    raises rank r+1's device flag over NVLink (kebab_chain_push); mode "pull":
    rank r copies chunk j out of rank r-1's B and raises its own flag
    (kebab_ring_pull). Which rank holds which chunk is shared through host
    shared memory ([P, chunks] uint32 slots holding the call's epoch, plus
    one "ready to receive" slot per rank; a file in /dev/shm created by rank
    0 and unlinked once every rank has mapped it).

    `B` is this rank's [N, K] buffer (rank 0's holds the data and is never
    written; the others are overwritten by every call). Collective: every
    rank constructs it and calls run() with the same shapes.

    `lib` replaces the C ABI (tests drive the host protocol on gloo ranks
    with CPU buffers and a stand-in for the copy and IPC calls); on CPU
    buffers there are no streams and run() takes A = None only."""

    def __init__(self, B, chunk_cols=None, group=None, timeout_s=20.0, copy_streams=1, mode="push", lib=None):
        import ctypes
        import mmap
        import uuid

        import numpy as np
        import torch
        import torch.distributed as dist

        import kebab_b200 as kb
        if mode not in ("push", "pull"):
            raise ShardError("mode must be push or pull")
        self.kb, self.torch, self.dist, self.group = kb, torch, dist, group
        self.mode = mode
        self.B = B
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        N, K = B.shape
        self.N, self.K = N, K
        self.chunk_cols = chunk_cols or chain_chunk_cols(N, K, B.element_size())
        self.chunk_bytes = self.chunk_cols * K * B.element_size()
        self.total_bytes = N * K * B.element_size()
        self.nchunks = -(-self.total_bytes // self.chunk_bytes)
        self.timeout_s = timeout_s
        self.timeout_us = int(timeout_s * 1e6)
        self.ready = torch.zeros(self.nchunks, dtype=torch.int32, device=B.device)
        self.epoch = 0
        cuda = B.is_cuda
        self.copy_stream = torch.cuda.Stream(device=B.device) if cuda else None
        self.copy_stream2 = torch.cuda.Stream(device=B.device) if cuda and copy_streams > 1 else None
        self.lib = lib or kb.lib()
        L = self.lib

        def export(t):
            h = (ctypes.c_char * 64)()
            off = ctypes.c_int64(0)
            kb.check(L.kebab_ipc_export(ctypes.c_void_p(t.data_ptr()), h, ctypes.byref(off)))
            return bytes(h), off.value

        handles = [None] * self.world
        dist.all_gather_object(handles, (export(B), export(self.ready)), group=group)
        self._opened = []

        def open_(hoff):
            hb = ctypes.create_string_buffer(hoff[0], 64)
            p = ctypes.c_void_p(0)
            kb.check(L.kebab_ipc_open(hb, hoff[1], ctypes.byref(p)))
            self._opened.append(hb)
            return p.value

        self.src_ptr = self.next_b = self.next_ready = None
        if mode == "pull" and self.rank > 0:
            self.src_ptr = open_(handles[self.rank - 1][0])
        if mode == "push" and self.rank + 1 < self.world:
            self.next_b = open_(handles[self.rank + 1][0])
            self.next_ready = open_(handles[self.rank + 1][1])
        # Host slots shared by the ranks of the node: [P, chunks] chunk slots,
        # then P "ready to receive" slots.
        nbytes = (self.world * self.nchunks + self.world) * 4
        name = [None]
        if self.rank == 0:
            name[0] = "/dev/shm/kebab_chain_%d_%s" % (os.getpid(), uuid.uuid4().hex[:12])
            with open(name[0], "wb") as f:
                f.write(b"\0" * nbytes)
        dist.broadcast_object_list(name, src=self._global(0), group=group)
        fd = os.open(name[0], os.O_RDWR)
        try:
            self._mm = mmap.mmap(fd, nbytes)
        finally:
            os.close(fd)
        flat = np.frombuffer(self._mm, dtype=np.uint32)
        self.slots = flat[:self.world * self.nchunks].reshape(self.world, self.nchunks)
        self.recv_ok = flat[self.world * self.nchunks:]
        self._anchor = ctypes.c_char.from_buffer(self._mm)
        self._base = ctypes.addressof(self._anchor)
        dist.barrier(group=group)
        if self.rank == 0:
            os.unlink(name[0])

    def _global(self, r):
        return r if self.group is None else self.dist.get_global_rank(self.group, r)

    def _slot(self, r):
        return self._base + r * self.nchunks * 4

    def run(self, A, C, version=120, stream=None):
        """C = A * B on this rank, B arriving from rank 0 during the GEMM.
        Returns once this rank's part of the broadcast is done (its chunks
        landed and, in push mode, forwarded); its GEMM may still run on
        `stream`. With A None only B is broadcast (no GEMM)."""
        import ctypes
        import time
        torch, kb = self.torch, self.kb
        cuda = self.B.is_cuda
        if not cuda and A is not None:
            raise ShardError("CPU buffers: broadcast only (A must be None)")
        stream = stream or (torch.cuda.current_stream() if cuda else None)
        self.epoch = (self.epoch + 1) & 0x7FFFFFFF or 1
        epoch = self.epoch
        L = self.lib
        s1 = ctypes.c_void_p(self.copy_stream.cuda_stream if cuda else None)
        s2 = ctypes.c_void_p(self.copy_stream2.cuda_stream if self.copy_stream2 else None)
        # This call's copies overwrite B: after every earlier use of B on `stream`.
        if cuda:
            self.copy_stream.wait_stream(stream)
            if self.copy_stream2 is not None:
                self.copy_stream2.wait_stream(stream)
        if self.mode == "push":
            if self.rank > 0:
                # The previous rank writes into this B: announce when every
                # earlier reader of it (on `stream`) has finished.
                if cuda:
                    stream.synchronize()
                self.recv_ok[self.rank] = epoch
            if A is not None:
                if self.rank == 0:
                    kb.gemm(A, self.B, C, version=version, stream=stream)
                else:
                    kb.gemm_gated(A, self.B, C, self.ready, self.chunk_cols, epoch, version=version, stream=stream)
            nxt = self.rank + 1 < self.world
            if nxt:
                t0 = time.monotonic()
                while self.recv_ok[self.rank + 1] != epoch:
                    if time.monotonic() - t0 > self.timeout_s:
                        raise kb.KebabError(kb.ETIMEOUT, "rank %d never became ready to receive" % (self.rank + 1))
            kb.check(L.kebab_chain_push(
                ctypes.c_void_p(self.B.data_ptr()), ctypes.c_void_p(self.next_b if nxt else None),
                self.chunk_bytes, self.total_bytes, ctypes.c_void_p(self.next_ready if nxt else None), epoch,
                ctypes.c_void_p(self._slot(self.rank) if self.rank > 0 else None),
                ctypes.c_void_p(self._slot(self.rank + 1) if nxt else None), s1, s2, self.timeout_us))
        else:
            if self.rank == 0:
                if A is not None:
                    kb.gemm(A, self.B, C, version=version, stream=stream)
                kb.check(L.kebab_ring_pull(ctypes.c_void_p(self.B.data_ptr()), None, self.chunk_bytes,
                                           self.total_bytes, None, epoch, None, ctypes.c_void_p(self._slot(0)),
                                           None, None, self.timeout_us))
                return C
            if A is not None:
                kb.gemm_gated(A, self.B, C, self.ready, self.chunk_cols, epoch, version=version, stream=stream)
            kb.check(L.kebab_ring_pull(ctypes.c_void_p(self.B.data_ptr()), ctypes.c_void_p(self.src_ptr),
                                       self.chunk_bytes, self.total_bytes, ctypes.c_void_p(self.ready.data_ptr()),
                                       epoch, ctypes.c_void_p(self._slot(self.rank - 1)),
                                       ctypes.c_void_p(self._slot(self.rank)), s1, s2, self.timeout_us))
        if cuda:
            stream.wait_stream(self.copy_stream)
        return C

    def close(self):
        for hb in self._opened:
            self.kb.check(self.lib.kebab_ipc_close(hb))
        self._opened = []
        self.slots = self.recv_ok = None
        self._anchor = None
        if getattr(self, "_mm", None) is not None:
            self._mm.close()
            self._mm = None
