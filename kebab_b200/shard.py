"""M-row-block sharding of one GEMM across the GPUs of a node.

Rank r of P owns rows [r*M/P, (r+1)*M/P) of A — a contiguous slab of the
row-major A — and computes its own column-major C shard (ldC = M/P) through
kebab_gemm. B is replicated once by a broadcast from rank 0 (NCCL over
NVLink on GPUs). C stays sharded unless gather_c() is called. The reference
has no multi-GPU path; this is the layout the north star asks for.

The collectives go through torch.distributed, so the same host logic runs
on `gloo` ranks on CPU (tests/test_shard.py) with a stand-in GEMM.
"""
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
