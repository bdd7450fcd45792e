"""Multi-rank host logic of the M-sharded GEMM on CPU `gloo` ranks
(world_size 2 and 4): partition arithmetic, the broadcast of B, the gather
re-layout of column-major C shards, and failure handling (a rank that dies
before the collective). The per-rank GEMM is the CPU oracle, so the sharded
result is checked bit-for-bit against the unsharded oracle."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kebab_b200.shard import (ShardError, broadcast_b, broadcast_gemm_pipelined, chunk_bounds, gather_c, row_block,
                              shard_a, sharded_gemm)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_row_block_arithmetic():
    blocks = [row_block(32768, 8, r) for r in range(8)]
    assert [b.start for b in blocks] == [r * 4096 for r in range(8)]
    assert all(b.rows == 4096 for b in blocks)
    assert row_block(16384, 8, 7).start == 14336
    with pytest.raises(ShardError):
        row_block(1000, 3, 0)            # remainder rejected
    with pytest.raises(ShardError):
        row_block(8 * 12, 8, 0)          # 12-row shards break 16-byte C pitch
    with pytest.raises(ShardError):
        row_block(64, 2, 2)              # bad rank


def _oracle_gemm(A, B, C):
    import oracle as O
    M, K = A.shape
    N = B.shape[0]
    c = O.gemm(A.view(torch.int16).numpy().view(np.uint16).reshape(-1),
               B.view(torch.int16).numpy().view(np.uint16).reshape(-1), M, N, K, O.F16)
    return torch.from_numpy(c.reshape(N, M)).to(torch.float16)


def test_chunk_bounds():
    assert chunk_bounds(8192, 4) == [(0, 2048), (2048, 4096), (4096, 6144), (6144, 8192)]
    assert chunk_bounds(1000, 4) == [(0, 256), (256, 512), (512, 768), (768, 1000)]
    assert chunk_bounds(48, 4) == [(0, 48)]      # one 256-aligned chunk covers it
    assert chunk_bounds(1, 1) == [(0, 1)]
    with pytest.raises(ShardError):
        chunk_bounds(0, 4)


def _worker(rank, world, port, M, N, K, q, pipelined=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        A_glob = (torch.randn(M, K, generator=g) / K ** 0.5).to(torch.float16)
        B = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.float16) if rank == 0 \
            else torch.zeros(N, K, dtype=torch.float16)
        blk = row_block(M, world, rank)
        stand_in = lambda a, b, c: _oracle_gemm(a, b, c)
        if pipelined:
            C_shard = broadcast_gemm_pipelined(shard_a(A_glob, blk).contiguous(), B, chunks=3, gemm_fn=stand_in)
        else:
            broadcast_b(B, src=0)
            C_shard = sharded_gemm(shard_a(A_glob, blk).contiguous(), B, gemm_fn=stand_in)
        C = gather_c(C_shard, world)
        if rank == 0:
            q.put(C.view(torch.int16).numpy().copy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,pipelined,N", [(2, False, 48), (4, False, 48), (2, True, 600), (4, True, 520)])
def test_sharded_equals_unsharded(world, pipelined, N):
    # pipelined: B broadcast in 256-column chunks overlapped with the per-chunk GEMMs.
    M, K = 64 * world, 40
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, K, q, pipelined)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = torch.Generator().manual_seed(0)
    A = (torch.randn(M, K, generator=g) / K ** 0.5).to(torch.float16)
    B = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.float16)
    want = _oracle_gemm(A, B, None).view(torch.int16).numpy()
    assert np.array_equal(got, want)


def _dying_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # leaves between steps, before the broadcast
    B = torch.ones(8, 8)
    try:
        broadcast_b(B, src=0)
        q.put("no error")
    except Exception as e:  # the surviving rank learns of it through the collective
        q.put("error: %s" % type(e).__name__)


def test_rank_failure_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert msg.startswith("error"), msg
    assert procs[1].exitcode == 3
