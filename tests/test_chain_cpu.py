"""Host protocol of the chained broadcast of B (shard.ChainBroadcastGemm) on
CPU `gloo` ranks (world_size 2 and 3, push and pull): IPC handle exchange,
the host-shared slots and their epochs, the "ready to receive" handshake and
repeated calls. The C ABI's copy and IPC calls are replaced by a stand-in
that does the same steps on shared host memory: every rank's B lives in a
/dev/shm file, the "IPC handle" is that file's path, and a chunk copy is a
memmove between the mappings. Afterwards every rank's B must equal rank 0's,
on every call. (The copy-engine version with the gated GEMM is checked on
GPUs by tests/test_multigpu.py.)"""
import ctypes
import mmap
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class FakeLib:
    """Stand-in for kebab_ipc_* / kebab_chain_push / kebab_ring_pull on host memory."""

    def __init__(self, registry):
        self.registry = registry  # data_ptr -> shm path
        self.maps = {}

    def kebab_ipc_export(self, ptr, handle, offset):
        path = self.registry.get(ptr.value, "none").encode()
        ctypes.memmove(handle, path.ljust(64, b"\0"), 64)
        offset._obj.value = 0
        return 0

    def kebab_ipc_open(self, handle, offset, out):
        path = handle.raw.rstrip(b"\0").decode()
        if path == "none":  # the device flags: no host stand-in needed
            out._obj.value = 0
            return 0
        fd = os.open(path, os.O_RDWR)
        mm = mmap.mmap(fd, 0)
        os.close(fd)
        anchor = ctypes.c_char.from_buffer(mm)
        self.maps[path] = (mm, anchor)
        out._obj.value = ctypes.addressof(anchor) + offset
        return 0

    def kebab_ipc_close(self, handle):
        path = handle.raw.rstrip(b"\0").decode()
        if path in self.maps:
            mm, anchor = self.maps.pop(path)
            del anchor
            mm.close()
        return 0

    @staticmethod
    def _v(p):
        return p.value if isinstance(p, ctypes.c_void_p) else p

    def _slots(self, p, n):
        a = self._v(p)
        return (ctypes.c_uint32 * n).from_address(a) if a else None

    @staticmethod
    def _wait(cond, timeout_us):
        t0 = time.monotonic()
        while not cond():
            if time.monotonic() - t0 > timeout_us * 1e-6:
                return False
            time.sleep(0)
        return True

    def kebab_chain_push(self, src, dst_next, chunk, total, ready_next, epoch, have_mine, have_next, s1, s2,
                         timeout_us):
        n = -(-total // chunk)
        mine, nxt = self._slots(have_mine, n), self._slots(have_next, n)
        for j in range(n):
            if mine is not None and not self._wait(lambda: mine[j] == epoch, timeout_us):
                return 1002
            if self._v(dst_next):
                off = j * chunk
                ctypes.memmove(self._v(dst_next) + off, self._v(src) + off, min(chunk, total - off))
                nxt[j] = epoch
        return 0

    def kebab_ring_pull(self, dst, src, chunk, total, ready, epoch, have_src, have_mine, s1, s2, timeout_us):
        n = -(-total // chunk)
        mine = self._slots(have_mine, n)
        if not self._v(src):
            for j in range(n):
                mine[j] = epoch
            return 0
        prev = self._slots(have_src, n)
        for j in range(n):
            if not self._wait(lambda: prev[j] == epoch, timeout_us):
                return 1002
            off = j * chunk
            ctypes.memmove(self._v(dst) + off, self._v(src) + off, min(chunk, total - off))
            mine[j] = epoch
        return 0


def _worker(rank, world, port, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kebab_b200.shard import ChainBroadcastGemm
        N, K = 1536, 64  # 3 chunks of 512 columns (64 KiB each)
        path = "/dev/shm/kebab_chain_test_%d_%d_%d" % (port, rank, os.getpid())
        with open(path, "wb") as f:
            f.write(b"\0" * (N * K * 2))
        mm = np.memmap(path, dtype=np.int16, mode="r+", shape=(N, K))
        B = torch.from_numpy(mm)
        chain = ChainBroadcastGemm(B, chunk_cols=512, mode=mode, lib=FakeLib({B.data_ptr(): path}))
        ok = True
        for call in range(3):  # B changes on rank 0 between calls
            if rank == 0:
                g = torch.Generator().manual_seed(100 + call)
                B.copy_(torch.randint(-30000, 30000, (N, K), generator=g, dtype=torch.int16))
            dist.barrier()
            chain.run(None, None)
            dist.barrier()
            ref = B.clone().view(torch.float16)  # gloo broadcasts no int16
            dist.broadcast(ref, src=0)
            ok = ok and torch.equal(B, ref.view(torch.int16)) and bool(np.all(chain.slots[1:] == chain.epoch))
        chain.close()
        os.unlink(path)
        q.put((rank, ok))
    except Exception as e:  # reported to the parent
        q.put((rank, "error: %r" % (e,)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,mode", [(2, "push"), (3, "push"), (3, "pull")])
def test_chain_protocol_gloo(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(v is True for v in res.values()), res
