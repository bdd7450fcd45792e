"""kebab_gemm_gated: the GEMM whose B arrives in chunks while it runs (the
consumer side of the chained broadcast). One GPU: the chunks come from host
memory on a second stream (copy engine), each followed by a flag raised with
a stream memory operation, issued only after the GEMM has started waiting;
the result must equal the ungated GEMM of the same rung bit for bit. A flag
that is never raised makes the bounded wait expire with the gated-B site in
the device status, and the context stays usable."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("version,M,N,K,chunk", [(107, 1024, 4096, 2048, 1024), (105, 768, 2560, 1024, 512),
                                                 (104, 512, 3072, 512, 768), (112, 768, 2688, 1024, 768)])
def test_gated_equals_ungated(cuda, version, M, N, K, chunk):
    import torch
    import kebab_b200 as kb
    g = torch.Generator(device=cuda).manual_seed(M + N)
    A = (torch.randn(M, K, generator=g, device=cuda) / K ** 0.5).half()
    B_final = (torch.randn(N, K, generator=g, device=cuda) / K ** 0.5).half()
    hB = B_final.cpu().pin_memory()
    ref = kb.gemm(A, B_final, version=version)
    B = torch.full_like(B_final, float("nan"))
    C = torch.full((N, M), float("nan"), dtype=torch.half, device=cuda)
    ready = torch.zeros(-(-N // chunk), dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    compute, copy = torch.cuda.Stream(), torch.cuda.Stream()
    for epoch in (1, 2):  # second call: flags hold the previous epoch
        B.fill_(float("nan"))
        torch.cuda.synchronize()
        kb.gemm_gated(A, B, C, ready, chunk, epoch, version=version, stream=compute)
        time.sleep(0.02)  # the GEMM is waiting for chunk 0 by now
        with torch.cuda.stream(copy):
            for j in range(ready.numel()):
                n0, n1 = j * chunk, min(N, (j + 1) * chunk)
                B[n0:n1].copy_(hB[n0:n1], non_blocking=True)
                kb.flag_write(ready.data_ptr() + 4 * j, epoch, stream=copy)
        torch.cuda.synchronize()
        rc, code = kb.device_status()
        assert rc == kb.OK, "device status 0x%x" % code
        assert torch.equal(C.view(torch.int16), ref.view(torch.int16)), "epoch %d" % epoch


def test_gated_wait_expires(cuda):
    import torch
    import kebab_b200 as kb
    M, N, K = 512, 1024, 512
    A = torch.randn(M, K, device=cuda).half()
    B = torch.randn(N, K, device=cuda).half()
    C = torch.empty((N, M), dtype=torch.half, device=cuda)
    ready = torch.zeros(2, dtype=torch.int32, device=cuda)
    kb.device_status()
    kb.set_wait_timeout_us(50000)
    try:
        kb.gemm_gated(A, B, C, ready, 512, 7, version=104)
        rc, code = kb.device_status()
    finally:
        kb.set_wait_timeout_us(2000000)
    assert rc == kb.ETIMEOUT
    # the producer's gated-B wait (10), or the MMA / epilogue waits behind it
    assert (code & 0xFF) == 1 and ((code >> 8) & 0xFF) in (1, 3, 10), hex(code)
    # context still usable
    ref = kb.gemm(A, B, version=104)
    torch.cuda.synchronize()
    assert kb.device_status()[0] == kb.OK
    assert torch.isfinite(ref.float()).all()


def test_gated_rejects(cuda):
    import torch
    import kebab_b200 as kb
    A = torch.zeros(64, 8192, device=cuda).half()
    B = torch.zeros(8192, 8192, device=cuda).half()
    C = torch.empty((8192, 64), dtype=torch.half, device=cuda)
    ready = torch.zeros(16, dtype=torch.int32, device=cuda)
    with pytest.raises(kb.KebabError) as e:  # resolves to the skinny rung 106
        kb.gemm_gated(A, B, C, ready, 512, 1)
    assert e.value.code == kb.ENOTSUP
    A = torch.zeros(1024, 1024, device=cuda).half()
    B = torch.zeros(2048, 1024, device=cuda).half()
    C = torch.empty((2048, 1024), dtype=torch.half, device=cuda)
    with pytest.raises(kb.KebabError) as e:  # chunk not a multiple of the 256-wide tile
        kb.gemm_gated(A, B, C, ready, 300, 1, version=105)
    assert e.value.code == kb.EINVAL
