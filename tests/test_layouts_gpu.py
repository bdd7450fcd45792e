"""Every storage layout of the tensor-core rungs against the oracle: A row- or
column-major, B column- or row-major (the reference's RC / RR / CR / CC
opmodes), C column-major (the reference's convention) or row-major (the
reference's v41, here rung 141 or a third opmode character 'R'). The oracle
works in RC, so inputs are re-laid out on the host for it."""
import os
import subprocess

import numpy as np
import pytest

import oracle as O
from gemm_util import assert_close, torch_dtype

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(cuda, M, N, K, opmode, version, dtype=O.F16, seed=0):
    import torch
    import kebab_b200 as kb
    A, B = O.fill_pair(M, N, K, seed=seed, dtype=dtype, dist=O.NORMAL, scale_a=1 / np.sqrt(K),
                       scale_b=1 / np.sqrt(K))
    ref = O.gemm(A, B, M, N, K, dtype).reshape(N, M)  # ref[j, i] = C[i, j]
    A2 = A.reshape(M, K)          # row-major A
    B2 = B.reshape(N, K)          # column-major B (stored N x K)
    lhs, rhs = opmode[0], opmode[1]
    c_row = (len(opmode) > 2 and opmode[2] == "R") or version == 141
    a_store = A2 if lhs == "R" else np.ascontiguousarray(A2.T)  # col-major A = K x M row-major
    b_store = B2 if rhs == "C" else np.ascontiguousarray(B2.T)  # row-major B = K x N
    td = torch_dtype(dtype)
    dA = torch.from_numpy(a_store.view(np.int16)).to(cuda).view(td)
    dB = torch.from_numpy(b_store.view(np.int16)).to(cuda).view(td)
    dC = torch.full((M * N,), float("nan"), dtype=td, device=cuda)
    rc = kb.gemm_raw(dtype, dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), M, N, K, opmode, version,
                     torch.cuda.current_stream().cuda_stream)
    assert rc == kb.OK, kb.last_error()
    torch.cuda.synchronize()
    assert kb.device_status()[0] == kb.OK
    c = dC.float().cpu().numpy()
    got = c.reshape(M, N).T if c_row else c.reshape(N, M)  # -> [j, i]
    assert_close(np.ascontiguousarray(got).reshape(-1), ref.reshape(-1), "%s v%d %dx%dx%d" % (opmode, version, M, N, K),
                 dtype)


@pytest.mark.parametrize("opmode", ["RC", "RR", "CR", "CC", "RCR", "RRR", "CRR", "CCR"])
@pytest.mark.parametrize("version", [1, 103, 104, 105, 107, 108, 109, 110, 111, 112, 120])
def test_layouts(cuda, opmode, version):
    if version == 112 and opmode[1] == "R":
        # rung 112 takes column-major B only, and says so
        import torch
        import kebab_b200 as kb
        p = torch.empty(1 << 20, dtype=torch.float16, device=cuda)
        assert kb.gemm_raw(0, p.data_ptr(), p.data_ptr(), p.data_ptr(), 384, 512, 320, opmode, version,
                           torch.cuda.current_stream().cuda_stream) == kb.ENOTSUP
        return
    _run(cuda, 384, 512, 320, opmode, version)


@pytest.mark.parametrize("opmode", ["RC", "CC", "RCR", "CCR"])
def test_v112_two_waves_ragged(cuda, opmode):
    """256 x 384 pair tiles: several tiles per pair, ragged N (last tile 1/3 full), both C layouts."""
    _run(cuda, 3072, 2176, 448, opmode, 112)


@pytest.mark.parametrize("version", [105, 110, 111])
@pytest.mark.parametrize("kps", ["1", "2"])
@pytest.mark.parametrize("opmode", ["RC", "RR", "CC", "CRR"])
def test_ring_shapes(cuda, opmode, kps, version, monkeypatch):
    """The rungs' two rings (one K-block per stage, or two): K = 200 ends
    inside the second K-block of a stage, ragged M and N."""
    monkeypatch.setenv("KEBAB_KPS", kps)
    _run(cuda, 520, 776, 200, opmode, version)


@pytest.mark.parametrize("opmode", ["RR", "CC", "RCR"])
def test_layouts_ragged_and_bf16(cuda, opmode):
    _run(cuda, 264, 520, 136, opmode, 105)
    _run(cuda, 512, 256, 1024, opmode, 104, dtype=O.BF16, seed=3)


def test_rung_141_and_reference_id_41(cuda):
    # v41 of the reference: RC inputs, row-major C.
    _run(cuda, 512, 768, 256, "RC", 141)
    _run(cuda, 512, 768, 256, "RCR", 141)
    import kebab_b200 as kb
    assert kb.version_name(41) == kb.version_name(141)


def test_unsupported_layouts_rejected(cuda):
    import torch
    import kebab_b200 as kb
    x = torch.empty(256 * 256, dtype=torch.float16, device=cuda)
    for v in (101, 102, 106):
        rc = kb.gemm_raw(kb.F16, x.data_ptr(), x.data_ptr(), x.data_ptr(), 256, 256, 256, "RR", v,
                         torch.cuda.current_stream().cuda_stream)
        assert rc == kb.ENOTSUP
    rc = kb.gemm_raw(kb.F16, x.data_ptr(), x.data_ptr(), x.data_ptr(), 256, 256, 256, "RCX", 104,
                     torch.cuda.current_stream().cuda_stream)
    assert rc == kb.EINVAL


def test_cute_alias_example(cuda):
    r = subprocess.run([os.path.join(ROOT, "kebab_b200", "bin", "simple_gemm")], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout + r.stderr
