"""Programmatic dependent launch (PDL): a GEMM launched right behind another
on the same stream may start its prologue early, but must read its inputs
only after the previous kernel finished.

The chained test makes the second GEMM consume the first one's output with
nothing in between on the stream; a read that came too early would see the
NaN fill the buffer held before. The results are compared bit for bit with
the same chain run with a host synchronisation between the two launches, and
with a process that has PDL switched off (KEBAB_PDL=0).
"""
import hashlib
import os
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# (M, N, K, version): each rung family that launches with PDL.
CASES = [
    (64, 4096, 4096, 106),   # skinny split-K cluster
    (1024, 1024, 2048, 104),  # persistent 1-CTA
    (1024, 2048, 2048, 105),  # CTA pairs
    (2048, 2048, 2048, 107),  # 256 x 512 pair tiles
    (1536, 1024, 4096, 109),  # stream-K pairs
]


def _chain(kb, M, N, K, version, sync_between, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A1 = (torch.randn(M, K, device="cuda", generator=g) / K ** 0.5).half()
    B1 = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).half()
    # Second GEMM: A2 = C1 read as an N x M row-major matrix (K2 = M).
    N2 = 512
    B2 = (torch.randn(N2, M, device="cuda", generator=g) / M ** 0.5).half()
    C1 = torch.full((N, M), float("nan"), device="cuda", dtype=torch.half)
    C2 = torch.full((N2, N), float("nan"), device="cuda", dtype=torch.half)
    torch.cuda.synchronize()
    kb.gemm(A1, B1, C1, version=version)
    if sync_between:
        torch.cuda.synchronize()
    kb.gemm(C1, B2, C2, version=120)
    torch.cuda.synchronize()
    return C1, C2


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,version", CASES)
def test_chained_gemms_read_completed_inputs(cuda, M, N, K, version):
    import kebab_b200 as kb

    C1, C2 = _chain(kb, M, N, K, version, sync_between=False)
    R1, R2 = _chain(kb, M, N, K, version, sync_between=True)
    assert torch.isfinite(C2.float()).all()
    assert torch.equal(C1, R1)
    assert torch.equal(C2, R2)
    # Back-to-back repeats of the same launch (the bench's pattern).
    g = torch.Generator(device="cuda").manual_seed(1)
    A = (torch.randn(M, K, device="cuda", generator=g) / K ** 0.5).half()
    B = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).half()
    outs = [torch.empty(N, M, device="cuda", dtype=torch.half) for _ in range(4)]
    for o in outs:
        kb.gemm(A, B, o, version=version)
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


_HASH_SCRIPT = r"""
import hashlib, sys, torch
sys.path.insert(0, sys.argv[1])
import kebab_b200 as kb
out = []
for M, N, K, v in %r:
    g = torch.Generator(device="cuda").manual_seed(3)
    A = (torch.randn(M, K, device="cuda", generator=g) / K ** 0.5).half()
    B = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).half()
    C = kb.gemm(A, B, version=v)
    torch.cuda.synchronize()
    out.append(hashlib.sha256(C.cpu().numpy().tobytes()).hexdigest())
print(" ".join(out))
""" % (CASES,)


@pytest.mark.gpu
def test_pdl_off_gives_identical_bits(cuda):
    def run(env_pdl):
        env = dict(os.environ)
        if env_pdl is None:
            env.pop("KEBAB_PDL", None)
        else:
            env["KEBAB_PDL"] = env_pdl
        r = subprocess.run([sys.executable, "-c", _HASH_SCRIPT, ROOT], env=env, capture_output=True, text=True,
                           timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        return r.stdout.split()

    on, off = run(None), run("0")
    assert len(on) == len(CASES) and on == off


_SERP_SCRIPT = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
import kebab_b200 as kb
g = torch.Generator(device="cuda").manual_seed(11)
M, N, K = 4096, 6144, 2048
A = (torch.randn(M, K, device="cuda", generator=g) / K ** 0.5).half()
B = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).half()
outs = []
for v in (104, 105, 107):
    c1 = kb.gemm(A, B, version=v); c2 = kb.gemm(A, B, version=v)
    torch.cuda.synchronize()
    ref = (A.float() @ B.float().t()).t()
    rel = ((c1.float() - ref).norm() / ref.norm()).item()
    outs.append("%d %d %.3e" % (v, int(torch.equal(c1, c2)), rel))
print(";".join(outs))
"""


@pytest.mark.gpu
def test_serpentine_k_order(cuda):
    """The serpentine K order (the default; reverse K on alternate tiles of a
    CTA) stays deterministic and within the FP16 tolerance of an FP32
    reference."""
    env = dict(os.environ, KEBAB_SERPENTINE="1")
    r = subprocess.run([sys.executable, "-c", _SERP_SCRIPT, ROOT], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    for item in r.stdout.strip().split(";"):
        v, same, rel = item.split()
        assert same == "1" and float(rel) < 1e-3, item
