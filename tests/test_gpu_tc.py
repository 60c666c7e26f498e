"""Tensor-core (tcgen05) matmul, g2k_matmul_tc, against the oracle's
restatement of the reference's prefill matmul (main.c:593-684: serial-k fp32
dot plus bias), with its gelu / add epilogues (main.c:1767-1774).

Tolerances, max|gpu - ref| <= RTOL * max|ref|:
* G2_F32 (three tf32 products of split operands): 2e-5, fp32-level;
* G2_F16 (fp16 operands): the oracle runs on the same fp16-rounded operands,
  so only the accumulation order and the tensor core's internal accumulation
  differ: 1e-3.
Shapes cover partial feature tiles (N % 128 != 0), partial row tiles, a single
row, split-K and the GPT-2 small / medium / XL projection shapes.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RNG = np.random.default_rng(7)
fp = oracle.fptr
L = oracle.cpu_lib


@pytest.fixture(scope="module")
def g2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gpt2b200
    return gpt2b200


def rnd(*shape, s=1.0):
    return (RNG.standard_normal(shape, dtype=np.float32) * np.float32(s)).astype(np.float32)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def ref_matmul(A, B, bias):
    M, K = A.shape
    N = B.shape[1]
    out = np.zeros((M, N), np.float32)
    L().ref_matmul(fp(A), fp(B), None if bias is None else fp(bias), fp(out), M, N, K)
    return out


def rel_err(got, want):
    return float(np.abs(got.astype(np.float64) - want).max() / max(np.abs(want).max(), 1e-30))


SHAPES = [(64, 2304, 768), (64, 768, 3072), (5, 384, 128), (1, 256, 64), (33, 200, 64), (130, 4800, 1600),
          (512, 3072, 768), (256, 1024, 4096), (32, 4800, 1600), (32, 1024, 4096)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("precision", ["f32", "f16"])
def test_matmul_tc(g2, M, N, K, precision):
    prec = g2.G2_F32 if precision == "f32" else g2.G2_F16
    A, B, b = rnd(M, K, s=1.0), rnd(K, N, s=0.02), rnd(N, s=0.1)
    if prec == g2.G2_F16:   # the oracle sees exactly the operands the tensor cores multiply
        A, B = A.astype(np.float16).astype(np.float32), B.astype(np.float16).astype(np.float32)
    want = ref_matmul(A, B, b)
    tol = 2e-5 if prec == g2.G2_F32 else 1e-3
    ws_bytes = g2.matmul_tc_workspace(M, N, K, prec)
    ws = torch.zeros(ws_bytes // 4 + 64, dtype=torch.float32, device="cuda")
    C_ = torch.full((M, N), float("nan"), device="cuda")
    g2.matmul_tc(dev(A), dev(B), C_, M, N, K, bias=dev(b), precision=prec, workspace=ws, workspace_bytes=ws_bytes)
    got = host(C_)
    assert int(ws[:1].view(torch.int32).item()) == 0, "a wait inside the kernel expired"
    assert np.isfinite(got).all()
    assert rel_err(got, want) <= tol, f"rel err {rel_err(got, want):.2e}"
    # GELU (launch_gelu, main.c:1774) and residual add (launch_add, main.c:1767), residual aliasing C
    g_want = want.copy().reshape(-1)
    L().ref_gelu(fp(g_want), M * N)
    g2.matmul_tc(dev(A), dev(B), C_, M, N, K, bias=dev(b), gelu=True, precision=prec, workspace=ws,
                 workspace_bytes=ws_bytes)
    assert rel_err(host(C_).reshape(-1), g_want) <= tol
    R = rnd(M, N)
    r_want = R.copy().reshape(-1)
    L().ref_add_inplace(fp(r_want), fp(want.reshape(-1).copy()), M * N)
    C_.copy_(dev(R))
    g2.matmul_tc(dev(A), dev(B), C_, M, N, K, bias=dev(b), residual=C_, precision=prec, workspace=ws,
                 workspace_bytes=ws_bytes)
    assert rel_err(host(C_).reshape(-1), r_want) <= tol


def test_matmul_tc_rejects_bad_shapes(g2):
    ws = torch.zeros(1 << 20, device="cuda")
    A, B, C_ = torch.zeros(4, 96, device="cuda"), torch.zeros(96, 64, device="cuda"), torch.zeros(4, 64, device="cuda")
    with pytest.raises(g2.G2Error):   # K % 64 != 0
        g2.matmul_tc(A, B, C_, 4, 64, 96, workspace=ws, workspace_bytes=4 << 20)
    with pytest.raises(g2.G2Error):   # workspace too small
        g2.matmul_tc(A, B, C_, 4, 64, 64, workspace=ws, workspace_bytes=64)


def test_matmul_tc_balanced_split(g2):
    """The balanced split (the K blocks of all tiles shared out equally over the
    SMs, a CTA's share spanning up to two tiles) applies by default to 3xTF32
    GEMMs of up to 32 rows only; the same cases are run again in a process
    where G2_TC_BALANCED extends it to every GEMM of up to 32 rows, fp16 too."""
    env = dict(os.environ, G2_TC_BALANCED="32")
    r = subprocess.run([sys.executable, "-m", "pytest", __file__, "-q", "-x", "-p", "no:cacheprovider", "-k",
                        "test_matmul_tc and not balanced"], env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
