"""Per-kernel parity on the GPU: each g2k_* entry point (C ABI, device
pointers) against the oracle's restatement of the reference kernel it
replaces, on the same seeded inputs.

Tolerance: the CUDA kernels sum in a different (parallel) order than the
reference's serial loops, so results agree to float32 rounding, not bit for
bit.  Each check requires max|gpu - ref| <= RTOL * max|ref| with RTOL = 1e-5
(the end-to-end bar in the north star is 1e-3 on logits).
"""
import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL = 1e-5


@pytest.fixture(scope="module")
def g2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gpt2b200
    return gpt2b200


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def close(got, want, rtol=RTOL):
    err = np.abs(got.astype(np.float64) - want).max()
    scale = np.abs(want).max()
    assert err <= rtol * scale + 1e-30, f"max err {err:.3e} vs scale {scale:.3e} ({err / scale:.2e} relative)"


RNG = np.random.default_rng(42)


def rnd(*shape, s=1.0):
    return (RNG.standard_normal(shape, dtype=np.float32) * np.float32(s)).astype(np.float32)


fp = oracle.fptr
L = oracle.cpu_lib


def ref_ln(x, g, b):
    out = np.zeros_like(x)
    L().ref_layernorm(fp(x), fp(out), fp(g), fp(b), x.shape[-1], 1)
    return out


@pytest.mark.parametrize("N,K", [(2304, 768), (768, 768), (3072, 768), (768, 3072), (50260, 768),
                                 (4800, 1600), (1600, 6400), (4096, 1024), (64, 16), (12, 48)])
@pytest.mark.parametrize("variant", ["plain", "ln_bias", "bias_gelu", "bias_resid"])
def test_matvec(g2, N, K, variant):
    x, W = rnd(K, s=2.0), rnd(K, N, s=0.02)
    bias = rnd(N, s=0.1) if variant != "plain" else None
    gamma, beta = (rnd(K, s=0.2) + 1.0, rnd(K, s=0.1)) if variant == "ln_bias" else (None, None)
    resid = rnd(N) if variant == "bias_resid" else None
    gelu = variant == "bias_gelu"
    # oracle: layernorm (math.cl:283) then matvec4 (math.cl:185) with its epilogue
    xin = ref_ln(x, gamma, beta) if gamma is not None else x
    want = np.zeros(N, np.float32)
    L().ref_matvec4(fp(xin), fp(W), None if bias is None else fp(bias), None if resid is None else fp(resid),
                    fp(want), N, K, int(gelu))
    ws_bytes = g2.matvec_workspace(N, K)
    ws = torch.zeros(ws_bytes // 4 + 64, dtype=torch.float32, device="cuda")
    dx, dW, dy = dev(x), dev(W), torch.zeros(N, device="cuda")
    dres = dev(resid) if resid is not None else None
    if resid is not None:
        dy.copy_(dres)   # in place: residual aliases the output, as decode does (main.c:1815)
    for rep in range(2):   # the second call reuses the workspace the first left behind
        if resid is not None:
            dy.copy_(dres)
        g2.matvec(dx, dW, dy, N, K, bias=None if bias is None else dev(bias), residual=dy if resid is not None else None,
                  gelu=gelu, ln_gamma=None if gamma is None else dev(gamma), ln_beta=None if beta is None else dev(beta),
                  workspace=ws, workspace_bytes=ws_bytes)
        close(host(dy), want)


@pytest.mark.parametrize("M", [1, 5, 64, 257])
@pytest.mark.parametrize("N,K", [(2304, 768), (768, 768), (3072, 768), (768, 3072)])
def test_matmul(g2, M, N, K):
    A, B, b = rnd(M, K), rnd(K, N, s=0.02), rnd(N, s=0.1)
    want = np.zeros((M, N), np.float32)
    L().ref_matmul(fp(A), fp(B), fp(b), fp(want), M, N, K)
    C_ = torch.zeros(M, N, device="cuda")
    g2.matmul(dev(A), dev(B), C_, M, N, K, bias=dev(b))
    close(host(C_), want)
    # fused GELU (prefill's launch_gelu, main.c:1774) and residual add (launch_add, main.c:1767)
    g_want = want.copy().reshape(-1)
    L().ref_gelu(fp(g_want), M * N)
    g2.matmul(dev(A), dev(B), C_, M, N, K, bias=dev(b), gelu=True)
    close(host(C_).reshape(-1), g_want)
    R = rnd(M, N)
    r_want = R.copy().reshape(-1)
    L().ref_add_inplace(fp(r_want), fp(want.reshape(-1).copy()), M * N)
    C_.copy_(dev(R))
    g2.matmul(dev(A), dev(B), C_, M, N, K, bias=dev(b), residual=C_)
    close(host(C_).reshape(-1), r_want)


@pytest.mark.parametrize("rows,E", [(1, 768), (64, 768), (3, 128), (2, 1600), (5, 1024)])
def test_layernorm(g2, rows, E):
    x = rnd(rows, E, s=3.0) + 0.7
    gm, bt = rnd(E, s=0.3) + 1.0, rnd(E, s=0.2)
    want = np.zeros_like(x)
    L().ref_layernorm(fp(x), fp(want), fp(gm), fp(bt), E, rows)
    out = torch.zeros(rows, E, device="cuda")
    g2.layernorm(dev(x), out, dev(gm), dev(bt), E, rows)
    close(host(out), want)


@pytest.mark.parametrize("NH,T", [(12, 1), (12, 2), (12, 63), (12, 64), (12, 65), (12, 128), (12, 1023),
                                  (12, 1024), (25, 300), (16, 512)])
def test_attention(g2, NH, T):
    DH, S = 64, 1024
    D = NH * DH
    q = rnd(D)
    kT, v = rnd(D, S), rnd(S, D)   # the reference's cache layouts (math.cl:355-357)
    scores = np.zeros((NH, S), np.float32)
    L().ref_attn_scores_1q(fp(q), fp(kT), fp(scores), 0, T, D, DH, NH, S, float(np.float32(1) / np.sqrt(np.float32(DH))))
    L().ref_attn_softmax_1q(fp(scores), T, NH, 64)
    want = np.zeros(D, np.float32)
    L().ref_attn_out_1q(fp(scores), fp(v), fp(want), T, D, DH, 0)
    # this engine's layout: [head][pos][64]
    Kh = np.ascontiguousarray(kT.reshape(NH, DH, S).transpose(0, 2, 1))
    Vh = np.ascontiguousarray(v.reshape(S, NH, DH).transpose(1, 0, 2))
    ws_bytes = g2.attention_workspace(NH, S)
    ws = torch.zeros(ws_bytes // 4 + 64, device="cuda")
    out = torch.zeros(D, device="cuda")
    for rep in range(2):
        g2.attention(dev(q), dev(Kh), dev(Vh), out, NH, S, T, ws, ws_bytes)
        close(host(out), want, rtol=2e-5)


def test_kernel_argument_errors(g2):
    x = torch.zeros(16, device="cuda")
    with pytest.raises(g2.G2Error) as ei:
        g2.matvec(x, x, x, 6, 16, workspace=x, workspace_bytes=64)   # N % 4
    assert ei.value.code == -1
    with pytest.raises(g2.G2Error):
        g2.attention(x, x, x, x, 1, 1024, 0, x, 64)                   # T_kv < 1
    with pytest.raises(g2.G2Error):
        g2.matvec(x, x, x, 16, 16, workspace=x, workspace_bytes=4)    # workspace too small
