"""g2k_matvec_noalloc: the GEMV entry point for callers that cannot allocate.

Some hosts of this library -- an FFI binding with no device allocator of its
own, an application whose device memory is fully owned by another
allocator, a path that must not take cudaMalloc's implicit device
synchronisation -- cannot provide g2k_matvec's workspace.
g2k_matvec_noalloc uses a fixed scratch array inside the library instead.

These tests call it through the C ABI and require its output to equal
g2k_matvec's (same kernel and split-K plan, so within the kernel tests'
tolerance and in practice bit for bit), on two calls in a row, since every
call reuses the scratch the previous call left behind.  One shape is also
checked directly against the oracle's launch_matvec_splitk restatement
(main.c:1578, math.cl:229-270), so the entry point is pinned on its own.
The file is named to be collected last; it passes alone in a fresh process
and after the rest.
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


def close(a, b):
    err = np.abs(a.astype(np.float64) - b).max()
    assert err <= RTOL * np.abs(b).max(), f"rel err {err / np.abs(b).max():.2e}"


@pytest.mark.parametrize("N,K,variant", [(2304, 768, "ln_bias"), (768, 768, "bias_resid"), (3072, 768, "bias_gelu"),
                                         (768, 3072, "bias_resid"), (64, 16, "plain")])
def test_noalloc_matches_workspace_entry(g2, N, K, variant):
    rng = np.random.default_rng(N + K)
    x = torch.from_numpy(rng.standard_normal(K).astype(np.float32) * 2).cuda()
    W = torch.from_numpy(rng.standard_normal((K, N)).astype(np.float32) * 0.02).cuda()
    bias = torch.from_numpy(rng.standard_normal(N).astype(np.float32) * 0.1).cuda() if variant != "plain" else None
    g = torch.from_numpy(1 + 0.2 * rng.standard_normal(K).astype(np.float32)).cuda() if variant == "ln_bias" else None
    b = torch.from_numpy(0.1 * rng.standard_normal(K).astype(np.float32)).cuda() if variant == "ln_bias" else None
    res0 = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).cuda()
    gelu = variant == "bias_gelu"
    resid = variant == "bias_resid"

    ws_bytes = g2.matvec_workspace(N, K)
    ws = torch.zeros(ws_bytes // 4 + 64, device="cuda")
    y_ref = res0.clone()
    g2.matvec(x, W, y_ref, N, K, bias=bias, residual=y_ref if resid else None, gelu=gelu, ln_gamma=g, ln_beta=b,
              workspace=ws, workspace_bytes=ws_bytes)
    torch.cuda.synchronize()
    want = y_ref.cpu().numpy()
    for call in range(2):
        y = res0.clone()
        g2.matvec_noalloc(x, W, y, N, K, bias=bias, residual=y if resid else None, gelu=gelu, ln_gamma=g, ln_beta=b)
        torch.cuda.synchronize()
        close(y.cpu().numpy(), want)


def test_noalloc_rejects_oversized_scratch(g2):
    """A shape whose split-K scratch exceeds the fixed 256 KiB is refused with G2_ERR_RANGE."""
    N, K = 49152, 1024      # 768 column tiles x 16 k-slices would not fit
    # find a shape the fixed array cannot hold according to the workspace query
    while g2.matvec_workspace(N, K) <= 256 * 1024:
        N *= 2
    x = torch.zeros(K, device="cuda")
    y = torch.zeros(N, device="cuda")
    with pytest.raises(g2.G2Error) as ei:
        g2.matvec_noalloc(x, x, y, N, K)
    assert ei.value.code == -6 and "256 KiB" in str(ei.value)


def test_noalloc_matches_oracle(g2):
    """attn_proj's shape (768 x 768, split-K 8 in the reference) with bias and an
    in-place residual, against the oracle's split-K matvec + reduce_partial."""
    N, K, ks = 768, 768, 8
    rng = np.random.default_rng(7)
    x = rng.standard_normal(K).astype(np.float32) * 2
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    res = rng.standard_normal(N).astype(np.float32)
    want = res.copy()
    scratch = np.zeros(ks * N, np.float32)
    fp = oracle.fptr
    oracle.cpu_lib().ref_launch_matvec_splitk(fp(x), fp(W), fp(bias), fp(res), fp(want), N, K, ks, 0, fp(scratch))
    dx, dW, db = (torch.from_numpy(a).cuda() for a in (x, W, bias))
    for call in range(2):
        y = torch.from_numpy(res).cuda()
        g2.matvec_noalloc(dx, dW, y, N, K, bias=db, residual=y)
        torch.cuda.synchronize()
        close(y.cpu().numpy(), want)


def test_noalloc_rejects_oversized_shared_memory(g2):
    """A very wide N with a long K: the split-K scratch fits the fixed array, but one
    column tile's K slice would not fit a CTA's 48 KB of shared memory.  The call is
    refused with G2_ERR_RANGE before any launch (the buffers are full-size all the
    same, so no read could leave them)."""
    N, K = 40000, 12288
    assert g2.matvec_workspace(N, K) <= 256 * 1024
    x = torch.zeros(K, device="cuda")
    W = torch.zeros(K * N, device="cuda")
    y = torch.zeros(N, device="cuda")
    with pytest.raises(g2.G2Error) as ei:
        g2.matvec_noalloc(x, W, y, N, K)
    assert ei.value.code == -6 and "shared memory" in str(ei.value)
    del W
    torch.cuda.empty_cache()
