"""Pin the restated oracle (oracle/ref_cpu.c) to the reference's own code.

The reference has no tests, golden vectors or fixtures of its own.  These
tests run its math.cl kernels and its main.c prefill/decode/sampler,
compiled from the reference sources onto a CPU OpenCL shim
(oracle/_ref/libref_main.so), and require the restatement to match them bit
for bit on the same inputs.  Skipped where oracle/_ref was not built.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built (reference sources absent)")

RNG = np.random.default_rng(1234)


def rnd(*shape, scale=1.0):
    return (RNG.standard_normal(shape, dtype=np.float32) * np.float32(scale)).astype(np.float32)


def bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


L = None


def lib():
    global L
    if L is None:
        L = oracle.cpu_lib()
    return L


fp = oracle.fptr


@pytest.mark.parametrize("N,K,gelu,bias,res", [(2304, 768, 0, 1, 0), (3072, 768, 1, 1, 0), (768, 768, 0, 1, 1),
                                               (52, 37, 1, 0, 1), (8, 5, 0, 0, 0)])
def test_matvec4(N, K, gelu, bias, res):
    A, B = rnd(K), rnd(K, N, scale=0.02)
    b = rnd(N) if bias else None
    r = rnd(N) if res else None
    C1 = np.zeros(N, np.float32)
    C2 = np.zeros(N, np.float32)
    oracle.run_ref_kernel("matvec4", [((N // 4 + 63) // 64) * 64], [64], [A, B, b, r, C1, N, K, gelu])
    lib().ref_matvec4(fp(A), fp(B), None if b is None else fp(b), None if r is None else fp(r), fp(C2), N, K, gelu)
    assert bits_equal(C1, C2)


@pytest.mark.parametrize("N,K", [(13, 9), (7, 64)])
def test_matvec_scalar(N, K):
    A, B, b, r = rnd(K), rnd(K, N), rnd(N), rnd(N)
    C1 = np.zeros(N, np.float32)
    C2 = np.zeros(N, np.float32)
    oracle.run_ref_kernel("matvec", [64], [64], [A, B, b, r, C1, N, K, 1])
    lib().ref_matvec(fp(A), fp(B), fp(b), fp(r), fp(C2), N, K, 1)
    assert bits_equal(C1, C2)


@pytest.mark.parametrize("N,K,ks", [(768, 768, 8), (768, 3072, 8), (3072, 768, 4), (2304, 768, 2), (16, 13, 3)])
def test_splitk(N, K, ks):
    A, B, b, r = rnd(K), rnd(K, N, scale=0.02), rnd(N), rnd(N)
    P = np.zeros(8 * N, np.float32)
    C1 = r.copy()
    n4 = N // 4
    oracle.run_ref_kernel("matvec4_sk", [((n4 + 127) // 128) * 128, ks], [128, 1], [A, B, P, N, K, ks])
    oracle.run_ref_kernel("reduce_partial", [((n4 + 63) // 64) * 64], [64], [P, b, C1, C1, N, ks, 0])
    C2 = r.copy()
    P2 = np.zeros(8 * N, np.float32)
    lib().ref_launch_matvec_splitk(fp(A), fp(B), fp(b), fp(C2), fp(C2), N, K, ks, 0, fp(P2))
    assert bits_equal(C1, C2)


@pytest.mark.parametrize("rows,E", [(1, 768), (5, 128), (3, 1600)])
def test_layernorm(rows, E):
    x, g, b = rnd(rows, E, scale=3.0) + 0.5, rnd(E), rnd(E)
    o1 = np.zeros((rows, E), np.float32)
    o2 = np.zeros((rows, E), np.float32)
    oracle.run_ref_kernel("layernorm", [64], [64], [x, o1, g, b, E, rows])
    lib().ref_layernorm(fp(x), fp(o2), fp(g), fp(b), E, rows)
    assert bits_equal(o1, o2)


def test_gelu_add_embed():
    x = rnd(1000, scale=4.0)
    y1, y2 = x.copy(), x.copy()
    oracle.run_ref_kernel("gelu", [1024], [64], [y1, 1000])
    lib().ref_gelu(fp(y2), 1000)
    assert bits_equal(y1, y2)
    a1, a2, b = x.copy(), x.copy(), rnd(1000)
    oracle.run_ref_kernel("add_inplace", [1024], [64], [a1, b, 1000])
    lib().ref_add_inplace(fp(a2), fp(b), 1000)
    assert bits_equal(a1, a2)
    wte, wpe = rnd(50, 64), rnd(40, 64)
    ids = np.array([3, 49, 0, 7], np.int32)
    o1 = np.zeros((4, 64), np.float32)
    o2 = np.zeros((4, 64), np.float32)
    oracle.run_ref_kernel("embed", [64, 4], [16, 1], [wte, wpe, o1, 64, 4, 5, ids])
    lib().ref_embed(fp(wte), fp(wpe), fp(o2), 64, 4, 5, oracle.iptr(ids))
    assert bits_equal(o1, o2)


@pytest.mark.parametrize("T_kv,NH,lws", [(1, 12, 64), (63, 12, 64), (65, 2, 64), (1024, 12, 64), (300, 25, 128)])
def test_attention_kernels(T_kv, NH, lws):
    DH, S = 64, 1024
    D = NH * DH
    qkv = rnd(3 * D)
    kc, vc = rnd(D, S), rnd(S, D)
    scale = np.float32(1.0) / np.sqrt(np.float32(DH))
    s1 = np.zeros((NH, S), np.float32)
    s2 = np.zeros((NH, S), np.float32)
    n = ((NH * T_kv + 63) // 64) * 64
    oracle.run_ref_kernel("attn_scores_1q", [n], [64], [qkv, kc, s1, 0, T_kv, D, DH, NH, S, float(scale)])
    lib().ref_attn_scores_1q(fp(qkv), fp(kc), fp(s2), 0, T_kv, D, DH, NH, S, float(scale))
    assert bits_equal(s1, s2)
    oracle.run_ref_kernel("attn_softmax_1q", [NH * lws], [lws], [s1, T_kv])
    lib().ref_attn_softmax_1q(fp(s2), T_kv, NH, lws)
    assert bits_equal(s1, s2)
    o1 = np.zeros(D, np.float32)
    o2 = np.zeros(D, np.float32)
    oracle.run_ref_kernel("attn_out_1q", [((D + 63) // 64) * 64], [64], [s1, vc, o1, T_kv, D, DH, 0])
    lib().ref_attn_out_1q(fp(s2), fp(vc), fp(o2), T_kv, D, DH, 0)
    assert bits_equal(o1, o2)


def test_split_kv():
    D, S, T = 128, 1024, 5
    qkv = rnd(T, 3 * D)
    k1, v1, k2, v2 = (np.zeros((D, S), np.float32), np.zeros((S, D), np.float32),
                      np.zeros((D, S), np.float32), np.zeros((S, D), np.float32))
    oracle.run_ref_kernel("split_kv", [((T * D + 63) // 64) * 64], [64], [qkv, k1, v1, 7, T, D, S])
    lib().ref_split_kv(fp(qkv), fp(k2), fp(v2), 7, T, D, S)
    assert bits_equal(k1, k2) and bits_equal(v1, v2)


@pytest.mark.parametrize("M,N,K", [(5, 72, 40), (64, 128, 96)])
def test_generated_matmul(M, N, K):
    """main.c's runtime-built matmul (tile 64x64x16/4x4) against the serial-k restatement."""
    A, B, b = rnd(M, K), rnd(K, N, scale=0.1), rnd(N)
    C1 = np.zeros((M, N), np.float32)
    C2 = np.zeros((M, N), np.float32)
    gws = [((N + 63) // 64) * 16, ((M + 63) // 64) * 16]
    oracle.run_ref_kernel("matmul", gws, [16, 16], [A, B, b, C1, M, N, K, 0], program_kind=1)
    lib().ref_matmul(fp(A), fp(B), fp(b), fp(C2), M, N, K)
    assert bits_equal(C1, C2)


def test_kth_largest_and_sampler():
    R = oracle.ref_lib()
    x = rnd(50257, scale=2.0)
    for k in (1, 40, 256):
        assert R.refmain_kth_largest(fp(x), 50257, k) == lib().ref_kth_largest(fp(x), 50257, k)


@pytest.fixture(scope="module")
def ref_pair(tiny_affine_model):
    main = oracle.RefMain(tiny_affine_model)
    cpu = oracle.RefModel(tiny_affine_model)
    yield main, cpu
    cpu.close()
    main.close()


def test_prefill_decode_bit_exact(ref_pair):
    """Whole forward passes of main.c (prefill, decode) against the restatement."""
    from gpt2b200 import synth
    main, cpu = ref_pair
    ids = synth.prompt_ids(3, 20)
    main.prefill(ids)
    cpu.prefill(ids)
    assert bits_equal(main.logits(), cpu.logits())
    tok = int(np.argmax(cpu.logits()[:50257]))
    for step in range(6):
        main.decode(tok, 20 + step)
        cpu.decode(tok, 20 + step)
        lm, lc = main.logits(), cpu.logits()
        assert bits_equal(lm, lc), f"step {step}"
        tok = int(np.argmax(lc[:50257]))
    for layer in range(2):
        km, vm = main.kv(layer)
        kc, vc = cpu.kv(layer)
        assert bits_equal(km, kc) and bits_equal(vm, vc)


def test_sampler_stream_matches_reference(ref_pair):
    """Greedy and stochastic (T, top-k, repetition penalty, rand()) streams."""
    from gpt2b200 import synth
    main, cpu = ref_pair
    prompt = synth.prompt_ids(4, 12)
    g_main = main.generate(prompt, 12)
    g_cpu = cpu.generate(prompt, 12)
    assert np.array_equal(g_main, g_cpu)
    oracle.ref_lib().refmain_srand(77)
    s_main = main.generate(prompt, 10, min_new=1, temperature=0.8, top_k=40, rep_penalty=1.1)
    lib().ref_srand(77)
    s_cpu = cpu.generate(prompt, 10, min_new=1, temperature=0.8, top_k=40, rep_penalty=1.1)
    assert np.array_equal(s_main, s_cpu)
