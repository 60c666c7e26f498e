"""The device sampler (g2_sample_device) against the host restatement of the
reference's sample_next_token (g2_sample, main.c:1872-1939), which the CPU
tests pin to the oracle.

Both run on the same logits with the same uniform draw: the host sampler
calls the C library's rand() after srand(seed); the device sampler is given
u = rand() / (RAND_MAX + 1.0) drawn after the same srand(seed).  Tokens must
be identical -- greedy, temperature, top-k (including k above the reference's
MAX_TOPK of 256), repetition penalty over a context with repeated ids, and the
EOS mask.
"""
import ctypes

import numpy as np
import pytest

from gpt2b200 import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

libc = ctypes.CDLL("libc.so.6")
libc.rand.restype = ctypes.c_int
RAND_MAX = 2147483647   # glibc


@pytest.fixture(scope="module")
def g2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gpt2b200
    return gpt2b200


CONFIGS = [  # temperature, top_k, rep_penalty, forbid_eos
    (0.0, 40, 1.0, False), (0.0, 0, 1.3, True), (0.8, 40, 1.1, True), (1.0, 0, 1.0, False),
    (0.5, 1, 1.0, False), (1.5, 256, 1.5, False), (0.9, 300, 1.2, True), (2.0, 7, 1.0, True),
]


def test_device_sampler_matches_host(g2, tiny_affine_model):
    prompt = synth.prompt_ids(31, 24)
    ctx = list(prompt) + list(prompt[:6])        # repeated ids: the penalty applies once per id
    with g2.Engine(tiny_affine_model) as eng:
        eng.prefill(prompt)
        V = eng.cfg.vocab_size
        checked = 0
        for step in range(4):
            logits = eng.logits()[:V].copy()
            for (T, k, pen, forbid) in CONFIGS:
                for seed in (1, 2, 3):
                    libc.srand(seed)
                    want = g2.sample(logits, ctx, forbid_eos=forbid, temperature=T, top_k=k, rep_penalty=pen)
                    libc.srand(seed)
                    u = libc.rand() / (RAND_MAX + 1.0)
                    got = eng.sample_device(ctx, forbid_eos=forbid, temperature=T, top_k=k, rep_penalty=pen, u=u)
                    assert got == want, f"step {step} T={T} k={k} pen={pen} forbid={forbid} seed={seed}: {got} vs {want}"
                    checked += 1
            assert np.array_equal(eng.logits()[:V], logits)   # the slot's logits are left unchanged
            tok = int(np.argmax(logits))
            eng.decode(tok, len(prompt) + step)
            ctx.append(tok)
        assert checked == 4 * len(CONFIGS) * 3


def test_device_sampler_edges(g2, tiny_model):
    with g2.Engine(tiny_model) as eng:
        with pytest.raises(g2.G2Error):   # nothing prefilled in the slot yet
            eng.sample_device([1, 2], u=0.5)
        eng.prefill([5, 6, 7])
        V = eng.cfg.vocab_size
        logits = eng.logits()[:V]
        assert eng.sample_device([5, 6, 7], temperature=0.0) == int(np.argmax(logits))
        # top-1: any draw above 0 lands on the argmax; a draw of exactly 0 gives
        # r = 0, which the reference's `acc >= r` accepts at index 0 (main.c:1935)
        assert eng.sample_device([5, 6, 7], temperature=1.0, top_k=1, u=0.5) == int(np.argmax(logits))
        assert eng.sample_device([5, 6, 7], temperature=1.0, top_k=1, u=1e-12) == int(np.argmax(logits))
        assert eng.sample_device([5, 6, 7], temperature=1.0, top_k=1, u=0.0) == 0
        with pytest.raises(g2.G2Error):
            eng.sample_device([1], temperature=1.0, u=1.0)
        with pytest.raises(g2.G2Error):
            eng.sample_device([1], temperature=1.0, u=0.5, slot=3)
