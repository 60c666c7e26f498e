"""The device top-k (g2k_topk on device pointers, g2_topk on an engine slot)
against the order of the reference's first-maximum scan (main.c:1898-1904)
and the oracle's kth_largest (main.c:1839-1868).

Bit-exact: ids must equal numpy's order (decreasing value, then increasing
index: np.lexsort), values must be the logits themselves, and values[k-1]
must equal ref_kth_largest on the same array.  Edge cases: massive ties,
all-equal inputs, signed zeros (equal as floats), -inf entries inside the top
k, n = 1, k = n, k = G2_MAX_TOPK, and out-of-range k.
"""
import os

import numpy as np
import pytest

import oracle
from gpt2b200 import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

V = 50257
MAX_K = 256   # G2_MAX_TOPK (main.c:55)


@pytest.fixture(scope="module")
def g2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gpt2b200
    return gpt2b200


def want_ids(x, k):
    return np.lexsort((np.arange(len(x)), -x.astype(np.float64)))[:k]


def run(g2, x, k):
    d = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    vals = torch.empty(k, dtype=torch.float32, device="cuda")
    ids = torch.empty(k, dtype=torch.int32, device="cuda")
    g2.topk(d, len(x), k, vals, ids)
    torch.cuda.synchronize()
    return vals.cpu().numpy(), ids.cpu().numpy()


def check(g2, x, k):
    x = np.ascontiguousarray(x, np.float32)
    vals, ids = run(g2, x, k)
    want = want_ids(x, k)
    assert ids.tolist() == want.tolist()
    assert np.array_equal(vals.view(np.uint32), x[want].view(np.uint32))
    kth = oracle.cpu_lib().ref_kth_largest(oracle.fptr(x), len(x), k)
    assert vals[k - 1] == np.float32(kth)


RNG = np.random.default_rng(11)


@pytest.mark.parametrize("k", [1, 2, 3, 40, 100, 255, 256])
def test_random_logits(g2, k):
    check(g2, RNG.standard_normal(V).astype(np.float32) * 4, k)


@pytest.mark.parametrize("k", [1, 7, 64, 256])
def test_massive_ties(g2, k):
    check(g2, RNG.integers(-5, 5, size=V).astype(np.float32), k)     # ~5,000 copies of each value


def test_all_equal(g2):
    check(g2, np.full(V, 0.5, np.float32), MAX_K)


def test_signed_zeros_are_equal(g2):
    x = np.zeros(V, np.float32)
    x[::2] = -0.0
    x[[10, 2000, 40000]] = 1.0
    check(g2, x, MAX_K)   # the zeros after the three ones come in index order, whatever their sign


def test_infinities_inside_the_top_k(g2):
    x = np.full(V, -np.inf, np.float32)
    x[RNG.choice(V, 10, replace=False)] = RNG.standard_normal(10).astype(np.float32)
    check(g2, x, 40)


def test_reference_scale_logits(g2):
    # GPT-2-like: a few large logits above a dense body, as the LM head produces
    x = (RNG.standard_normal(V) * 2 - 60).astype(np.float32)
    x[RNG.choice(V, 30, replace=False)] += 25
    for k in (1, 40, 256):
        check(g2, x, k)


@pytest.mark.parametrize("n,k", [(1, 1), (5, 5), (300, 256), (1000, 17), (256, 256), (257, 256)])
def test_small_arrays(g2, n, k):
    check(g2, RNG.standard_normal(n).astype(np.float32), k)


def test_rejects_bad_k(g2):
    x = torch.zeros(100, device="cuda")
    vals = torch.empty(MAX_K + 1, device="cuda")
    ids = torch.empty(MAX_K + 1, dtype=torch.int32, device="cuda")
    for n, k in ((100, 0), (100, 101), (1000, MAX_K + 1), (0, 1)):
        with pytest.raises(g2.G2Error):
            g2.topk(x, n, k, vals, ids)


def _model():
    from conftest import MODEL_CACHE
    return synth.ensure_model(os.path.join(MODEL_CACHE, "tiny_s2"), synth.TINY, seed=2)


def test_engine_slots(g2):
    """g2_topk on the logits a prefill and a batched decode leave in each slot."""
    prompts = [synth.prompt_ids(70 + s, 11 + 4 * s) for s in range(3)]
    with g2.Engine(_model(), max_batch=3) as eng:
        with pytest.raises(g2.G2Error):   # no logits yet
            eng.topk(5, slot=1)
        toks = []
        for s, p in enumerate(prompts):
            eng.prefill(p, slot=s)
            x = eng.logits(s)[:V]
            vals, ids = eng.topk(MAX_K, slot=s)
            assert ids.tolist() == want_ids(x, MAX_K).tolist()
            assert np.array_equal(vals, x[ids])
            assert ids[0] == eng.argmax(s)[0]
            toks.append(int(ids[0]))
        slots = np.arange(3, dtype=np.int32)
        eng.decode_batch(slots, np.array(toks, np.int32), np.array([len(p) for p in prompts], np.int32))
        for s in range(3):
            x = eng.logits(s)[:V]
            vals, ids = eng.topk(40, slot=s)
            assert ids.tolist() == want_ids(x, 40).tolist()
            assert np.array_equal(vals, x[ids])
        for k in (0, MAX_K + 1):
            with pytest.raises(g2.G2Error):
                eng.topk(k, slot=0)
