"""The bounds-checked build (-DG2_CHECK) on the GPU.

In that build every data-dependent index a kernel is about to use (token ids,
positions, slots, key counts) is tested first; a failure is recorded and
reported by the next synchronising call as G2_ERR_RANGE, in place of a device
assert (compute-sanitizer is not available on this pool).  These runs drive
the main paths -- persistent B = 1 decode (whole-head and split attention),
tiled prefill attention, batched decode on the tensor cores, fp16 -- through
that build in a child process (the library is mapped once per process) and
require the oracle's results with no bounds failure reported.
"""
import os
import subprocess
import sys
import textwrap

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "gpt2-opencl-1.1_b200", "libgpt2b200_check.so")

SCRIPT = textwrap.dedent('''
    import os, sys, tempfile
    import numpy as np
    sys.path[:0] = [os.path.join(ROOT, "gpt2-opencl-1.1_b200"), os.path.join(ROOT, "oracle")]
    import gpt2b200 as g2, oracle
    from gpt2b200 import synth
    assert g2.LIB_PATH.endswith("libgpt2b200_check.so"), g2.LIB_PATH
    d = synth.ensure_model(os.path.join(synth.default_cache(), "tiny_affine_s1"), synth.TINY, seed=1, affine=True)
    ref = oracle.RefModel(d)
    p1 = synth.prompt_ids(61, 40)
    p2 = synth.prompt_ids(62, 400)
    with g2.Engine(d, max_batch=3) as eng:
        assert eng.cfg.persistent == 1
        assert list(eng.generate(p1, 30)) == list(ref.generate(p1, 30))            # whole-head attention
        assert list(eng.generate(p2, 20, slot=1)) == list(ref.generate(p2, 20))    # split keys, tiled prefill
        bp = [p2[:64], p2[:128], p2[200:328]]                                       # whole 64-row tiles:
        want = [list(ref.generate(p, 12)) for p in bp]
        got = eng.generate_batch(bp, 12)                                            # grouped prefill, batched decode
        assert [list(x) for x in got] == want
        eng.synchronize()
    f = synth.ensure_model(os.path.join(synth.default_cache(), "tiny_f16_s4"), synth.TINY, seed=4, affine=True, dtype="f16")
    ref16 = oracle.RefModel(f)
    ref16.prefill(p2)
    with g2.Engine(f, dtype=g2.G2_F16) as eng:
        eng.prefill(p2)
        lg = eng.logits()
        want = ref16.logits()
        assert float(np.abs(lg - want).max() / np.abs(want).max()) <= 2e-2
        eng.synchronize()
    print("checked build ok")
''')


def test_checked_build_parity():
    if not os.path.exists(LIB):
        pytest.skip("checked build not made (make -C gpt2-opencl-1.1_b200 check)")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    env = dict(os.environ, G2_LIB=LIB)
    r = subprocess.run([sys.executable, "-c", "ROOT = %r\n" % ROOT + SCRIPT], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "checked build ok" in r.stdout
