"""Parity at the sizes of the batched configurations (BASELINE configs c4, c5).

* c4's model: GPT-2 medium, fp16 weights; three sequences of different prompt
  lengths prefilled and decoded together (the batched path: tensor-core GEMMs
  with fp16 operands).  The oracle runs in fp32 on the same fp16-rounded
  weights; logits within 2e-2 of max |ref| at every step (the fp16 bar).
* c5's model: GPT-2 XL, fp32 (3xTF32 tensor-core GEMMs in prefill and the
  batched step); logits within 1e-3 of max |ref| (the fp32 bar) after prefill
  and for three decode steps, on two sequences.

The oracle's greedy token is fed back at every step (teacher forcing), so a
near tie cannot make the two sides diverge.
"""
import os

import numpy as np
import pytest

import oracle
from gpt2b200 import synth

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu, pytest.mark.slow]


@pytest.fixture(scope="module")
def g2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gpt2b200
    return gpt2b200


def rel(got, want):
    return float(np.abs(got.astype(np.float64) - want).max() / np.abs(want).max())


def model(name, shape, dtype):
    from conftest import MODEL_CACHE
    return synth.ensure_model(os.path.join(MODEL_CACHE, name), shape, seed=0, dtype=dtype)


def run_batched(g2, d, dtype, lens, steps, tol):
    V = 50257
    prompts = [synth.prompt_ids(300 + i, n) for i, n in enumerate(lens)]
    refs = [oracle.RefModel(d) for _ in prompts]
    with g2.Engine(d, max_batch=len(prompts), dtype=dtype) as eng:
        toks = []
        for i, (p, ref) in enumerate(zip(prompts, refs)):
            ref.prefill(p)
            eng.prefill(p, slot=i)
            assert rel(eng.logits(i), ref.logits()) <= tol, f"prefill of sequence {i}"
            toks.append(int(np.argmax(ref.logits()[:V])))
        for step in range(steps):
            pos = [n + step for n in lens]
            for ref, t, q in zip(refs, toks, pos):
                ref.decode(t, q)
            eng.decode_batch(list(range(len(prompts))), toks, pos)
            for i, ref in enumerate(refs):
                want = ref.logits()
                assert rel(eng.logits(i), want) <= tol, f"step {step} sequence {i}"
                toks[i] = int(np.argmax(want[:V]))
    for ref in refs:
        ref.close()


def test_medium_fp16_batched_vs_oracle(g2):
    d = model("cfg_medium_f16_s0", synth.MEDIUM, "f16")
    run_batched(g2, d, g2.G2_F16, [16, 40, 70], 4, 2e-2)


def test_xl_fp32_batched_vs_oracle(g2):
    d = model("cfg_xl_f32_s0", synth.XL, "f32")
    run_batched(g2, d, g2.G2_F32, [24, 9], 3, 1e-3)
