"""The restatement pinned to the reference at full size: GPT-2 small (the
benchmark's model), the reference's own main.c + math.cl (oracle/_ref, barrier
kernels on fibers) against oracle/ref_cpu.c, bit for bit -- logits after
prefill and after decode steps, and the K/V caches of the first and last
layers.  CPU only."""
import numpy as np
import pytest

import oracle

pytestmark = [pytest.mark.slow,
              pytest.mark.skipif(not (oracle.ref_available() and oracle.ref_fast()),
                                 reason="oracle/_ref with the fiber executor not built")]


def bits_equal(a, b):
    return np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


def test_small_prefill_decode_bit_exact(small_model):
    from gpt2b200 import synth
    main = oracle.RefMain(small_model)
    cpu = oracle.RefModel(small_model)
    try:
        ids = synth.prompt_ids(8, 32)
        main.prefill(ids)
        cpu.prefill(ids)
        assert bits_equal(main.logits(), cpu.logits())
        tok = int(np.argmax(cpu.logits()[:50257]))
        for step in range(3):
            main.decode(tok, 32 + step)
            cpu.decode(tok, 32 + step)
            assert bits_equal(main.logits(), cpu.logits()), f"step {step}"
            tok = int(np.argmax(cpu.logits()[:50257]))
        for layer in (0, 11):
            km, vm = main.kv(layer)
            kc, vc = cpu.kv(layer)
            assert bits_equal(km, kc) and bits_equal(vm, vc), f"layer {layer}"
    finally:
        cpu.close()
        main.close()
