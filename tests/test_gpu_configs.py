"""Parity at the full sizes of the other BASELINE configurations, against
golden fixtures (tests/golden/, made by tests/golden/make_golden.py).

* c3 -- GPT-2 small fp32, B = 1, a 512-token prompt, then greedy decode to
  the end of the context (512 tokens, prefill's included).  The golden stream
  comes from the reference itself (main.c + math.cl on the CPU OpenCL shim):
  the persistent decode kernel must reproduce all 512 tokens, and the logits
  at steps 0, 1, 256 and 511 within 1e-3 of max |logit|.
* c5 -- GPT-2 XL fp32, 32 sequences in one engine (the benchmark's prompts,
  sequence i seeded by i), so the tensor-core GEMMs take their 32-row plan.
  Sequences 0 and 1 must reproduce the golden greedy streams (129 tokens) of
  the restated oracle (pinned bit for bit to the reference, which cannot load
  XL past its compile-time ceilings, main.c:46-56); fed the golden tokens, the
  batched step's logits stay within 1e-3 of the golden ones at every step.
  Every other sequence must equal its own B = 1 run (the persistent kernel).
* c4 -- GPT-2 medium fp16, 32 sequences: fed the golden tokens (teacher
  forcing), sequences 0..3 stay within 2e-2 of the fp32 oracle on the same
  fp16-rounded weights at every step; their free-running streams may leave
  the golden ones only where the golden top-2 gap is within that tolerance.
  Every other sequence must equal its own run in a batch of one.

A stream that differs is reported with the step and the gap between the two
candidate tokens, so a near tie is visible, not hidden.  Where sequences are
compared with their own B = 1 runs, a divergence is accepted only at a near
tie: a gap, in the B = 1 run's own logits, within the precision's tolerance.
"""
import json
import os

import numpy as np
import pytest

from gpt2b200 import synth

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu, pytest.mark.slow]

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
FP32_TOL = 1e-3
FP16_TOL = 2e-2
V = 50257


@pytest.fixture(scope="module")
def g2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gpt2b200
    return gpt2b200


def rel(got, want):
    return float(np.abs(got.astype(np.float64) - want).max() / np.abs(want).max())


def golden(case):
    p = os.path.join(GOLD, case + ".json")
    if not os.path.exists(p):
        pytest.skip(f"fixture {case} not generated")
    meta = json.load(open(p))
    arr = dict(np.load(os.path.join(GOLD, case + ".npz")))
    d = synth.ensure_model(os.path.join(synth.default_cache(), meta["model_dir"]), getattr(synth, meta["shape"]),
                           seed=meta["model_seed"], dtype=meta["dtype"])
    return meta, arr, d


def first_diff(a, b):
    for i, (x, y) in enumerate(zip(a, b)):
        if int(x) != int(y):
            return i
    return None


def masked(lg):
    m = lg[:V].astype(np.float64).copy()
    m[50256] = -np.inf
    return m


def check_step_logits(lg, arr, si, step, st, tol):
    """Logits of sequence si at `step` against the golden ones at the per-step indices and top-8."""
    scale = st["absmax"]
    at = arr[f"s{si}_at_idx"][step]
    err = np.abs(lg[arr["idx_step"]].astype(np.float64) - at).max()
    ti, tv = arr[f"s{si}_top_i"][step], arr[f"s{si}_top_v"][step]
    err = max(err, np.abs(lg[ti].astype(np.float64) - tv).max())
    assert err <= tol * scale, f"sequence {si} step {step}: logits differ by {err / scale:.2e} of max |logit|"


def near_tie_or_fail(eng_logits_at, got, want, step, tol, what):
    """Streams `got` and `want` first differ at `step`: accept it only when the two
    tokens' logits (from eng_logits_at(step)) are within tol of max |logit|."""
    lg = masked(eng_logits_at(step))
    gap = abs(lg[int(got[step])] - lg[int(want[step])])
    scale = np.abs(lg[np.isfinite(lg)]).max()
    if gap > tol * scale:
        pytest.fail(f"{what}: streams differ at step {step} ({int(got[step])} vs {int(want[step])}) with a logit gap "
                    f"of {gap:.3e} ({gap / scale:.1e} of max |logit|): not a near tie")
    print(f"{what}: near tie at step {step}, gap {gap:.3e} ({gap / scale:.1e} of max |logit|)")


def test_c3_long_context_stream_and_logits(g2):
    meta, arr, d = golden("c3_small_s0")
    s0 = meta["seqs"][0]
    prompt = np.array(s0["prompt"], np.int32)
    want = s0["tokens"]
    with g2.Engine(d) as eng:
        assert eng.cfg.persistent == 1
        got = eng.generate(prompt, meta["n_new"])
        i = first_diff(got, want)
        if i is not None or len(got) != len(want):
            i = min(len(got), len(want)) if i is None else i
            st = s0["stats"][min(i, len(want) - 1)]
            pytest.fail(f"c3 greedy stream differs at step {i}: got {list(got[i:i + 4])} want {want[i:i + 4]}; "
                        f"reference top1 {st['top1']:.6f}, top1-top2 gap {st['gap']:.3e}")
        # logits at the recorded steps (g2_prefill / g2_decode / g2_logits)
        eng.prefill(prompt)
        n = len(prompt)
        for step in range(max(meta["logit_steps"]) + 1):
            if step > 0:
                eng.decode(want[step - 1], n + step - 1)
            if step in meta["logit_steps"]:
                lg = eng.logits()
                assert rel(lg[arr["idx"]], arr[f"s0_logits_step{step}"]) <= FP32_TOL, f"step {step}"
                assert np.all(lg[V:] == 0.0)


def _batched(g2, meta, arr, d, dtype, tol, exact_golden):
    B = 32
    nn = meta["n_new"]
    plen = meta["prompt_len"]
    prompts = [synth.prompt_ids(i, plen) for i in range(B)]
    for s in meta["seqs"]:
        assert list(prompts[s["prompt_seed"]]) == s["prompt"]
    gold = {s["prompt_seed"]: si for si, s in enumerate(meta["seqs"])}
    with g2.Engine(d, max_batch=B, dtype=dtype) as eng:
        toks = eng.generate_batch(prompts, nn)
        # (1) the golden sequences' free-running streams
        for seed, si in gold.items():
            want = meta["seqs"][si]["tokens"]
            i = first_diff(toks[seed], want)
            if i is None:
                continue
            st = meta["seqs"][si]["stats"][i]
            msg = (f"sequence {seed}: greedy stream differs at step {i} ({int(toks[seed][i])} vs {want[i]}); "
                   f"golden top1-top2 gap {st['gap']:.3e} ({st['gap'] / st['absmax']:.1e} of max |logit|)")
            if exact_golden or st["gap"] > 2 * tol * st["absmax"]:
                pytest.fail(msg)
            print(msg + " -- within the tolerance")
        # (2) teacher forcing: every slot decodes together; the golden sequences are
        # fed the golden tokens, the others their own generated tokens
        feed = [list(toks[i]) for i in range(B)]
        for seed, si in gold.items():
            feed[seed] = meta["seqs"][si]["tokens"]
        for i, p in enumerate(prompts):
            eng.prefill(p, slot=i)
        for step in range(nn):
            if step > 0:
                eng.decode_batch(list(range(B)), [feed[i][step - 1] for i in range(B)], [plen + step - 1] * B)
            for seed, si in gold.items():
                lg = eng.logits(seed)
                check_step_logits(lg, arr, si, step, meta["seqs"][si]["stats"][step], tol)
                if step in meta["logit_steps"]:
                    assert rel(lg[arr["idx"]], arr[f"s{si}_logits_step{step}"]) <= tol
                    assert np.all(lg[V:] == 0.0)
    return prompts, toks


def _b1_logits_fn(eng, prompt, tokens, run_one):
    """Logits of a B = 1 run at `step`, fed `tokens` (the common prefix)."""
    def at(step):
        run_one(prompt, tokens, step)
        return eng.logits(0)
    return at


def test_c5_xl_fp32_32_sequences(g2):
    meta, arr, d = golden("c5_xl_s0")
    prompts, toks = _batched(g2, meta, arr, d, g2.G2_F32, FP32_TOL, exact_golden=True)
    gold = {s["prompt_seed"] for s in meta["seqs"]}
    nn = meta["n_new"]
    with g2.Engine(d) as eng:   # B = 1: the persistent kernel
        assert eng.cfg.persistent == 1

        def run_one(prompt, tokens, step):
            eng.prefill(prompt)
            for s in range(1, step + 1):
                eng.decode(int(tokens[s - 1]), len(prompt) + s - 1)

        for i in range(len(prompts)):
            if i in gold:
                continue
            one = eng.generate(prompts[i], nn)
            j = first_diff(one, toks[i])
            if j is not None:
                near_tie_or_fail(_b1_logits_fn(eng, prompts[i], one, run_one), one, toks[i], j, 1e-4,
                                 f"c5 sequence {i}: 32-sequence batch vs B = 1")


def test_c4_medium_fp16_32_sequences(g2):
    meta, arr, d = golden("c4_medium_f16_s0")
    prompts, toks = _batched(g2, meta, arr, d, g2.G2_F16, FP16_TOL, exact_golden=False)
    gold = {s["prompt_seed"] for s in meta["seqs"]}
    nn = meta["n_new"]
    B = len(prompts)
    with g2.Engine(d, max_batch=B, dtype=g2.G2_F16) as eng:
        def run_one(prompt, tokens, step):
            eng.prefill(prompt, slot=0)
            for s in range(1, step + 1):
                eng.decode_batch([0], [int(tokens[s - 1])], [len(prompt) + s - 1])

        for i in range(B):
            if i in gold:
                continue
            one = eng.generate_batch([prompts[i]], nn, slots=[i])[0]
            j = first_diff(one, toks[i])
            if j is not None:
                near_tie_or_fail(_b1_logits_fn(eng, prompts[i], one, run_one), one, toks[i], j, FP16_TOL,
                                 f"c4 sequence {i}: 32-sequence batch vs a batch of one")
