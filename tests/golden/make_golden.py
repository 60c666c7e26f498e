"""Generate the golden fixtures in this directory from the reference itself.

Runs the reference's own main.c + math.cl (oracle/_ref/libref_main.so, built
from the reference sources by oracle/Makefile onto a CPU OpenCL shim) on
seeded synthetic models and records, per case:

* the greedy token stream (main.c:2106-2150 with --greedy, --rep-penalty 1,
  EOS masked for every step as --min-tokens = --max-tokens),
* per-step logit statistics (float64 sum and sum of squares, top-1 value and
  index, top-1/top-2 gap),
* logits at a few steps, at fixed indices, to full float32 precision.

It also replays each case through the restated oracle (oracle/ref_cpu.c)
and refuses to write a fixture unless the two agree bit for bit.

Cases listed in PORT_CASES would be made by the restated oracle alone (for
shapes too slow for the reference build); none are, since the shim runs the
reference's barrier kernels on fibers.

Usage: python tests/golden/make_golden.py [case ...]   (needs /root/reference
or a prebuilt oracle/_ref).  Each case runs in its own process because the
reference keeps one model in global state.
"""
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "gpt2-opencl-1.1_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

CASES = {
    # name: (shape, model seed, affine, prompt seed, prompt length, tokens to generate)
    "tiny_affine_s1": ("TINY", 1, True, 5, 16, 33),
    "c1_small_s0": ("SMALL", 0, False, 0, 64, 129),
}
PORT_CASES = set()   # cases made by the restatement alone (none: the fiber executor runs every case)
N_IDX = 1024
LOGIT_STEPS = (0, 1, 32)


def model_dir(name):
    return os.path.join(os.environ.get("G2_MODEL_CACHE", os.path.join(ROOT, "_work", "models")), "golden_" + name)


def run_case(name):
    import oracle
    from gpt2b200 import synth
    shape, mseed, affine, pseed, plen, n_new = CASES[name]
    d = synth.ensure_model(model_dir(name), getattr(synth, shape), seed=mseed, affine=affine)
    prompt = synth.prompt_ids(pseed, plen)
    port = name in PORT_CASES
    cpu = oracle.RefModel(d)
    ref = cpu if port else oracle.RefMain(d)
    V, Vp = cpu.cfg.vocab_size, cpu.cfg.padded_vocab
    idx = np.sort(np.random.default_rng(99).choice(V, N_IDX, replace=False)).astype(np.int64)
    ids = [int(t) for t in prompt]
    tokens, stats, saved = [], [], {}
    for step in range(n_new):
        if step == 0:
            if not port:
                ref.prefill(np.array(ids, np.int32))
            cpu.prefill(np.array(ids, np.int32))
        else:
            if not port:
                ref.decode(ids[-1], len(ids) - 1)
            cpu.decode(ids[-1], len(ids) - 1)
        lg = ref.logits()
        if not port:
            assert np.array_equal(lg.view(np.uint32), cpu.logits().view(np.uint32)), f"restatement differs at step {step}"
            tok = ref.sample(np.array(ids, np.int32), True, 0.0, 40, 1.0)
        else:
            tok = oracle.sample(lg, V, np.array(ids, np.int32), True, 0.0, 40, 1.0)
        l64 = lg[:V].astype(np.float64)
        masked = lg[:V].copy()
        masked[50256 if V > 50256 else 0] = -np.inf if V > 50256 else masked[0]
        top2 = np.sort(masked)[-2:]
        stats.append({"sum": float(l64.sum()), "sumsq": float((l64 * l64).sum()), "top1": float(top2[1]),
                      "gap": float(top2[1] - top2[0]), "argmax": int(tok)})
        if step in LOGIT_STEPS:
            saved[f"logits_step{step}"] = lg[idx]
            saved[f"pad_step{step}"] = lg[V:Vp]
        tokens.append(tok)
        ids.append(tok)
    if not port:
        ref.close()
    cpu.close()
    meta = {"case": name, "shape": shape, "model_seed": mseed, "affine": affine, "prompt_seed": pseed,
            "prompt_len": plen, "n_new": n_new, "prompt": [int(t) for t in prompt], "tokens": tokens,
            "stats": stats, "logit_steps": list(LOGIT_STEPS), "tuning": {"ks_attn_proj": 8, "ks_ffn2": 8,
                                                                        "attn_lws": 64},
            "source": ("restated oracle (oracle/ref_cpu.c), pinned bit for bit to the reference by "
                       "tests/test_oracle_pin.py" if port else
                       "reference main.c + math.cl on the CPU OpenCL shim (oracle/_ref)")}
    with open(os.path.join(HERE, name + ".json"), "w") as f:
        json.dump(meta, f)
    np.savez(os.path.join(HERE, name + ".npz"), idx=idx, **saved)
    print(f"{name}: {n_new} tokens, min gap {min(s['gap'] for s in stats):.3e}")


if __name__ == "__main__":
    names = sys.argv[1:] or list(CASES)
    if len(names) == 1:
        run_case(names[0])
    else:
        for n in names:
            subprocess.run([sys.executable, __file__, n], check=True)
