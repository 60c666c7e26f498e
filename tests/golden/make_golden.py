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

Cases listed in PORT_CASES are made by the restated oracle alone, which is
pinned bit for bit to the reference by tests/test_oracle_pin*.py: GPT-2 XL
is past the reference's compile-time ceilings (main.c:46-56), and the fp16
medium model is outside its F32-only loader (main.c:1213), so for those the
restatement runs in fp32 on the file's values.

The batched cases (c4, c5: several sequences, named by their prompt seeds,
which are the benchmark's sequence indices) also record, at every step, the
logits at 128 fixed indices and the 8 largest logits with their indices, so
that a GPU run fed the same tokens (teacher forcing) can be compared at every
step.  The c3..c5 cases use the benchmark's own model directories.

Usage: python tests/golden/make_golden.py [case ...]   (needs a prebuilt
oracle/_ref, or the reference sources to build it, for the reference cases).
Each case runs in its own process because the reference keeps one model in
global state.
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
# Cases at the other benchmark configurations, in the benchmark's model directories:
# name: (shape, dtype, model dir, prompt seeds, prompt length, tokens to generate, logit steps)
BIG_CASES = {
    "c3_small_s0": ("SMALL", "f32", "small_f32_s0", (0,), 512, 512, (0, 1, 256, 511)),
    "c4_medium_f16_s0": ("MEDIUM", "f16", "medium_f16_s0", (0, 1, 2, 3), 256, 129, (0, 128)),
    "c5_xl_s0": ("XL", "f32", "xl_f32_s0", (0, 1), 128, 129, (0, 128)),
}
PORT_CASES = {"c4_medium_f16_s0", "c5_xl_s0"}   # made by the restatement alone (see above)
EVERY_STEP = {"c4_medium_f16_s0", "c5_xl_s0"}   # per-step logits recorded
N_IDX = 1024
N_IDX_STEP = 128
TOPK_STEP = 8
LOGIT_STEPS = (0, 1, 32)


def model_dir(name):
    from gpt2b200 import synth
    return os.path.join(synth.default_cache(), "golden_" + name)


def run_big_case(name):
    """A BIG_CASES entry: each sequence prefilled and decoded greedily (EOS masked)."""
    import oracle
    from gpt2b200 import synth
    shape, dtype, mdir, seeds, plen, n_new, lsteps = BIG_CASES[name]
    d = synth.ensure_model(os.path.join(synth.default_cache(), mdir), getattr(synth, shape), seed=0, dtype=dtype)
    port = name in PORT_CASES
    cpu = oracle.RefModel(d)
    V, Vp = cpu.cfg.vocab_size, cpu.cfg.padded_vocab
    idx = np.sort(np.random.default_rng(99).choice(V, N_IDX, replace=False)).astype(np.int64)
    idx_s = np.sort(np.random.default_rng(98).choice(V, N_IDX_STEP, replace=False)).astype(np.int64)
    seqs, saved = [], {"idx": idx, "idx_step": idx_s}
    for si, pseed in enumerate(seeds):
        prompt = synth.prompt_ids(pseed, plen)
        ref = None if port else oracle.RefMain(d)
        seq = cpu.new_seq()
        ids = [int(t) for t in prompt]
        tokens, stats = [], []
        at_idx = np.zeros((n_new, N_IDX_STEP), np.float32)
        top_i = np.zeros((n_new, TOPK_STEP), np.int32)
        top_v = np.zeros((n_new, TOPK_STEP), np.float32)
        for step in range(n_new):
            if step == 0:
                cpu.prefill(np.array(ids, np.int32), seq=seq)
                if ref:
                    ref.prefill(np.array(ids, np.int32))
            else:
                cpu.decode(ids[-1], len(ids) - 1, seq=seq)
                if ref:
                    ref.decode(ids[-1], len(ids) - 1)
            lg = cpu.logits(seq=seq)
            if ref:
                assert np.array_equal(lg.view(np.uint32), ref.logits().view(np.uint32)), \
                    f"{name}: restatement differs from the reference at step {step}"
            tok = oracle.sample(lg, V, np.array(ids, np.int32), True, 0.0, 40, 1.0)
            l64 = lg[:V].astype(np.float64)
            masked = lg[:V].copy()
            masked[50256] = -np.inf
            order = np.argsort(-masked, kind="stable")[:TOPK_STEP]
            assert order[0] == tok
            stats.append({"sum": float(l64.sum()), "sumsq": float((l64 * l64).sum()), "top1": float(masked[order[0]]),
                          "gap": float(masked[order[0]] - masked[order[1]]), "argmax": int(tok),
                          "absmax": float(np.abs(l64).max())})
            if name in EVERY_STEP:
                at_idx[step] = lg[idx_s]
                top_i[step] = order
                top_v[step] = masked[order]
            if step in lsteps:
                saved[f"s{si}_logits_step{step}"] = lg[idx]
                saved[f"s{si}_pad_step{step}"] = lg[V:Vp]
            tokens.append(tok)
            ids.append(tok)
        if name in EVERY_STEP:
            saved[f"s{si}_at_idx"] = at_idx
            saved[f"s{si}_top_i"] = top_i
            saved[f"s{si}_top_v"] = top_v
        if ref:
            ref.close()
        cpu.L.ref_seq_free(seq)
        seqs.append({"prompt_seed": pseed, "prompt": [int(t) for t in prompt], "tokens": tokens, "stats": stats})
        print(f"{name} seq {pseed}: {n_new} tokens, min gap {min(s['gap'] for s in stats):.3e}", flush=True)
    cpu.close()
    meta = {"case": name, "shape": shape, "dtype": dtype, "model_dir": mdir, "model_seed": 0, "prompt_len": plen,
            "n_new": n_new, "logit_steps": list(lsteps), "every_step": name in EVERY_STEP, "seqs": seqs,
            "tuning": {"ks_attn_proj": 8, "ks_ffn2": 8, "attn_lws": 64},
            "source": ("restated oracle (oracle/ref_cpu.c) in fp32 on the file's values, pinned bit for bit to the "
                       "reference by tests/test_oracle_pin*.py" if port else
                       "reference main.c + math.cl on the CPU OpenCL shim (oracle/_ref), equal bit for bit to the "
                       "restated oracle at every step")}
    with open(os.path.join(HERE, name + ".json"), "w") as f:
        json.dump(meta, f)
    np.savez(os.path.join(HERE, name + ".npz"), **saved)


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
    names = sys.argv[1:] or list(CASES) + list(BIG_CASES)
    if len(names) == 1:
        (run_big_case if names[0] in BIG_CASES else run_case)(names[0])
    else:
        for n in names:
            subprocess.run([sys.executable, __file__, n], check=True)
