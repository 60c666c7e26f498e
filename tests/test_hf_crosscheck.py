"""The oracle's GPT-2 against the Hugging Face implementation of GPT-2 on the same weights.

The oracle (oracle/ref_cpu.c) restates the reference's main.c / math.cl and is
pinned bit-exact to the reference's own code.  This test checks the other side:
that the arithmetic the reference performs is GPT-2's.  transformers'
GPT2LMHeadModel (tanh GELU, LayerNorm eps 1e-5, causal attention scaled by
1/sqrt(64), LM head tied to wte), loaded with the synthetic safetensors files
the engine and the oracle read, gives the same logits after a prompt and after
greedy decode steps, within fp32 summation-order differences: 1e-5 relative
to the largest logit (measured: under 1e-6; the exact-erf GELU instead of the
tanh form would differ by 4e-5).  CPU only.
"""
import json
import os

import numpy as np
import pytest

import oracle
from gpt2b200 import synth

transformers = pytest.importorskip("transformers")
torch = pytest.importorskip("torch")
st = pytest.importorskip("safetensors.numpy")

TOL = 1e-5


def rel(got, want):
    return float(np.abs(np.asarray(got, np.float64) - want).max() / np.abs(want).max())


def hf_model(d):
    cfg = json.load(open(os.path.join(d, "config.json")))
    conf = transformers.GPT2Config(
        vocab_size=cfg["vocab_size"], n_positions=cfg["n_positions"], n_embd=cfg["n_embd"],
        n_layer=cfg["n_layer"], n_head=cfg["n_head"], n_inner=cfg.get("n_inner"),
        activation_function=cfg["activation_function"], layer_norm_epsilon=cfg["layer_norm_epsilon"],
        resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0, tie_word_embeddings=True)
    m = transformers.GPT2LMHeadModel(conf).eval()
    tensors = st.load_file(os.path.join(d, "model.safetensors"))
    sd = {"transformer." + k: torch.from_numpy(np.array(v, np.float32)) for k, v in tensors.items()}
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    # the tied head and the causal-mask buffers are the only parameters not in the file
    assert all(k == "lm_head.weight" or k.endswith(".attn.bias") or k.endswith(".attn.masked_bias")
               for k in missing), missing
    m.tie_weights()
    return m


@pytest.mark.parametrize("affine", [False, True])
def test_oracle_matches_hf_gpt2(tmp_path, affine):
    d = synth.make_model(str(tmp_path / "m"), synth.TINY, seed=7, affine=affine)
    m = hf_model(d)
    ref = oracle.RefModel(d)
    prompt = [int(t) for t in synth.prompt_ids(5, 24)]
    V = synth.TINY.vocab_size
    ref.prefill(prompt)
    ids = list(prompt)
    with torch.no_grad():
        for step in range(4):
            hf = m(torch.tensor([ids])).logits[0, -1].numpy()
            got = ref.logits()[:V]
            assert rel(got, hf) <= TOL, f"step {step}"
            tok = int(np.argmax(hf))
            ref.decode(tok, len(ids))
            ids.append(tok)
    ref.close()
