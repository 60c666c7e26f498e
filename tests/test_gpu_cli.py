"""gpt2b200-cli end to end on the GPU: prompt text -> tokens -> generation ->
text.  Greedy output must be the oracle's greedy stream decoded with the
reference tokenizer's rules; stochastic output must not depend on where the
sampling runs (device sampler vs --host-sampler draw the same rand() stream)."""
import os
import shutil
import subprocess

import numpy as np
import pytest

import oracle
from gpt2b200 import Tokenizer, synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "gpt2-opencl-1.1_b200", "gpt2b200-cli")
TOK = os.path.join(ROOT, "tests", "golden", "tok")


@pytest.fixture(scope="module")
def model_dir(tiny_affine_model, tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d = tmp_path_factory.mktemp("cli_model")
    for f in ("config.json", "model.safetensors"):
        os.symlink(os.path.join(tiny_affine_model, f), d / f)
    for f in ("vocab.json", "merges.txt"):
        shutil.copy(os.path.join(TOK, f), d / f)
    return str(d)


def generated_text(stdout: str) -> str:
    lines = stdout.split("\n")
    i = next(k for k, l in enumerate(lines) if l.startswith("Tokenizer:"))
    j = next(k for k in range(i + 1, len(lines)) if lines[k].startswith("["))
    return "\n".join(lines[i + 1:j])


def test_cli_greedy_matches_oracle(model_dir):
    prompt = "kato rimu nesa, lovi's pedu"
    n = 12
    r = subprocess.run([CLI, "--model", model_dir, "--greedy", "--rep-penalty", "1.0", "--max-tokens", str(n),
                        "--min-tokens", str(n), "--prompt", prompt], capture_output=True, timeout=300)
    assert r.returncode == 0, r.stderr
    tk = Tokenizer(model_dir)
    ids = tk.encode(prompt)
    ref = oracle.RefModel(model_dir)
    want = ref.generate(np.array(ids, np.int32), n)
    ref.close()
    out = generated_text(r.stdout.decode("latin-1"))
    assert out.encode("latin-1") == tk.decode([t for t in want if t != 50256])


def test_cli_device_and_host_sampling_agree(model_dir):
    outs = []
    for extra in ([], ["--host-sampler"]):
        r = subprocess.run([CLI, "--model", model_dir, "--temperature", "0.9", "--top-k", "50", "--rep-penalty", "1.2",
                            "--max-tokens", "16", "--seed", "1234", "--prompt", "anerthinon stqu", *extra],
                           capture_output=True, timeout=300)
        assert r.returncode == 0, r.stderr
        outs.append(generated_text(r.stdout.decode("latin-1")))
    assert outs[0] == outs[1]
