"""Robustness of the engine on the GPU: inputs and situations outside the
benchmark's synthetic N(0, 0.02) models.

* Outlier residual columns (~10^3, as real GPT-2 checkpoints have): the
  persistent decode kernel's fixed-point split-K accumulators and its folded
  LayerNorm must stay within the fp32 bar (1e-3 of max |logit|) of the
  oracle, and no accumulator contribution may reach the +-2^21 clamp (the
  kernel reports one as G2_ERR_RANGE).
* BF16 checkpoints (the reference loads F32 only, main.c:1213): the engine's
  logits from a BF16 file equal, bit for bit, its logits from the F32 file
  holding the same bf16-rounded values.
* nn.Linear-layout checkpoints, transposed on the device at load
  (main.c:1252-1300 transposes on the host): the same logits and greedy
  stream as the Conv1D file of the same weights, on the persistent kernel
  too (whose unit packing reads either layout).
* A bounded device-side wait that runs out: with a short wait limit and a
  host-seeded accumulator word that can never turn ready, the persistent
  kernel returns G2_ERR_TIMEOUT (no hang, no fault), and the same engine
  then serves a correct generation.
* Engines on two devices in one process, each prefilling more than 64 rows
  (the tiled prefill attention raises its shared-memory limit per device);
  skipped with fewer than two GPUs.
"""
import os

import numpy as np
import pytest

import oracle
from gpt2b200 import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3


@pytest.fixture(scope="module")
def g2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gpt2b200
    return gpt2b200


def rel(got, want):
    return float(np.abs(got.astype(np.float64) - want).max() / np.abs(want).max())


def test_outlier_columns_persistent_vs_oracle(g2, tmp_path):
    """GPT-2 small with two residual columns near 10^3: logits after prefill and
    over 24 persistent decode steps within 1e-3 of the oracle, identical greedy
    stream, and no clamped accumulator contribution (which would raise
    G2_ERR_RANGE)."""
    d = synth.make_model(str(tmp_path / "outl"), synth.SMALL, seed=3, affine=True, outliers=True)
    prompt = synth.prompt_ids(31, 40)
    ref = oracle.RefModel(d)
    ref.prefill(prompt)
    h = ref.hidden()
    assert np.abs(h[list(synth.OUTLIER_COLS)]).min() > 300.0, "the outlier columns are not large"
    want = ref.generate(prompt, 25)
    with g2.Engine(d) as eng:
        assert eng.cfg.persistent == 1
        got = eng.generate(prompt, 25)
        assert list(got) == list(want)
        ids = list(prompt)
        ref.prefill(prompt)
        eng.prefill(prompt)
        assert rel(eng.logits(), ref.logits()) <= FP32_TOL
        for step in range(24):
            tok = int(want[step])
            ref.decode(tok, len(ids))
            eng.decode(tok, len(ids))
            ids.append(tok)
            assert rel(eng.logits(), ref.logits()) <= FP32_TOL, f"decode step {step}"
    ref.close()


def test_bf16_file_equals_rounded_f32_file(g2, tmp_path):
    a = synth.make_model(str(tmp_path / "bf16"), synth.TINY, seed=8, affine=True, dtype="bf16")
    b = synth.make_model(str(tmp_path / "f32r"), synth.TINY, seed=8, affine=True, round_to="bf16")
    prompt = synth.prompt_ids(9, 21)
    outs = []
    for d in (a, b):
        with g2.Engine(d) as eng:
            eng.prefill(prompt)
            lg = eng.logits()
            toks = eng.generate(prompt, 12)
            outs.append((lg, list(toks)))
    assert np.array_equal(outs[0][0].view(np.uint32), outs[1][0].view(np.uint32))
    assert outs[0][1] == outs[1][1]
    ref = oracle.RefModel(b)
    ref.prefill(prompt)
    assert rel(outs[1][0], ref.logits()) <= FP32_TOL
    ref.close()


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_linear_layout_transposed_on_device(g2, tmp_path, dtype):
    a = synth.make_model(str(tmp_path / "conv"), synth.TINY, seed=6, affine=True, dtype=dtype)
    b = synth.make_model(str(tmp_path / "lin"), synth.TINY, seed=6, affine=True, dtype=dtype, layout="linear")
    prompt = synth.prompt_ids(3, 70)
    outs = []
    for d in (a, b):
        with g2.Engine(d, dtype=g2.G2_F16 if dtype == "f16" else g2.G2_F32) as eng:
            eng.prefill(prompt)
            lg = eng.logits()
            toks = eng.generate(prompt, 16)
            outs.append((lg, list(toks)))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert outs[0][1] == outs[1][1]


def test_expired_wait_returns_timeout_then_recovers(g2, tiny_affine_model, monkeypatch):
    prompt = synth.prompt_ids(17, 10)
    ref = oracle.RefModel(tiny_affine_model)
    want = ref.generate(prompt, 6)
    ref.close()
    monkeypatch.setenv("G2_WAIT_LIMIT_MS", "50")
    monkeypatch.setenv("G2_TEST_STALL", "acc")
    with g2.Engine(tiny_affine_model) as eng:
        assert eng.cfg.persistent == 1
        with pytest.raises(g2.G2Error) as ei:
            eng.generate(prompt, 6)
        assert ei.value.code == -8, str(ei.value)
        got = eng.generate(prompt, 6)          # the stall was one-shot
        assert list(got) == list(want)
        eng.prefill(prompt)
        eng.decode(int(want[0]), len(prompt))  # single-step launches work too
        ref = oracle.RefModel(tiny_affine_model)
        ref.prefill(prompt)
        ref.decode(int(want[0]), len(prompt))
        assert rel(eng.logits(), ref.logits()) <= FP32_TOL
        ref.close()


def test_two_devices_long_prefill(g2, tiny_affine_model):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    prompt = synth.prompt_ids(44, 130)
    ref = oracle.RefModel(tiny_affine_model)
    ref.prefill(prompt)
    want = ref.logits()
    ref.close()
    e0 = g2.Engine(tiny_affine_model, device=0)
    e1 = g2.Engine(tiny_affine_model, device=1)
    try:
        for eng in (e0, e1, e0):
            eng.prefill(prompt)
            assert rel(eng.logits(), want) <= 1e-4
    finally:
        e0.close()
        e1.close()
