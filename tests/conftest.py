"""Shared test setup: markers, import paths, synthetic model fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gpt2-opencl-1.1_b200")
for p in (PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

from gpt2b200 import synth as _synth  # noqa: E402

MODEL_CACHE = _synth.default_cache()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def tiny_affine_model():
    """Two-layer GPT-2 (E=128, 2 heads, full vocabulary) with random LN and bias values."""
    from gpt2b200 import synth
    return synth.ensure_model(os.path.join(MODEL_CACHE, "tiny_affine_s1"), synth.TINY, seed=1, affine=True)


@pytest.fixture(scope="session")
def tiny_model():
    from gpt2b200 import synth
    return synth.ensure_model(os.path.join(MODEL_CACHE, "tiny_s2"), synth.TINY, seed=2)


@pytest.fixture(scope="session")
def small_model():
    """GPT-2 small shape, seeded N(0, 0.02), the benchmark's weights."""
    from gpt2b200 import synth
    return synth.ensure_model(os.path.join(MODEL_CACHE, "small_s0"), synth.SMALL, seed=0)
