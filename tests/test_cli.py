"""Command-line program (gpt2b200-cli, the host flow of main.c:1966-2160):
argument handling without a GPU."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "gpt2-opencl-1.1_b200", "gpt2b200-cli")

pytestmark = pytest.mark.skipif(not os.path.exists(CLI), reason="gpt2b200-cli not built")


def run(*args):
    return subprocess.run([CLI, *args], capture_output=True, text=True, timeout=120)


def test_usage_without_model():
    r = run()
    assert r.returncode == 1 and "Usage:" in r.stderr
    r = run("--bogus-flag")
    assert r.returncode == 1 and "Usage:" in r.stderr


def test_list_devices():
    r = run("--list-devices")
    assert r.returncode == 0
    assert "no CUDA devices" in r.stdout or "SMs" in r.stdout


def test_missing_model_fails_cleanly(tmp_path):
    r = run("--model", str(tmp_path), "--greedy", "--prompt", "hi")
    assert r.returncode == 1
    assert "model.safetensors" in r.stderr or "Failed" in r.stderr
