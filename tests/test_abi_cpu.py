"""CPU-only checks of the C ABI: exports, host sampler, model-file validation.

No GPU is needed: g2_sample is host code, and g2_open validates config.json
and model.safetensors before it looks for a device, so malformed inputs give
G2_ERR_IO / G2_ERR_FORMAT here exactly as on a GPU box.
"""
import ctypes as C
import json
import os
import re
import shutil
import struct

import numpy as np
import pytest

import gpt2b200 as g2
import oracle
from gpt2b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gpt2b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(g2k?_[a-z_0-9]+)\s*\(", src)))


def test_library_exports_every_declared_function():
    names = declared_functions()
    assert len(names) >= 20
    lib = C.CDLL(g2.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_checked_build_exports_every_declared_function():
    """The bounds-checked build (make check, -DG2_CHECK) is the same ABI."""
    path = os.path.join(ROOT, "gpt2-opencl-1.1_b200", "libgpt2b200_check.so")
    if not os.path.exists(path):
        pytest.skip("checked build not made (make -C gpt2-opencl-1.1_b200 check)")
    lib = C.CDLL(path)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_workspace_queries_without_device():
    assert g2.matvec_workspace(2304, 768) > 0
    assert g2.matvec_workspace(0, 768) == 0
    # per head: one partial of 64 outputs + running max and sum for each 128-key chunk
    assert g2.attention_workspace(12, 1024) >= 12 * (1024 // 128) * 66 * 4
    assert g2.attention_workspace(12, 1024) < g2.attention_workspace(12, 2048)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_sampler_greedy_matches_oracle(seed):
    rng = np.random.default_rng(seed)
    V = 50257
    logits = rng.standard_normal(V).astype(np.float32)
    logits[123] = logits.max()   # a tie: first index wins (main.c:1898-1904)
    ctx = rng.integers(0, V, 40).astype(np.int32)
    for forbid in (0, 1):
        for rep in (1.0, 1.1, 1.3):
            want = oracle.sample(logits, V, ctx, forbid, 0.0, 40, rep)
            assert g2.sample(logits, ctx, forbid, 0.0, 40, rep) == want


def test_sampler_eos_mask():
    logits = np.zeros(50257, np.float32)
    logits[g2.EOS] = 5.0
    assert g2.sample(logits, [], forbid_eos=False) == g2.EOS
    assert g2.sample(logits, [], forbid_eos=True) == 0


@pytest.mark.parametrize("T,k,rep", [(0.8, 40, 1.1), (1.0, 0, 1.0), (0.5, 256, 1.2), (1.3, 1, 1.0)])
def test_sampler_stochastic_stream_matches_oracle(T, k, rep):
    """Same rand() stream -> same draws as the reference's sample_next_token."""
    rng = np.random.default_rng(7)
    V = 50257
    libc = C.CDLL(None)
    for trial in range(20):
        logits = (rng.standard_normal(V) * 2).astype(np.float32)
        ctx = rng.integers(0, V, 30).astype(np.int32)
        libc.srand(1000 + trial)
        want = oracle.sample(logits, V, ctx, trial % 2, T, k, rep)
        libc.srand(1000 + trial)
        got = g2.sample(logits, ctx, trial % 2, T, k, rep)
        assert got == want


def test_sampler_does_not_modify_input():
    logits = np.arange(100, dtype=np.float32)
    before = logits.copy()
    g2.sample(logits, [5, 6], True, 0.7, 10, 1.5)
    assert np.array_equal(logits, before)


def test_sampler_bad_args():
    with pytest.raises(g2.G2Error) as ei:
        g2.sample(np.zeros(0, np.float32), [])
    assert ei.value.code == -1


# ---- model-file validation (host side of g2_open) ------------------------------------
@pytest.fixture()
def model_copy(tmp_path, tiny_model):
    d = tmp_path / "m"
    shutil.copytree(tiny_model, d)
    return str(d)


def open_err(d):
    with pytest.raises(g2.G2Error) as ei:
        g2.Engine(d)
    return ei.value.code, str(ei.value)


def test_open_missing_dir():
    code, msg = open_err("/nonexistent/model")
    assert code == -2 and "model.safetensors" in msg


def test_open_valid_model_reaches_device_check(model_copy):
    """A well-formed model passes validation; without a GPU the next error is CUDA."""
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        pytest.skip("GPU present: covered by the GPU tests")
    code, _ = open_err(model_copy)
    assert code == -4


def _rewrite_header(d, mutate):
    p = os.path.join(d, "model.safetensors")
    raw = open(p, "rb").read()
    n = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + n])
    mutate(hdr)
    hb = json.dumps(hdr).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    # keep the data segment where it was relative to the header end
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(hb)) + hb + raw[8 + n:])


def test_truncated_header(model_copy):
    p = os.path.join(model_copy, "model.safetensors")
    with open(p, "r+b") as f:
        f.truncate(5)
    assert open_err(model_copy)[0] == -3


def test_garbage_header(model_copy):
    p = os.path.join(model_copy, "model.safetensors")
    raw = bytearray(open(p, "rb").read())
    raw[8:16] = b"notjson!"
    open(p, "wb").write(raw)
    assert open_err(model_copy)[0] == -3


def test_missing_tensor(model_copy):
    _rewrite_header(model_copy, lambda h: h.pop("h.1.mlp.c_fc.bias"))
    code, msg = open_err(model_copy)
    assert code == -3 and "h.1.mlp.c_fc.bias" in msg


def test_wrong_shape(model_copy):
    def m(h):
        h["h.0.attn.c_proj.weight"]["shape"] = [64, 256]
    _rewrite_header(model_copy, m)
    assert open_err(model_copy)[0] == -3


def test_bad_dtype(model_copy):
    def m(h):
        h["ln_f.weight"]["dtype"] = "I32"
    _rewrite_header(model_copy, m)
    code, msg = open_err(model_copy)
    assert code == -3 and "dtype" in msg


def test_offsets_past_end(model_copy):
    def m(h):
        h["wte.weight"]["data_offsets"][1] += 1 << 30
    _rewrite_header(model_copy, m)
    assert open_err(model_copy)[0] == -3


def test_config_over_context_limit(model_copy):
    cfg = json.load(open(os.path.join(model_copy, "config.json")))
    cfg["n_positions"] = cfg["n_ctx"] = 2048
    json.dump(cfg, open(os.path.join(model_copy, "config.json"), "w"))
    assert open_err(model_copy)[0] == -3


def test_config_bad_head_size(model_copy):
    cfg = json.load(open(os.path.join(model_copy, "config.json")))
    cfg["n_head"] = 3
    json.dump(cfg, open(os.path.join(model_copy, "config.json"), "w"))
    assert open_err(model_copy)[0] == -3


def test_open_bad_args(tiny_model):
    h = C.c_void_p()
    assert g2.lib.g2_open(None, 0, 1, 0, C.byref(h)) == -1
    assert g2.lib.g2_open(tiny_model.encode(), 0, 0, 0, C.byref(h)) == -1
    assert g2.lib.g2_open(tiny_model.encode(), 0, 1, 7, C.byref(h)) == -1


def test_topk_argument_checks_without_device():
    """g2_topk and g2k_topk reject bad arguments on the host before any device work
    (every call below fails a check that precedes the launch)."""
    vals, ids = (C.c_float * 4)(), (C.c_int * 4)()
    assert g2.lib.g2_topk(None, 0, 1, vals, ids) == -1                        # null engine
    assert g2.lib.g2k_topk(None, 100, 1, C.cast(vals, C.c_void_p), C.cast(ids, C.c_void_p), None) == -1
    buf = (C.c_float * 100)()
    for n, k in ((100, 0), (100, 101), (1000, 257), (0, 1), (-5, 1)):        # k in [1, min(256, n)]
        assert g2.lib.g2k_topk(C.cast(buf, C.c_void_p), n, k, C.cast(vals, C.c_void_p),
                               C.cast(ids, C.c_void_p), None) == -6, (n, k)
    assert "g2k_topk" in g2.lib.g2_last_error().decode()


def test_linear_layout_model_validates(tmp_path):
    """nn.Linear [out,in] files are accepted (transposed at load, main.c:1252-1300)."""
    d = synth.make_model(str(tmp_path / "lin"), synth.TINY, seed=3, layout="linear")
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("GPU present: covered by the GPU tests")
    except Exception:
        pass
    assert open_err(d)[0] == -4
