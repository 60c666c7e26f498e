"""Seeded synthetic GPT-2 checkpoints and prompts.

Writes a model directory in the layout the reference loader expects
(``main.c:1339-1417``): ``config.json`` read by ``load_config``
(``main.c:294-331``) and ``model.safetensors`` with GPT-2 tensor names
(``wte.weight``, ``h.{l}.attn.c_attn.weight`` ... ``ln_f.bias``) in the
Conv1D ``[in, out]`` layout (``main.c:1234-1250``), and no
``lm_head.weight`` so the head is tied to ``wte`` (``main.c:1374-1386``).

Weights are N(0, 0.02) for ``wte``, ``wpe`` and every projection; LayerNorm
gamma = 1, beta = 0; biases 0.  ``affine=True`` draws LN and bias values too,
so tests exercise the bias and LN arithmetic.  ``dtype="f16"`` stores every
tensor as IEEE half (the engine's fp16 path; the reference only loads F32);
``dtype="bf16"`` stores bfloat16 (the fp32 values rounded to nearest even).
``outliers=True`` adds a few large residual-stream columns, as real GPT-2
checkpoints have: a large constant in two ``wpe`` columns and those columns
of every ``mlp.c_proj.weight`` scaled up, so the stream reaches ~10^3 there.

The stream of random numbers is fixed by ``seed`` and the tensor order
below, so the same directory is produced on every machine with this numpy.
"""
from __future__ import annotations

import json
import os
import struct
import tempfile
from dataclasses import dataclass, asdict

import numpy as np


@dataclass(frozen=True)
class GPT2Shape:
    n_layer: int
    n_embd: int
    n_head: int
    n_ctx: int = 1024
    vocab_size: int = 50257
    n_inner: int = 0          # 0 -> 4 * n_embd, as main.c:315-316

    @property
    def ffn(self) -> int:
        return self.n_inner if self.n_inner > 0 else 4 * self.n_embd

    @property
    def padded_vocab(self) -> int:
        return (self.vocab_size + 3) & ~3


# The shapes named by the benchmark configurations.
SMALL = GPT2Shape(n_layer=12, n_embd=768, n_head=12)
MEDIUM = GPT2Shape(n_layer=24, n_embd=1024, n_head=16)
XL = GPT2Shape(n_layer=48, n_embd=1600, n_head=25)
# A two-layer model with the full vocabulary (EOS id 50256 exists) for fast tests.
TINY = GPT2Shape(n_layer=2, n_embd=128, n_head=2, n_ctx=1024, vocab_size=50257)

_DT = {"f32": ("F32", np.float32), "f16": ("F16", np.float16), "bf16": ("BF16", None)}
OUTLIER_COLS = (5, 77)   # residual-stream columns made large by outliers=True


def default_cache() -> str:
    """Directory for generated synthetic checkpoints: $G2_MODEL_CACHE, else one
    under the system's temporary directory."""
    return os.environ.get("G2_MODEL_CACHE", os.path.join(tempfile.gettempdir(), "g2_models"))


def to_bf16(a: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bits (uint16), rounded to nearest even (finite inputs)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def from_bf16(b: np.ndarray) -> np.ndarray:
    """bfloat16 bits (uint16) -> float32."""
    return (b.astype(np.uint32) << 16).view(np.float32)


def tensor_plan(s: GPT2Shape):
    """(name, shape, kind) in file order; kind is 'w' (N(0,.02)), 'g' (gamma), 'b' (bias/beta)."""
    E, F = s.n_embd, s.ffn
    plan = [("wte.weight", (s.vocab_size, E), "w"), ("wpe.weight", (s.n_ctx, E), "w")]
    for l in range(s.n_layer):
        p = f"h.{l}."
        plan += [
            (p + "ln_1.weight", (E,), "g"), (p + "ln_1.bias", (E,), "b"),
            (p + "attn.c_attn.weight", (E, 3 * E), "w"), (p + "attn.c_attn.bias", (3 * E,), "b"),
            (p + "attn.c_proj.weight", (E, E), "w"), (p + "attn.c_proj.bias", (E,), "b"),
            (p + "ln_2.weight", (E,), "g"), (p + "ln_2.bias", (E,), "b"),
            (p + "mlp.c_fc.weight", (E, F), "w"), (p + "mlp.c_fc.bias", (F,), "b"),
            (p + "mlp.c_proj.weight", (F, E), "w"), (p + "mlp.c_proj.bias", (E,), "b"),
        ]
    plan += [("ln_f.weight", (E,), "g"), ("ln_f.bias", (E,), "b")]
    return plan


def _draw(rng, shape, kind, affine):
    if kind == "w":
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
    if not affine:
        return np.ones(shape, np.float32) if kind == "g" else np.zeros(shape, np.float32)
    if kind == "g":
        return np.float32(1.0) + rng.standard_normal(shape, dtype=np.float32) * np.float32(0.1)
    return rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)


def write_safetensors(path: str, tensors):
    """Write (name, np.ndarray) pairs as a safetensors file (8-byte LE header length + JSON + data)."""
    header, off = {}, 0
    for name, arr in tensors:
        tag = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.uint16): "BF16"}[arr.dtype]
        n = arr.nbytes
        header[name] = {"dtype": tag, "shape": list(arr.shape), "data_offsets": [off, off + n]}
        off += n
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for _, arr in tensors:
            f.write(np.ascontiguousarray(arr).tobytes())


def write_config(d: str, s: GPT2Shape):
    cfg = {"model_type": "gpt2", "n_layer": s.n_layer, "n_embd": s.n_embd, "n_head": s.n_head,
           "n_positions": s.n_ctx, "n_ctx": s.n_ctx, "vocab_size": s.vocab_size,
           "activation_function": "gelu_new", "layer_norm_epsilon": 1e-5}
    if s.n_inner:
        cfg["n_inner"] = s.n_inner
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)


def _outliers(name: str, a: np.ndarray) -> np.ndarray:
    """The outlier columns: +500 in wpe (every position), x40 in mlp.c_proj's output columns."""
    if name == "wpe.weight":
        a = a.copy()
        a[:, list(OUTLIER_COLS)] += np.float32(500.0)
    elif name.endswith("mlp.c_proj.weight"):
        a = a.copy()
        a[:, list(OUTLIER_COLS)] *= np.float32(40.0)
    return a


def make_model(d: str, s: GPT2Shape, seed: int = 0, dtype: str = "f32", affine: bool = False,
               layout: str = "conv1d", outliers: bool = False, round_to: str = None) -> str:
    """Create ``d`` with config.json and model.safetensors; return ``d``.

    ``layout="linear"`` stores projections as ``[out, in]`` (nn.Linear), which
    the loader must detect and transpose (``main.c:1252-1300``).
    ``round_to="bf16"`` stores the bf16-rounded values in the file's dtype (the
    F32 twin of a bf16 file).
    """
    os.makedirs(d, exist_ok=True)
    rng = np.random.default_rng(seed)
    out = []
    for name, shape, kind in tensor_plan(s):
        a = _draw(rng, shape, kind, affine)
        if outliers:
            a = _outliers(name, a)
        if round_to == "bf16":
            a = from_bf16(to_bf16(a))
        if layout == "linear" and a.ndim == 2 and name.startswith("h."):
            a = np.ascontiguousarray(a.T)
        out.append((name, to_bf16(a) if dtype == "bf16" else a.astype(_DT[dtype][1])))
    write_safetensors(os.path.join(d, "model.safetensors"), out)
    write_config(d, s)
    with open(os.path.join(d, "synth.json"), "w") as f:
        json.dump(_tag(s, seed, dtype, affine, layout, outliers, round_to), f)
    return d


def _tag(s, seed, dtype, affine, layout, outliers, round_to):
    t = {"shape": asdict(s), "seed": seed, "dtype": dtype, "affine": affine, "layout": layout}
    if outliers:
        t["outliers"] = True
    if round_to:
        t["round_to"] = round_to
    return t


def ensure_model(d: str, s: GPT2Shape, seed: int = 0, dtype: str = "f32", affine: bool = False,
                 layout: str = "conv1d", outliers: bool = False, round_to: str = None) -> str:
    """make_model unless ``d`` already holds the same synthetic model."""
    tag = os.path.join(d, "synth.json")
    want = _tag(s, seed, dtype, affine, layout, outliers, round_to)
    try:
        with open(tag) as f:
            if json.load(f) == want and os.path.exists(os.path.join(d, "model.safetensors")):
                return d
    except (OSError, ValueError):
        pass
    return make_model(d, s, seed, dtype, affine, layout, outliers, round_to)


def prompt_ids(seed: int, n: int, vocab: int = 50257) -> np.ndarray:
    """Seeded uniform token ids in [0, vocab) (the benchmark prompts)."""
    return np.random.default_rng(1_000_003 + seed).integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("dir")
    ap.add_argument("--shape", default="small", choices=["tiny", "small", "medium", "xl"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--dtype", default="f32", choices=list(_DT))
    ap.add_argument("--affine", action="store_true")
    a = ap.parse_args()
    make_model(a.dir, {"tiny": TINY, "small": SMALL, "medium": MEDIUM, "xl": XL}[a.shape],
               a.seed, a.dtype, a.affine)
