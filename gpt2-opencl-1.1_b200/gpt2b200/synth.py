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
tensor as IEEE half (the engine's fp16 path; the reference only loads F32).

The stream of random numbers is fixed by ``seed`` and the tensor order
below, so the same directory is produced on every machine with this numpy.
"""
from __future__ import annotations

import json
import os
import struct
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

_DT = {"f32": ("F32", np.float32), "f16": ("F16", np.float16)}


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
        tag = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16"}[arr.dtype]
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


def make_model(d: str, s: GPT2Shape, seed: int = 0, dtype: str = "f32", affine: bool = False,
               layout: str = "conv1d") -> str:
    """Create ``d`` with config.json and model.safetensors; return ``d``.

    ``layout="linear"`` stores projections as ``[out, in]`` (nn.Linear), which
    the loader must detect and transpose (``main.c:1252-1300``).
    """
    os.makedirs(d, exist_ok=True)
    rng = np.random.default_rng(seed)
    np_dt = _DT[dtype][1]
    out = []
    for name, shape, kind in tensor_plan(s):
        a = _draw(rng, shape, kind, affine)
        if layout == "linear" and a.ndim == 2 and name.startswith("h."):
            a = np.ascontiguousarray(a.T)
        out.append((name, a.astype(np_dt)))
    write_safetensors(os.path.join(d, "model.safetensors"), out)
    write_config(d, s)
    with open(os.path.join(d, "synth.json"), "w") as f:
        json.dump({"shape": asdict(s), "seed": seed, "dtype": dtype, "affine": affine,
                   "layout": layout}, f)
    return d


def ensure_model(d: str, s: GPT2Shape, seed: int = 0, dtype: str = "f32", affine: bool = False,
                 layout: str = "conv1d") -> str:
    """make_model unless ``d`` already holds the same synthetic model."""
    tag = os.path.join(d, "synth.json")
    want = {"shape": asdict(s), "seed": seed, "dtype": dtype, "affine": affine, "layout": layout}
    try:
        with open(tag) as f:
            if json.load(f) == want and os.path.exists(os.path.join(d, "model.safetensors")):
                return d
    except (OSError, ValueError):
        pass
    return make_model(d, s, seed, dtype, affine, layout)


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
