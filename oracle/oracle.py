"""ctypes access to the parity oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs may import this module.  It loads

* ``oracle/libref_cpu.so`` -- the C restatement of the reference hot path
  (``ref_cpu.c``), and
* ``oracle/_ref/libref_main.so`` -- the reference's own ``main.c``,
  ``math.cl`` and ``tokenizer.c`` compiled from the reference tree onto a CPU
  OpenCL shim (``oracle/Makefile``).  It holds the reference's global state,
  so one model per process.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_CPU = os.path.join(HERE, "libref_cpu.so")
LIB_REF = os.path.join(HERE, "_ref", "libref_main.so")

_fp = C.POINTER(C.c_float)
_ip = C.POINTER(C.c_int)


def build(quiet: bool = True) -> None:
    """Run oracle/Makefile (builds _ref/ only where the reference sources exist)."""
    out = subprocess.run(["make", "-C", HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


def iptr(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_ip)


def _opt(a):
    return None if a is None else fptr(a)


class RefConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in
                ("n_layer", "n_embd", "n_head", "n_ctx", "vocab_size", "ffn_dim", "padded_vocab")]


_cpu = None


def cpu_lib():
    """The restated oracle (libref_cpu.so)."""
    global _cpu
    if _cpu is None:
        if not os.path.exists(LIB_CPU):
            build()
        L = C.CDLL(LIB_CPU)
        L.ref_last_error.restype = C.c_char_p
        L.ref_gelu_f.restype = C.c_float
        L.ref_gelu_f.argtypes = [C.c_float]
        L.ref_kth_largest.restype = C.c_float
        L.ref_seq_logits.restype = _fp
        L.ref_seq_hidden.restype = _fp
        L.ref_seq_kcache.restype = _fp
        L.ref_seq_vcache.restype = _fp
        L.ref_model_lm_head.restype = _fp
        L.ref_attn_scores_1q.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.c_int, C.c_float]
        L.ref_sample_next_token.argtypes = [_fp, C.c_int, _ip, C.c_int, C.c_int, C.c_float, C.c_int,
                                            C.c_float]
        L.ref_generate.argtypes = [C.c_void_p, _ip, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int,
                                   C.c_float, _ip]
        _cpu = L
    return _cpu


class RefModel:
    """A model and one sequence state in the restated oracle."""

    def __init__(self, model_dir: str, ks_attn_proj: int = 8, ks_ffn2: int = 8, attn_lws: int = 64):
        L = cpu_lib()
        self.L = L
        self.m = C.c_void_p()
        rc = L.ref_model_open(model_dir.encode(), C.byref(self.m))
        if rc:
            raise RuntimeError(f"ref_model_open: {rc} {L.ref_last_error().decode()}")
        L.ref_model_set_tuning(self.m, ks_attn_proj, ks_ffn2, attn_lws)
        c = RefConfig()
        L.ref_model_get_config(self.m, C.byref(c))
        self.cfg = c
        self.seq = C.c_void_p()
        if L.ref_seq_new(self.m, C.byref(self.seq)):
            raise RuntimeError(L.ref_last_error().decode())

    def new_seq(self):
        s = C.c_void_p()
        if self.L.ref_seq_new(self.m, C.byref(s)):
            raise RuntimeError(self.L.ref_last_error().decode())
        return s

    def prefill(self, ids, seq=None) -> None:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        rc = self.L.ref_prefill(seq or self.seq, iptr(ids), len(ids))
        if rc:
            raise RuntimeError(self.L.ref_last_error().decode())

    def decode(self, tok: int, pos: int, seq=None) -> None:
        rc = self.L.ref_decode(seq or self.seq, int(tok), int(pos))
        if rc:
            raise RuntimeError(self.L.ref_last_error().decode())

    def logits(self, seq=None) -> np.ndarray:
        p = self.L.ref_seq_logits(seq or self.seq)
        return np.ctypeslib.as_array(p, shape=(self.cfg.padded_vocab,)).copy()

    def hidden(self, seq=None) -> np.ndarray:
        p = self.L.ref_seq_hidden(seq or self.seq)
        return np.ctypeslib.as_array(p, shape=(self.cfg.n_embd,)).copy()

    def kv(self, layer: int, seq=None):
        E = self.cfg.n_embd
        k = np.ctypeslib.as_array(self.L.ref_seq_kcache(seq or self.seq, layer), shape=(E, 1024)).copy()
        v = np.ctypeslib.as_array(self.L.ref_seq_vcache(seq or self.seq, layer), shape=(1024, E)).copy()
        return k, v

    def generate(self, prompt, max_new: int, min_new: int = None, temperature: float = 0.0,
                 top_k: int = 40, rep_penalty: float = 1.0, seq=None) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max_new, np.int32)
        n = self.L.ref_generate(seq or self.seq, iptr(prompt), len(prompt), max_new,
                                max_new if min_new is None else min_new, temperature, top_k,
                                rep_penalty, iptr(out))
        if n < 0:
            raise RuntimeError(self.L.ref_last_error().decode())
        return out[:n]

    def close(self):
        if self.seq:
            self.L.ref_seq_free(self.seq)
            self.seq = None
        if self.m:
            self.L.ref_model_close(self.m)
            self.m = None


def sample(logits: np.ndarray, vocab: int, ctx, forbid_eos: bool, temperature: float, top_k: int,
           rep_penalty: float) -> int:
    L = cpu_lib()
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    ctx = np.ascontiguousarray(ctx, dtype=np.int32)
    return L.ref_sample_next_token(fptr(logits), vocab, iptr(ctx), len(ctx), int(forbid_eos),
                                   temperature, top_k, rep_penalty)


_refmain = None


def ref_available() -> bool:
    return os.path.exists(LIB_REF)


def ref_fast() -> bool:
    """Whether the reference build runs barrier kernels on fibers (fast enough
    for GPT-2-small prefill); the thread-per-work-item executor is not."""
    if not ref_available():
        return False
    return hasattr(ref_lib(), "refcl_fiber_executor")


def ref_lib():
    """The reference's own code (libref_main.so)."""
    global _refmain
    if _refmain is None:
        L = C.CDLL(LIB_REF)
        L.refmain_kth_largest.restype = C.c_float
        L.refmain_sample.argtypes = [_ip, C.c_int, C.c_int, C.c_float, C.c_int, C.c_float]
        L.refcl_run_kernel.argtypes = [C.c_char_p, C.c_int, C.c_int, C.POINTER(C.c_size_t),
                                       C.POINTER(C.c_size_t), C.POINTER(C.c_uint64), C.c_int]
        _refmain = L
    return _refmain


class RefMain:
    """The reference's main.c state (one per process)."""
    _open = False

    def __init__(self, model_dir: str, ks_attn_proj: int = 8, ks_ffn2: int = 8, attn_lws: int = 64):
        if RefMain._open:
            raise RuntimeError("the reference holds one model per process")
        self.L = ref_lib()
        rc = self.L.refmain_open(model_dir.encode())
        if rc:
            raise RuntimeError(f"refmain_open failed: {rc}")
        RefMain._open = True
        self.L.refmain_set_tuning(ks_attn_proj, ks_ffn2, attn_lws)
        c = (C.c_int * 7)()
        self.L.refmain_config(c)
        self.cfg = RefConfig(*c)

    def prefill(self, ids) -> None:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        self.L.refmain_prefill(iptr(ids), len(ids))

    def decode(self, tok: int, pos: int) -> None:
        self.L.refmain_decode(int(tok), int(pos))

    def logits(self) -> np.ndarray:
        out = np.zeros(self.cfg.padded_vocab, np.float32)
        self.L.refmain_read_logits(fptr(out), self.cfg.padded_vocab)
        return out

    def kv(self, layer: int):
        E = self.cfg.n_embd
        k = np.zeros((E, 1024), np.float32)
        v = np.zeros((1024, E), np.float32)
        self.L.refmain_read_kv(layer, fptr(k), fptr(v))
        return k, v

    def sample(self, ctx, forbid_eos: bool, temperature: float = 0.0, top_k: int = 40,
               rep_penalty: float = 1.0) -> int:
        ctx = np.ascontiguousarray(ctx, dtype=np.int32)
        return self.L.refmain_sample(iptr(ctx), len(ctx), int(forbid_eos), temperature, top_k, rep_penalty)

    def generate(self, prompt, max_new: int, min_new: int = None, temperature: float = 0.0,
                 top_k: int = 40, rep_penalty: float = 1.0) -> np.ndarray:
        """main.c:2106-2150 (prefill, sample, decode loop) through the reference's functions."""
        min_new = max_new if min_new is None else min_new
        ids = list(int(t) for t in prompt)
        self.prefill(np.array(ids, np.int32))
        nxt = self.sample(np.array(ids, np.int32), 0 < min_new, temperature, top_k, rep_penalty)
        ids.append(nxt)
        out = [nxt]
        generated = 1
        while generated < max_new and nxt != 50256 and len(ids) < 1024:
            self.decode(ids[-1], len(ids) - 1)
            nxt = self.sample(np.array(ids, np.int32), generated < min_new, temperature, top_k, rep_penalty)
            ids.append(nxt)
            generated += 1
            out.append(nxt)
        return np.array(out, np.int32)

    def close(self):
        if RefMain._open:
            self.L.refmain_close()
            RefMain._open = False


def run_ref_kernel(name: str, gws, lws, args, program_kind: int = 0) -> None:
    """Run one of the reference's math.cl kernels (or its generated matmul,
    program_kind=1) over an NDRange on host arrays.  ``args`` holds numpy
    arrays (buffers), None (NULL buffer), ints and floats in kernel order."""
    L = ref_lib()
    raw = (C.c_uint64 * len(args))()
    for i, a in enumerate(args):
        if a is None:
            raw[i] = 0
        elif isinstance(a, np.ndarray):
            raw[i] = a.ctypes.data
        elif isinstance(a, float) or isinstance(a, np.floating):
            raw[i] = int(np.array([a], np.float32).view(np.uint32)[0])
        else:
            raw[i] = int(np.array([a], np.int32).view(np.uint32)[0])
    g = (C.c_size_t * 3)(*list(gws) + [1] * (3 - len(gws)))
    l = (C.c_size_t * 3)(*list(lws) + [1] * (3 - len(lws)))
    rc = L.refcl_run_kernel(name.encode(), program_kind, len(gws), g, l, raw, len(args))
    if rc:
        raise RuntimeError(f"refcl_run_kernel({name}) = {rc}")


class RefTokenizer:
    """The reference's own tokenizer.c (in libref_main.so): gpt2_tokenizer_load /
    gpt2_encode / gpt2_decode."""

    def __init__(self, directory: str):
        L = ref_lib()
        L.gpt2_tokenizer_load.restype = C.c_void_p
        L.gpt2_tokenizer_load.argtypes = [C.c_char_p]
        L.gpt2_tokenizer_free.argtypes = [C.c_void_p]
        L.gpt2_encode.argtypes = [C.c_void_p, C.c_char_p, _ip, C.c_int]
        L.gpt2_decode.argtypes = [C.c_void_p, _ip, C.c_int, C.c_char_p, C.c_int]
        L.gpt2_tokenizer_vocab_size.argtypes = [C.c_void_p]
        self.L = L
        self.h = L.gpt2_tokenizer_load(directory.encode())
        if not self.h:
            raise RuntimeError(f"reference tokenizer failed to load {directory}")

    def close(self):
        if self.h:
            self.L.gpt2_tokenizer_free(self.h)
            self.h = None

    def encode(self, data: bytes, max_ids: int = None) -> list:
        cap = max_ids if max_ids is not None else len(data) + 1
        out = (C.c_int * max(cap, 1))()
        n = self.L.gpt2_encode(self.h, data, out, max(cap, 1))
        return list(out[:n])

    def decode(self, ids, max_bytes: int = None) -> bytes:
        a = np.ascontiguousarray(ids, dtype=np.int32)
        cap = max_bytes if max_bytes is not None else 16 * len(a) + 1
        buf = C.create_string_buffer(max(cap, 1))
        n = self.L.gpt2_decode(self.h, iptr(a), len(a), buf, max(cap, 1))
        return buf.raw[:n]
