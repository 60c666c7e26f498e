"""Python binding of the B200 GPT-2 engine's C ABI (include/gpt2b200.h).

A thin ctypes layer over ``libgpt2b200.so`` (built in-tree by the package
Makefile / ``__graft_entry__.build()``).  The library is mapped on the first
call into it (or by ``load()``), so that importing the package's pure-Python
helpers (``synth``, ``replicas``) maps no engine code.  There is no fallback:
that first call raises ``ImportError`` if the library is missing, and every
call raises ``G2Error`` on a non-zero status.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# G2_LIB selects another build of the same ABI, e.g. the bounds-checked
# libgpt2b200_check.so (`make -C gpt2-opencl-1.1_b200 check`).
LIB_PATH = os.environ.get("G2_LIB") or os.path.join(PKG_DIR, "libgpt2b200.so")

G2_F32, G2_F16 = 0, 1
EOS = 50256
ERRORS = {-1: "ARG", -2: "IO", -3: "FORMAT", -4: "CUDA", -5: "OOM", -6: "RANGE", -7: "STATE", -8: "TIMEOUT"}


class G2Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"G2_ERR_{ERRORS.get(code, code)} ({code}): {msg}")
        self.code = code


class Config(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("n_embd", C.c_int), ("n_head", C.c_int), ("n_ctx", C.c_int),
                ("vocab_size", C.c_int), ("ffn_dim", C.c_int), ("padded_vocab", C.c_int), ("dtype", C.c_int),
                ("max_batch", C.c_int), ("device", C.c_int), ("weight_bytes", C.c_size_t),
                ("device_bytes", C.c_size_t), ("persistent", C.c_int)]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {PKG_DIR}` "
                          "or __graft_entry__.build()")
    L = C.CDLL(LIB_PATH)
    vp, ip, fp = C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_float)
    L.g2_last_error.restype = C.c_char_p
    L.g2_open.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.POINTER(vp)]
    L.g2_close.argtypes = [vp]
    L.g2_get_config.argtypes = [vp, C.POINTER(Config)]
    L.g2_prefill.argtypes = [vp, C.c_int, ip, C.c_int]
    L.g2_decode.argtypes = [vp, C.c_int, C.c_int, C.c_int]
    L.g2_decode_batch.argtypes = [vp, C.c_int, ip, ip, ip]
    L.g2_decode_batch_rows.argtypes = [vp, C.c_int, ip, ip, ip, vp]
    L.g2_lm_head_rows.argtypes = [vp, C.c_int, vp, C.c_int, C.c_int, vp, vp]
    L.g2_logits.argtypes = [vp, C.c_int, fp, C.c_int]
    L.g2_argmax.argtypes = [vp, C.c_int, C.c_int, ip, fp]
    L.g2_topk.argtypes = [vp, C.c_int, C.c_int, fp, ip]
    L.g2_sample.argtypes = [fp, C.c_int, ip, C.c_int, C.c_int, C.c_float, C.c_int, C.c_float, ip]
    L.g2_sample_device.argtypes = [vp, C.c_int, ip, C.c_int, C.c_int, C.c_float, C.c_int, C.c_float, C.c_double, ip]
    L.g2_tokenizer_load.argtypes = [C.c_char_p, C.POINTER(vp)]
    L.g2_tokenizer_free.argtypes = [vp]
    L.g2_tokenizer_free.restype = None
    L.g2_tokenizer_vocab_size.argtypes = [vp]
    L.g2_tok_encode.argtypes = [vp, C.c_char_p, ip, C.c_int]
    L.g2_tok_decode.argtypes = [vp, ip, C.c_int, C.c_char_p, C.c_int]
    L.g2_generate.argtypes = [vp, C.c_int, ip, C.c_int, C.c_int, C.c_int, ip]
    L.g2_generate_batch.argtypes = [vp, C.c_int, ip, ip, ip, C.c_int, ip]
    L.g2_synchronize.argtypes = [vp]
    L.g2_last_timing.argtypes = [vp, fp, fp, ip]
    L.g2_launch_count.argtypes = [vp]
    L.g2_launch_count.restype = C.c_longlong
    L.g2k_matvec_workspace.argtypes = [C.c_int, C.c_int]
    L.g2k_matvec_workspace.restype = C.c_size_t
    L.g2k_matvec.argtypes = [vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, vp, vp, vp, C.c_size_t, vp]
    L.g2k_matvec_noalloc.argtypes = [vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, vp, vp, vp]
    L.g2k_matmul.argtypes = [vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp]
    L.g2k_matmul_tc_workspace.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int]
    L.g2k_matmul_tc_workspace.restype = C.c_size_t
    L.g2k_matmul_tc.argtypes = [vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp, C.c_size_t, vp]
    L.g2k_layernorm.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int, vp]
    L.g2k_attention_workspace.argtypes = [C.c_int, C.c_int]
    L.g2k_attention_workspace.restype = C.c_size_t
    L.g2k_attention.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, vp, C.c_size_t, vp]
    L.g2k_topk.argtypes = [vp, C.c_int, C.c_int, vp, vp, vp]
    return L


class _Lib:
    """The engine library, mapped on first attribute access."""

    def __init__(self):
        self._L = None

    def __getattr__(self, name):
        if self._L is None:
            self._L = _load()
        return getattr(self._L, name)


lib = _Lib()


def load():
    """Map libgpt2b200.so now (raises ImportError if it is missing)."""
    lib.g2_last_error
    return lib._L


def check(rc: int) -> int:
    if rc < 0:
        raise G2Error(rc, lib.g2_last_error().decode(errors="replace"))
    return rc


def _i32(a):
    a = np.ascontiguousarray(a, dtype=np.int32)
    return a, a.ctypes.data_as(C.POINTER(C.c_int))


class Engine:
    """One GPT-2 model on one GPU (g2_open ... g2_close)."""

    def __init__(self, model_dir: str, device: int = 0, max_batch: int = 1, dtype: int = G2_F32):
        self.h = C.c_void_p()
        check(lib.g2_open(model_dir.encode(), device, max_batch, dtype, C.byref(self.h)))
        self.cfg = Config()
        check(lib.g2_get_config(self.h, C.byref(self.cfg)))

    def close(self):
        if self.h:
            check(lib.g2_close(self.h))
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prefill(self, ids, slot: int = 0):
        a, p = _i32(ids)
        check(lib.g2_prefill(self.h, slot, p, len(a)))

    def decode(self, token: int, pos: int, slot: int = 0):
        check(lib.g2_decode(self.h, slot, int(token), int(pos)))

    def decode_batch(self, slots, tokens, pos):
        s, sp = _i32(slots)
        t, tp = _i32(tokens)
        q, qp = _i32(pos)
        check(lib.g2_decode_batch(self.h, len(s), sp, tp, qp))

    def logits(self, slot: int = 0, n: int = None) -> np.ndarray:
        n = self.cfg.padded_vocab if n is None else n
        out = np.zeros(n, np.float32)
        check(lib.g2_logits(self.h, slot, out.ctypes.data_as(C.POINTER(C.c_float)), n))
        return out

    def argmax(self, slot: int = 0, forbid_eos: bool = False):
        t, v = C.c_int(), C.c_float()
        check(lib.g2_argmax(self.h, slot, int(forbid_eos), C.byref(t), C.byref(v)))
        return t.value, v.value

    def topk(self, k: int, slot: int = 0):
        """The k largest logits of `slot` (device): (values [k] decreasing,
        token ids [k]), equal values by increasing id."""
        vals, ids = np.zeros(k, np.float32), np.zeros(k, np.int32)
        check(lib.g2_topk(self.h, slot, k, vals.ctypes.data_as(C.POINTER(C.c_float)),
                          ids.ctypes.data_as(C.POINTER(C.c_int))))
        return vals, ids

    def sample_device(self, context, forbid_eos: bool = False, temperature: float = 0.0, top_k: int = 0,
                      rep_penalty: float = 1.0, u: float = 0.0, slot: int = 0) -> int:
        """sample_next_token on the device with the uniform draw `u` in [0, 1)."""
        a, p = _i32(context)
        t = C.c_int()
        check(lib.g2_sample_device(self.h, slot, p, len(a), int(forbid_eos), temperature, top_k, rep_penalty, u,
                                   C.byref(t)))
        return t.value

    def generate(self, prompt, n_new: int, min_new: int = None, slot: int = 0) -> np.ndarray:
        a, p = _i32(prompt)
        out = np.zeros(n_new, np.int32)
        n = check(lib.g2_generate(self.h, slot, p, len(a), n_new, n_new if min_new is None else min_new,
                                  out.ctypes.data_as(C.POINTER(C.c_int))))
        return out[:n]

    def generate_batch(self, prompts, n_new: int, slots=None) -> np.ndarray:
        slots = list(range(len(prompts))) if slots is None else slots
        s, sp = _i32(slots)
        lens, lp = _i32([len(x) for x in prompts])
        flat, fp_ = _i32(np.concatenate([np.asarray(x, np.int32) for x in prompts]))
        out = np.zeros((len(prompts), n_new), np.int32)
        check(lib.g2_generate_batch(self.h, len(s), sp, fp_, lp, n_new, out.ctypes.data_as(C.POINTER(C.c_int))))
        return out

    def decode_batch_rows(self, slots, tokens, pos, rows):
        """One decode step of several sequences without the LM head; the final
        LayerNorm of each row into `rows` (a device tensor [n, n_embd], fp32)."""
        s, sp = _i32(slots)
        t, tp = _i32(tokens)
        q, qp = _i32(pos)
        check(lib.g2_decode_batch_rows(self.h, len(s), sp, tp, qp, _ptr(rows)))

    def lm_head_rows(self, rows, nrows: int, v0: int, v1: int, best_value, best_index):
        """LM head over vocabulary rows [v0, v1) for `nrows` normalised rows (device
        tensors): each row's first maximum there and its vocabulary index."""
        check(lib.g2_lm_head_rows(self.h, nrows, _ptr(rows), v0, v1, _ptr(best_value), _ptr(best_index)))

    def synchronize(self):
        check(lib.g2_synchronize(self.h))

    def last_timing(self):
        a, b, n = C.c_float(), C.c_float(), C.c_int()
        check(lib.g2_last_timing(self.h, C.byref(a), C.byref(b), C.byref(n)))
        return a.value, b.value, n.value

    def launch_count(self) -> int:
        return lib.g2_launch_count(self.h)


def sample(logits, ctx, forbid_eos=False, temperature=0.0, top_k=40, rep_penalty=1.0, vocab_size=None) -> int:
    """g2_sample: main.c:1872 semantics on host logits."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    c, cp = _i32(ctx)
    out = C.c_int()
    check(lib.g2_sample(lg.ctypes.data_as(C.POINTER(C.c_float)), len(lg) if vocab_size is None else vocab_size,
                        cp, len(c), int(forbid_eos), temperature, top_k, rep_penalty, C.byref(out)))
    return out.value


class Tokenizer:
    """GPT-2 byte-level BPE (g2_tokenizer_*; tokenizer.c semantics) from vocab.json + merges.txt."""

    def __init__(self, directory: str):
        self.h = C.c_void_p()
        rc = lib.g2_tokenizer_load(directory.encode(), C.byref(self.h))
        if rc < 0:
            raise G2Error(rc, f"cannot load vocab.json / merges.txt from {directory}")

    def close(self):
        if self.h:
            lib.g2_tokenizer_free(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def vocab_size(self) -> int:
        return lib.g2_tokenizer_vocab_size(self.h)

    def encode(self, text, max_ids: int = None) -> list:
        b = text.encode() if isinstance(text, str) else bytes(text)
        cap = max_ids if max_ids is not None else len(b) + 1
        out = (C.c_int * max(cap, 1))()
        n = check(lib.g2_tok_encode(self.h, b, out, max(cap, 1)))
        return list(out[:n])

    def decode(self, ids, max_bytes: int = None) -> bytes:
        a, p = _i32(ids)
        cap = max_bytes if max_bytes is not None else 16 * len(a) + 1
        buf = C.create_string_buffer(max(cap, 1))
        n = check(lib.g2_tok_decode(self.h, p, len(a), buf, max(cap, 1)))
        return buf.raw[:n]


# ---- single kernels on device pointers (ints = device addresses) ---------------------
def _ptr(t):
    if t is None:
        return None
    return C.c_void_p(t.data_ptr() if hasattr(t, "data_ptr") else int(t))


def matvec_workspace(N: int, K: int) -> int:
    return lib.g2k_matvec_workspace(N, K)


def matvec(x, W, y, N, K, bias=None, residual=None, gelu=False, ln_gamma=None, ln_beta=None, workspace=None,
           workspace_bytes=0, stream=0):
    check(lib.g2k_matvec(_ptr(x), _ptr(W), _ptr(bias), _ptr(residual), _ptr(y), N, K, int(gelu), _ptr(ln_gamma),
                         _ptr(ln_beta), _ptr(workspace), workspace_bytes, C.c_void_p(stream)))


def matvec_noalloc(x, W, y, N, K, bias=None, residual=None, gelu=False, ln_gamma=None, ln_beta=None, stream=0):
    """g2k_matvec with the library's fixed scratch instead of a caller workspace."""
    check(lib.g2k_matvec_noalloc(_ptr(x), _ptr(W), _ptr(bias), _ptr(residual), _ptr(y), N, K, int(gelu),
                                 _ptr(ln_gamma), _ptr(ln_beta), C.c_void_p(stream)))


def matmul(A, B, C_, M, N, K, bias=None, residual=None, gelu=False, stream=0):
    check(lib.g2k_matmul(_ptr(A), _ptr(B), _ptr(bias), _ptr(residual), _ptr(C_), M, N, K, int(gelu),
                         C.c_void_p(stream)))


def matmul_tc_workspace(M: int, N: int, K: int, precision: int = G2_F32) -> int:
    return lib.g2k_matmul_tc_workspace(M, N, K, precision)


def matmul_tc(A, B, C_, M, N, K, bias=None, residual=None, gelu=False, precision=G2_F32, workspace=None,
              workspace_bytes=0, stream=0):
    """Tensor-core matmul (tcgen05): G2_F32 = 3xTF32 split operands, G2_F16 = fp16 operands."""
    check(lib.g2k_matmul_tc(_ptr(A), _ptr(B), _ptr(bias), _ptr(residual), _ptr(C_), M, N, K, int(gelu), precision,
                            _ptr(workspace), workspace_bytes, C.c_void_p(stream)))


def layernorm(x, out, gamma, beta, n_embd, rows, stream=0):
    check(lib.g2k_layernorm(_ptr(x), _ptr(out), _ptr(gamma), _ptr(beta), n_embd, rows, C.c_void_p(stream)))


def topk(logits, n, k, values, ids, stream=0):
    """g2k_topk on device tensors: the k largest of logits[0..n) into values / ids."""
    check(lib.g2k_topk(_ptr(logits), n, k, _ptr(values), _ptr(ids), C.c_void_p(stream)))


def attention_workspace(n_head: int, max_seq: int) -> int:
    return lib.g2k_attention_workspace(n_head, max_seq)


def attention(q, K, V, out, n_head, max_seq, T_kv, workspace, workspace_bytes, stream=0):
    check(lib.g2k_attention(_ptr(q), _ptr(K), _ptr(V), _ptr(out), n_head, max_seq, T_kv, _ptr(workspace),
                            workspace_bytes, C.c_void_p(stream)))
