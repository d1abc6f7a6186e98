"""ctypes wrapper of the CPU oracle (oracle/oracle.c).

TEST INFRASTRUCTURE ONLY: the parity tests, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` use this module as the checker. The product
library never imports it.

Each wrapper names the reference kernel or host routine it restates; the C file
carries the file:line citations.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
F64P = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
U16P = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
u32, u64, i32, f32 = C.c_uint32, C.c_uint64, C.c_int32, C.c_float


def build() -> str:
    """Compile liboracle.so from oracle.c when it is missing or stale."""
    src = os.path.join(_HERE, "oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE])
    return _LIB_PATH


class OrConfig(C.Structure):
    _fields_ = [
        ("dim", u32), ("layers", u32), ("heads", u32), ("kv_heads", u32),
        ("head_dim", u32), ("hidden", u32), ("vocab", u32), ("seq", u32),
        ("theta", f32), ("eps", f32), ("bf16", i32),
    ]


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    L = C.CDLL(build())
    sig = {
        "or_f32_to_bf16": (None, [F32P, U16P, u64]),
        "or_bf16_to_f32": (None, [U16P, F32P, u64]),
        "or_stream_key": (u64, [u64, u64]),
        "or_normal_at": (f32, [u64, u64, f32, f32]),
        "or_fill_normal_f32": (None, [F32P, u64, u64, u64, f32, f32]),
        "or_fill_normal_bf16": (None, [U16P, u64, u64, u64, f32, f32]),
        "or_uniform_tokens": (None, [I32P, u32, u64, u64, u32, u32]),
        "or_pseudo_random": (None, [F32P, u32, u32]),
        "or_embed": (None, [F32P, u32, u32, F32P]),
        "or_gemv": (None, [F32P, u32, F32P, u32, F32P, u32]),
        "or_matmul_f32": (None, [F32P, u32, u32, F32P, F32P]),
        "or_matmul_bf16": (None, [U16P, u32, u32, F32P, F32P]),
        "or_rmsnorm": (None, [F32P, F32P, F32P, u32]),
        "or_rmsnorm_inplace": (None, [F32P, F32P, u32]),
        "or_rope": (None, [F32P, u32, u32, F32P, u32, u32, f32]),
        "or_rope_store": (None, [F32P, u32, u32, F32P, u32, F32P, u32, f32]),
        "or_cache_store": (None, [F32P, u32, F32P, u32, u32]),
        "or_attention_partial": (None, [F32P, u32, u32, F32P, F32P, u32, F32P, u32, u32]),
        "or_attention_combine": (None, [F32P, u32, u32, u32, F32P, u32]),
        "or_attention": (None, [F32P, u32, u32, F32P, u32, F32P, F32P, F32P, u32, u32]),
        "or_swiglu": (None, [F32P, F32P, u32]),
        "or_add": (None, [F32P, F32P, F32P, u32]),
        "or_cpu_attention_f64": (None, [u32, u32, u32, F32P, F32P, F32P, u32, F64P]),
        "or_sample_argmax": (i32, [F32P, u32]),
        "or_model_create": (C.c_void_p, [C.POINTER(OrConfig), u64, f32]),
        "or_model_destroy": (None, [C.c_void_p]),
        "or_model_weight": (C.c_void_p, [C.c_void_p, C.c_int, u32]),
        "or_state_create": (C.c_void_p, [C.c_void_p]),
        "or_state_destroy": (None, [C.c_void_p]),
        "or_model_step": (C.POINTER(f32), [C.c_void_p, C.c_void_p, u32, u32]),
        "or_embed_token": (None, [C.c_void_p, C.c_void_p, u32]),
        "or_attention_block": (None, [C.c_void_p, C.c_void_p, u32, u32]),
        "or_ffn_block": (None, [C.c_void_p, C.c_void_p, u32]),
        "or_classify": (None, [C.c_void_p, C.c_void_p]),
        "or_state_tensor": (C.POINTER(f32), [C.c_void_p, C.c_int]),
        "or_state_cache": (C.c_void_p, [C.c_void_p, C.c_int]),
        "or_generate_tokens": (i32, [C.c_void_p, C.c_void_p, I32P, u32, u32, i32, i32, I32P,
                                     F32P, u32]),
        "or_set_threads": (None, [i32]),
        "or_get_threads": (i32, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# --------------------------------------------------------------------------
# Element helpers
# --------------------------------------------------------------------------
def to_bf16_bits(a) -> np.ndarray:
    a = _f32(a).ravel()
    out = np.empty(a.size, np.uint16)
    lib().or_f32_to_bf16(a, out, a.size)
    return out


def from_bf16_bits(bits) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16).ravel()
    out = np.empty(bits.size, np.float32)
    lib().or_bf16_to_f32(bits, out, bits.size)
    return out


def round_bf16(a) -> np.ndarray:
    a = _f32(a)
    return from_bf16_bits(to_bf16_bits(a)).reshape(a.shape)


def normal(n, seed, stream, mean=0.0, std=1.0) -> np.ndarray:
    out = np.empty(int(n), np.float32)
    lib().or_fill_normal_f32(out, int(n), seed, stream, mean, std)
    return out


def normal_bf16_bits(n, seed, stream, mean=0.0, std=1.0) -> np.ndarray:
    out = np.empty(int(n), np.uint16)
    lib().or_fill_normal_bf16(out, int(n), seed, stream, mean, std)
    return out


def uniform_tokens(n, seed, stream, lo, hi) -> np.ndarray:
    out = np.empty(int(n), np.int32)
    lib().or_uniform_tokens(out, int(n), seed, stream, lo, hi)
    return out


def pseudo_random(length, seed) -> np.ndarray:
    """tests/kernels.rs:380-390."""
    out = np.empty(int(length), np.float32)
    lib().or_pseudo_random(out, int(length), seed)
    return out


# --------------------------------------------------------------------------
# Kernel restatements (src/kernels.rs)
# --------------------------------------------------------------------------
def embed(table, token):
    table = _f32(table)
    vocab, dim = table.shape
    x = np.empty(dim, np.float32)
    lib().or_embed(table.ravel(), dim, token, x)
    return x


def gemv(x, w, xout, pos):
    """Serial pos-strided GEMV into xout [seq, d] (in place)."""
    x, w = _f32(x), _f32(w)
    d, n = w.shape
    lib().or_gemv(x, n, w.ravel(), d, xout.reshape(-1), pos)
    return xout


def matmul(w, x):
    w, x = _f32(w), _f32(x)
    out = np.empty(w.shape[0], np.float32)
    lib().or_matmul_f32(w.ravel(), w.shape[0], w.shape[1], x, out)
    return out


def matmul_bf16(w_bits, x):
    w_bits = np.ascontiguousarray(w_bits, np.uint16)
    x = _f32(x)
    out = np.empty(w_bits.shape[0], np.float32)
    lib().or_matmul_bf16(w_bits.ravel(), w_bits.shape[0], w_bits.shape[1], x, out)
    return out


def rmsnorm(x, w):
    x, w = _f32(x), _f32(w)
    o = np.empty_like(x)
    lib().or_rmsnorm(x, w, o, x.size)
    return o


def rmsnorm_inplace(x, w):
    lib().or_rmsnorm_inplace(x, _f32(w), x.size)
    return x


def rope(q, k, pos, theta):
    """q [heads, head] and k [seq, kv_heads, head], both rotated in place."""
    head = q.shape[1]
    kv_dim = k.shape[1] * k.shape[2]
    lib().or_rope(q.reshape(-1), q.size, head, k.reshape(-1), kv_dim, pos, theta)


def rope_store(q, k_proj, k, pos, theta):
    head = q.shape[1]
    lib().or_rope_store(q.reshape(-1), q.size, head, _f32(k_proj), k_proj.size,
                        k.reshape(-1), pos, theta)


def cache_store(src, dst, pos):
    row = dst.shape[1] * dst.shape[2]
    lib().or_cache_store(_f32(src), src.size, dst.reshape(-1), row, pos)


def attention_partial(q, key, value, partial, pos):
    q_heads, head = q.shape
    kv_heads = key.shape[1]
    splits = partial.shape[1]
    lib().or_attention_partial(_f32(q).ravel(), q_heads, head, _f32(key).ravel(),
                               _f32(value).ravel(), kv_heads, partial.reshape(-1), splits, pos)


def attention_combine(partial, head, pos):
    q_heads, splits, _ = partial.shape
    xb = np.empty((q_heads, head), np.float32)
    lib().or_attention_combine(_f32(partial).ravel(), q_heads, splits, head, xb.reshape(-1), pos)
    return xb


def attention(q, key, value, seq, pos):
    q_heads, head = q.shape
    kv_heads = key.shape[1]
    att = np.zeros((q_heads, seq), np.float32)
    xb = np.zeros((q_heads, head), np.float32)
    lib().or_attention(_f32(q).ravel(), q_heads, head, att.reshape(-1), seq, xb.reshape(-1),
                       _f32(key).ravel(), _f32(value).ravel(), kv_heads, pos)
    return xb


def swiglu(hb, hb2):
    hb = _f32(hb).copy()
    lib().or_swiglu(hb, _f32(hb2), hb.size)
    return hb


def add(a, b):
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    lib().or_add(a, b, out, a.size)
    return out


def cpu_attention_f64(q_heads, kv_heads, head, q, key, value, pos):
    """tests/kernels.rs:400-427."""
    out = np.empty(q_heads * head, np.float64)
    lib().or_cpu_attention_f64(q_heads, kv_heads, head, _f32(q).ravel(), _f32(key).ravel(),
                               _f32(value).ravel(), pos, out)
    return out


def sample_argmax(logits):
    logits = _f32(logits)
    return int(lib().or_sample_argmax(logits, logits.size))


def set_threads(n):
    lib().or_set_threads(int(n))


def get_threads():
    return int(lib().or_get_threads())


# --------------------------------------------------------------------------
# Model (composition of the modules; see oracle.c)
# --------------------------------------------------------------------------
WEIGHTS = {"embed": 0, "wcls": 1, "rms_final": 2, "rms_att": 3, "wq": 4, "wk": 5, "wv": 6,
           "wo": 7, "rms_ffn": 8, "w1": 9, "w2": 10, "w3": 11}


class Model:
    """Seeded synthetic Llama-shaped model and one decode state."""

    def __init__(self, dim, layers, heads, kv_heads, head_dim, hidden, vocab, seq,
                 theta=10000.0, eps=1e-5, bf16=False, seed=0, std=0.02):
        self.cfg = OrConfig(dim, layers, heads, kv_heads, head_dim, hidden, vocab, seq,
                            theta, eps, 1 if bf16 else 0)
        self.bf16 = bool(bf16)
        self.seed = seed
        self.std = std
        self._m = lib().or_model_create(C.byref(self.cfg), seed, std)
        self._s = lib().or_state_create(self._m)

    def close(self):
        states = getattr(self, "_states", {0: self._s})
        states[None] = self._s
        for h in {v for v in states.values() if v}:
            lib().or_state_destroy(h)
        self._states = {}
        self._s = None
        if self._m:
            lib().or_model_destroy(self._m)
            self._m = None

    def select_stream(self, k):
        """Make decode state k current (one KV cache per stream, sharing the weights); state
        0 is the one the model starts with, others are created zeroed on first use."""
        if not hasattr(self, "_states"):
            self._states = {0: self._s}
        if k not in self._states:
            self._states[k] = lib().or_state_create(self._m)
        self._s = self._states[k]

    def set_cache(self, layer, key, value):
        """Overwrite layer `layer` of the current state's K/V cache ([seq, kv_heads, head]:
        float32 values, or uint16 bf16 bits for a bf16 model)."""
        c = self.cfg
        per = c.seq * c.kv_heads * c.head_dim
        dt, ct = (np.uint16, C.c_uint16) if self.bf16 else (np.float32, C.c_float)
        for which, src in ((0, key), (1, value)):
            src = np.ascontiguousarray(src, dt).ravel()
            if src.size != per:
                raise ValueError(f"cache layer needs {per} elements, got {src.size}")
            ptr = lib().or_state_cache(self._s, which)
            dst = np.frombuffer((ct * (c.layers * per)).from_address(ptr), dt)
            dst[layer * per:(layer + 1) * per] = src

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        """Zero the current decode state (a new sequence)."""
        fresh = lib().or_state_create(self._m)
        states = getattr(self, "_states", None)
        if states is not None:
            for k, v in states.items():
                if v == self._s:
                    states[k] = fresh
        lib().or_state_destroy(self._s)
        self._s = fresh

    def weight(self, name, layer=0) -> np.ndarray:
        """Copy of one weight tensor: float32 for gains and fp32 models, uint16 bf16
        bits for bf16 linear/embedding weights."""
        c = self.cfg
        qd, kvd = c.heads * c.head_dim, c.kv_heads * c.head_dim
        shapes = {"embed": (c.vocab, c.dim), "wcls": (c.vocab, c.dim), "rms_final": (c.dim,),
                  "rms_att": (c.dim,), "rms_ffn": (c.dim,), "wq": (qd, c.dim),
                  "wk": (kvd, c.dim), "wv": (kvd, c.dim), "wo": (c.dim, qd),
                  "w1": (c.hidden, c.dim), "w2": (c.dim, c.hidden), "w3": (c.hidden, c.dim)}
        shape = shapes[name]
        n = int(np.prod(shape))
        ptr = lib().or_model_weight(self._m, WEIGHTS[name], layer)
        gain = name.startswith("rms")
        if self.bf16 and not gain:
            buf = (C.c_uint16 * n).from_address(ptr)
            return np.frombuffer(buf, np.uint16).reshape(shape).copy()
        buf = (C.c_float * n).from_address(ptr)
        return np.frombuffer(buf, np.float32).reshape(shape).copy()

    def step(self, token, pos) -> np.ndarray:
        p = lib().or_model_step(self._m, self._s, token, pos)
        return np.ctypeslib.as_array(p, shape=(self.cfg.vocab,)).copy()

    def tensor(self, which) -> np.ndarray:
        names = {"x": (0, self.cfg.dim), "xb": (1, self.cfg.dim),
                 "q": (2, self.cfg.heads * self.cfg.head_dim), "logits": (3, self.cfg.vocab),
                 "hb": (4, self.cfg.hidden)}
        idx, n = names[which]
        p = lib().or_state_tensor(self._s, idx)
        return np.ctypeslib.as_array(p, shape=(n,)).copy()

    def set_x(self, x):
        p = lib().or_state_tensor(self._s, 0)
        np.ctypeslib.as_array(p, shape=(self.cfg.dim,))[:] = _f32(x)

    def cache(self, value=False) -> np.ndarray:
        c = self.cfg
        shape = (c.layers, c.seq, c.kv_heads, c.head_dim)
        n = int(np.prod(shape))
        ptr = lib().or_state_cache(self._s, 1 if value else 0)
        if self.bf16:
            return from_bf16_bits(np.frombuffer((C.c_uint16 * n).from_address(ptr),
                                                np.uint16)).reshape(shape)
        return np.frombuffer((C.c_float * n).from_address(ptr), np.float32).reshape(shape).copy()

    def embed_token(self, token):
        lib().or_embed_token(self._m, self._s, token)

    def attention_block(self, layer, pos):
        lib().or_attention_block(self._m, self._s, layer, pos)

    def ffn_block(self, layer):
        lib().or_ffn_block(self._m, self._s, layer)

    def classify(self):
        lib().or_classify(self._m, self._s)
        return self.tensor("logits")

    def generate_tokens(self, prompt, max_new_tokens, stop_on=None, cap=None):
        """src/generate.rs:43-91. Returns (tokens, margins)."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        cap = cap or max(int(max_new_tokens), 1)
        out = np.zeros(cap, np.int32)
        margins = np.zeros(cap, np.float32)
        n = lib().or_generate_tokens(self._m, self._s, prompt, prompt.size, max_new_tokens,
                                     0 if stop_on is None else 1,
                                     0 if stop_on is None else int(stop_on), out, margins, cap)
        if n < 0:
            raise ValueError("expected at least one prompt token")
        n = min(n, cap)
        return out[:n].tolist(), margins[:n]
