"""ctypes view of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference legs of bench.py. The product package never imports
this module.

Each wrapper takes numpy arrays, passes their true lengths (the reference
kernels validate slice lengths) and raises OracleError carrying the
KernelError variant (crates/backends/backend-cpu/src/reference/mod.rs:44-61).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

OK, LENGTH_MISMATCH, SHAPE_OVERFLOW, INVALID_SHAPE, UNSUPPORTED = range(5)
INT4, INT8 = 0, 1
ROLES = ("embed", "attn_norm", "q", "k", "v", "o", "mlp_norm", "gate", "up",
         "down", "final_norm", "lm_head")
LAYER_ROLES = ROLES[1:10]


class OracleError(Exception):
    def __init__(self, code, expected=0, actual=0, reason=None):
        self.code = code
        self.expected = expected
        self.actual = actual
        self.reason = reason
        names = {1: "LengthMismatch", 2: "ShapeOverflow", 3: "InvalidShape", 4: "Unsupported"}
        super().__init__(f"{names.get(code, code)}: {reason or ''} (expected={expected}, actual={actual})")


class _Err(C.Structure):
    _fields_ = [("code", C.c_int), ("expected", C.c_size_t), ("actual", C.c_size_t),
                ("reason", C.c_char_p)]


class _Lcg(C.Structure):
    _fields_ = [("state", C.c_uint64)]


class LlamaConfig(C.Structure):
    _fields_ = [("layers", C.c_uint32), ("hidden", C.c_uint32), ("heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("inter", C.c_uint32),
                ("vocab", C.c_uint32), ("max_seq", C.c_uint32), ("batch", C.c_uint32),
                ("eps", C.c_float), ("theta", C.c_float), ("quant_format", C.c_int),
                ("group_size", C.c_uint32)]


def build():
    """Compile liboracle.so from the C sources (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = C.CDLL(_LIB_PATH)
        _lib.orc_lcg_next_u32.restype = C.c_uint32
        _lib.orc_lcg_uniform.restype = C.c_float
        _lib.orc_lcg_uniform.argtypes = [C.POINTER(_Lcg), C.c_float, C.c_float]
        _lib.orc_lcg_normal.restype = C.c_float
        _lib.orc_lcg_normal.argtypes = [C.POINTER(_Lcg), C.c_float, C.c_float]
        _lib.orc_lcg_below.restype = C.c_size_t
        _lib.orc_lcg_below.argtypes = [C.POINTER(_Lcg), C.c_size_t]
        _lib.orc_lcg_fill.argtypes = [C.POINTER(_Lcg), C.c_void_p, C.c_size_t, C.c_float, C.c_float]
        _lib.orc_lcg_fill_normal.argtypes = [C.POINTER(_Lcg), C.c_void_p, C.c_size_t, C.c_float, C.c_float]
        _lib.orc_silu_scalar.restype = C.c_float
        _lib.orc_silu_scalar.argtypes = [C.c_float]
        _lib.orc_quant_row_bytes.restype = C.c_size_t
        _lib.orc_quant_groups.restype = C.c_size_t
        _lib.orc_quant_row_bytes.argtypes = [C.c_int, C.c_size_t]
        _lib.orc_quant_groups.argtypes = [C.c_size_t, C.c_size_t]
        _lib.orc_llama_create.restype = C.c_void_p
        _lib.orc_llama_create.argtypes = [C.POINTER(LlamaConfig)]
        _lib.orc_llama_destroy.argtypes = [C.c_void_p]
        _lib.orc_llama_weight_len.restype = C.c_size_t
        _lib.orc_llama_weight_len.argtypes = [C.c_void_p, C.c_int, C.c_uint32]
        _lib.orc_llama_weight.restype = C.POINTER(C.c_float)
        _lib.orc_llama_weight.argtypes = [C.c_void_p, C.c_int, C.c_uint32]
        _lib.orc_llama_weight_source.restype = C.POINTER(C.c_float)
        _lib.orc_llama_weight_source.argtypes = [C.c_void_p, C.c_int, C.c_uint32]
        _lib.orc_llama_codes.restype = C.POINTER(C.c_uint8)
        _lib.orc_llama_codes.argtypes = [C.c_void_p, C.c_int, C.c_uint32]
        _lib.orc_llama_scales.restype = C.POINTER(C.c_float)
        _lib.orc_llama_scales.argtypes = [C.c_void_p, C.c_int, C.c_uint32]
        _lib.orc_llama_init_random.argtypes = [C.c_void_p, C.c_uint64, C.c_float]
        _lib.orc_llama_step.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32,
                                        C.c_uint32, C.c_void_p, C.POINTER(_Err)]
        _lib.orc_llama_reset_cache.argtypes = [C.c_void_p]
        _lib.orc_llama_cache.restype = C.POINTER(C.c_float)
        _lib.orc_llama_cache.argtypes = [C.c_void_p, C.POINTER(C.c_size_t)]
        _lib.orc_argmax.restype = C.c_uint32
        _lib.orc_argmax.argtypes = [C.c_void_p, C.c_size_t]
        _lib.orc_set_threads.argtypes = [C.c_int]
    return _lib


def set_threads(n: int):
    lib().orc_set_threads(int(n))


# ---------------------------------------------------------------- LCG ------

class Lcg:
    """Deterministic LCG of reference/mod.rs:118-148 (plus a Box-Muller normal)."""

    def __init__(self, seed: int):
        self._s = _Lcg(seed & 0xFFFFFFFFFFFFFFFF)

    def next_u32(self) -> int:
        return lib().orc_lcg_next_u32(C.byref(self._s))

    def uniform(self, low, high) -> float:
        return lib().orc_lcg_uniform(C.byref(self._s), low, high)

    def below(self, upper: int) -> int:
        return lib().orc_lcg_below(C.byref(self._s), upper)

    def fill(self, n: int, low: float, high: float) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib().orc_lcg_fill(C.byref(self._s), out.ctypes.data, n, low, high)
        return out

    def normal(self, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib().orc_lcg_fill_normal(C.byref(self._s), out.ctypes.data, n, mean, std)
        return out


# ------------------------------------------------------------- kernels -----

def _f(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data, a.size


def _u(a):
    a = np.ascontiguousarray(a, dtype=np.uint32)
    return a, a.ctypes.data, a.size


def _check(rc, err):
    if rc != OK:
        raise OracleError(rc, err.expected, err.actual,
                          err.reason.decode() if err.reason else None)


def _call(name, *args):
    err = _Err()
    fn = getattr(lib(), name)
    conv = []
    for a in args:
        if isinstance(a, float):
            conv.append(C.c_float(a))
        elif isinstance(a, int):
            conv.append(C.c_size_t(a))
        else:
            conv.append(C.c_void_p(a))
    fn.restype = C.c_int
    _check(fn(*conv, C.byref(err)), err)


def matmul_nt(a, b, batch, m, k, n, out_len=None):
    a, pa, la = _f(a); b, pb, lb = _f(b)
    out = np.zeros(batch * m * n if out_len is None else out_len, np.float32)
    _call("orc_matmul_nt", pa, la, pb, lb, out.ctypes.data, out.size, batch, m, k, n)
    return out


def matmul_nn(a, b, batch, m, k, n, out_len=None):
    a, pa, la = _f(a); b, pb, lb = _f(b)
    out = np.zeros(batch * m * n if out_len is None else out_len, np.float32)
    _call("orc_matmul_nn", pa, la, pb, lb, out.ctypes.data, out.size, batch, m, k, n)
    return out


def softmax(x, rows, cols):
    x = np.array(x, dtype=np.float32, copy=True)
    _call("orc_softmax", x.ctypes.data, x.size, rows, cols)
    return x


def softmax_causal(x, rows, cols, seq, past_len):
    x = np.array(x, dtype=np.float32, copy=True)
    _call("orc_softmax_causal", x.ctypes.data, x.size, rows, cols, seq, past_len)
    return x


def rms_norm(x, weight, rows, hidden, eps, out_len=None):
    x, px, lx = _f(x); w, pw, lw = _f(weight)
    out = np.zeros(rows * hidden if out_len is None else out_len, np.float32)
    _call("orc_rms_norm", px, lx, pw, lw, out.ctypes.data, out.size, rows, hidden, float(eps))
    return out


def rope(x, positions, batch, heads, seq, head_dim, theta, variant="neox"):
    x = np.array(x, dtype=np.float32, copy=True)
    p, pp, lp = _u(positions)
    name = "orc_rope_neox" if variant == "neox" else "orc_rope_gptj"
    _call(name, x.ctypes.data, x.size, pp, lp, batch, heads, seq, head_dim, float(theta))
    return x


def silu(x):
    x = np.array(x, dtype=np.float32, copy=True)
    _call("orc_silu", x.ctypes.data, x.size)
    return x


def mul(a, b, length, out_len=None):
    a, pa, la = _f(a); b, pb, lb = _f(b)
    out = np.zeros(length if out_len is None else out_len, np.float32)
    _call("orc_mul", pa, la, pb, lb, out.ctypes.data, out.size, length)
    return out


def add(a, b, length, out_len=None):
    a, pa, la = _f(a); b, pb, lb = _f(b)
    out = np.zeros(length if out_len is None else out_len, np.float32)
    _call("orc_add", pa, la, pb, lb, out.ctypes.data, out.size, length)
    return out


def scale(x, factor):
    x = np.array(x, dtype=np.float32, copy=True)
    _call("orc_scale", x.ctypes.data, x.size, float(factor))
    return x


def gather(table, ids, vocab, hidden, rows, out=None):
    t, pt, lt = _f(table); i, pi, li = _u(ids)
    if out is None:
        out = np.zeros(rows * hidden, np.float32)
    _call("orc_gather", pt, lt, pi, li, out.ctypes.data, out.size, vocab, hidden, rows)
    return out


def last_token(x, batch, seq, hidden, seq_len, out_len=None):
    x, px, lx = _f(x)
    out = np.zeros(batch * hidden if out_len is None else out_len, np.float32)
    _call("orc_last_token", px, lx, out.ctypes.data, out.size, batch, seq, hidden, seq_len)
    return out


def split_heads(x, batch, seq, heads, head_dim, out_len=None):
    x, px, lx = _f(x)
    out = np.zeros(batch * seq * heads * head_dim if out_len is None else out_len, np.float32)
    _call("orc_split_heads", px, lx, out.ctypes.data, out.size, batch, seq, heads, head_dim)
    return out


def merge_heads(x, batch, seq, heads, head_dim, out_len=None):
    x, px, lx = _f(x)
    out = np.zeros(batch * seq * heads * head_dim if out_len is None else out_len, np.float32)
    _call("orc_merge_heads", px, lx, out.ctypes.data, out.size, batch, seq, heads, head_dim)
    return out


def kv_append(k, v, cache, batch, layers, layer, kv_heads, head_dim, max_seq, past_len, seq):
    k, pk, lk = _f(k); v, pv, lv = _f(v)
    cache = np.array(cache, dtype=np.float32, copy=True)
    _call("orc_kv_append", pk, lk, pv, lv, cache.ctypes.data, cache.size, batch, layers,
          layer, kv_heads, head_dim, max_seq, past_len, seq)
    return cache


def causal_attention(q, k, v, cache, batch, layers, layer, heads, kv_heads, seq, past_len,
                     head_dim, max_seq, scale_, out_len=None):
    q, pq, lq = _f(q); k, pk, lk = _f(k); v, pv, lv = _f(v)
    cache = np.array(cache, dtype=np.float32, copy=True)
    out = np.zeros(batch * heads * seq * head_dim if out_len is None else out_len, np.float32)
    _call("orc_causal_attention", pq, lq, pk, lk, pv, lv, cache.ctypes.data, cache.size,
          out.ctypes.data, out.size, batch, layers, layer, heads, kv_heads, seq, past_len,
          head_dim, max_seq, float(scale_))
    return out, cache


def swiglu(x, w_gate, w_up, w_down, rows, hidden, inter, out_len=None):
    x, px, lx = _f(x); g, pg, lg = _f(w_gate); u, pu, lu = _f(w_up); d, pd, ld = _f(w_down)
    out = np.zeros(rows * hidden if out_len is None else out_len, np.float32)
    _call("orc_swiglu", px, lx, pg, lg, pu, lu, pd, ld, out.ctypes.data, out.size, rows,
          hidden, inter)
    return out


def rms_norm_matmul(x, weight, w, rows, hidden, out_features, eps, out_len=None):
    x, px, lx = _f(x); g, pg, lg = _f(weight); w, pw, lw = _f(w)
    out = np.zeros(rows * out_features if out_len is None else out_len, np.float32)
    _call("orc_rms_norm_matmul", px, lx, pg, lg, pw, lw, out.ctypes.data, out.size, rows,
          hidden, out_features, float(eps))
    return out


# --------------------------------------------------------- quantization ----

def quant_row_bytes(fmt, k):
    return lib().orc_quant_row_bytes(fmt, k)


def quant_groups(k, group):
    return lib().orc_quant_groups(k, group)


def quantize(fmt, w, n, k, group):
    w, pw, _ = _f(w)
    codes = np.zeros(n * quant_row_bytes(fmt, k), np.uint8)
    scales = np.zeros(n * quant_groups(k, group), np.float32)
    err = _Err()
    fn = lib().orc_quantize
    fn.argtypes = [C.c_int, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_void_p,
                   C.c_void_p, C.POINTER(_Err)]
    _check(fn(fmt, pw, n, k, group, codes.ctypes.data, scales.ctypes.data, C.byref(err)), err)
    return codes, scales


def dequantize(fmt, codes, scales, n, k, group):
    codes = np.ascontiguousarray(codes, np.uint8)
    scales = np.ascontiguousarray(scales, np.float32)
    w = np.zeros(n * k, np.float32)
    err = _Err()
    fn = lib().orc_dequantize
    fn.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t,
                   C.c_void_p, C.POINTER(_Err)]
    _check(fn(fmt, codes.ctypes.data, scales.ctypes.data, n, k, group, w.ctypes.data,
              C.byref(err)), err)
    return w


def codes_as_int(fmt, codes, n, k):
    """Unpack a payload to int32 codes [n, k]."""
    codes = np.ascontiguousarray(codes, np.uint8)
    if fmt == INT8:
        return codes.reshape(n, k).view(np.int8).astype(np.int32)
    rb = quant_row_bytes(fmt, k)
    rows = codes.reshape(n, rb)
    lo = (rows & 0xF).astype(np.int32)
    hi = (rows >> 4).astype(np.int32)
    out = np.empty((n, 2 * rb), np.int32)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    out = np.where(out >= 8, out - 16, out)
    return out[:, :k]


# -------------------------------------------------------------- llama -------

class Llama:
    """The llama-dense fixture executed through the restated reference kernels."""

    def __init__(self, cfg: LlamaConfig):
        self.cfg = cfg
        self._p = lib().orc_llama_create(C.byref(cfg))

    def __del__(self):
        if getattr(self, "_p", None):
            lib().orc_llama_destroy(self._p)
            self._p = None

    def init_random(self, seed, std=0.02):
        lib().orc_llama_init_random(self._p, seed, std)

    def weight(self, role, layer=0) -> np.ndarray:
        r = ROLES.index(role)
        n = lib().orc_llama_weight_len(self._p, r, layer)
        return np.ctypeslib.as_array(lib().orc_llama_weight(self._p, r, layer), (n,)).copy()

    def weight_source(self, role, layer=0) -> np.ndarray:
        """The weight before quantization (equal to weight() for dense roles)."""
        r = ROLES.index(role)
        n = lib().orc_llama_weight_len(self._p, r, layer)
        return np.ctypeslib.as_array(lib().orc_llama_weight_source(self._p, r, layer), (n,)).copy()

    def codes(self, role, layer, nbytes) -> np.ndarray:
        r = ROLES.index(role)
        return np.ctypeslib.as_array(lib().orc_llama_codes(self._p, r, layer), (nbytes,)).copy()

    def scales(self, role, layer, count) -> np.ndarray:
        r = ROLES.index(role)
        return np.ctypeslib.as_array(lib().orc_llama_scales(self._p, r, layer), (count,)).copy()

    def reset(self):
        lib().orc_llama_reset_cache(self._p)

    def cache(self) -> np.ndarray:
        n = C.c_size_t()
        ptr = lib().orc_llama_cache(self._p, C.byref(n))
        return np.ctypeslib.as_array(ptr, (n.value,)).copy()

    def step(self, ids, positions, seq, past_len) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32)
        positions = np.ascontiguousarray(positions, np.uint32)
        logits = np.zeros(self.cfg.batch * self.cfg.vocab, np.float32)
        err = _Err()
        _check(lib().orc_llama_step(self._p, ids.ctypes.data, positions.ctypes.data, seq,
                                    past_len, logits.ctypes.data, C.byref(err)), err)
        return logits

    def generate(self, prompt, steps):
        """Prefill the prompt, then `steps` greedy decode steps (batch 1).

        Returns the 1 + steps greedy ids (one after the prefill, one after each
        decode step) and the logits of every step."""
        self.reset()
        prompt = np.asarray(prompt, np.uint32)
        t = len(prompt)
        logits = self.step(prompt, np.arange(t, dtype=np.uint32), t, 0)
        all_logits = [logits]
        nxt = argmax(logits)
        out_ids = [nxt]
        for s in range(steps):
            logits = self.step(np.array([nxt], np.uint32), np.array([t + s], np.uint32), 1, t + s)
            all_logits.append(logits)
            nxt = argmax(logits)
            out_ids.append(nxt)
        return out_ids, all_logits


def argmax(row) -> int:
    row = np.ascontiguousarray(row, np.float32)
    return int(lib().orc_argmax(row.ctypes.data, row.size))
