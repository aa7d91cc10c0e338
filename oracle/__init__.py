"""numpy front end of the CPU oracle (libq8_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / ``--impl reference`` legs of bench.py, always as the checker or
the timed CPU baseline, never by the product path.  Each function restates the
reference's scalar Rust path; the file:line it follows is cited in
q8_oracle.h.  Errors come back as ``OracleError`` carrying the reference's
OcrError variant name.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libq8_oracle.so")

BLOCK = 32
WEIGHTS_ONLY, DYNAMIC, DYNAMIC_ROWWISE = 0, 1, 2
ERROR_NAMES = {1: "Io", 2: "Json", 3: "Format", 4: "Shape", 5: "Unsupported", 6: "Resource",
               7: "Numerical"}


class OracleError(RuntimeError):
    def __init__(self, code: int):
        super().__init__(ERROR_NAMES.get(code, f"status {code}"))
        self.code = code
        self.kind = ERROR_NAMES.get(code, "Unknown")


def build() -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


class _Mat(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_size_t), ("cols", ctypes.c_size_t),
                ("w", ctypes.c_void_p), ("s", ctypes.c_void_p)]


class _Ffn(ctypes.Structure):
    _fields_ = [("gate", _Mat), ("up", _Mat), ("down", _Mat)]


def _declare(L):
    P, S = ctypes.c_void_p, ctypes.c_size_t
    I, F = ctypes.c_int, ctypes.c_float
    sig = {
        "q8o_set_threads": (None, [I]),
        "q8o_get_threads": (I, []),
        "q8o_from_parts_check": (I, [S, S, S, S, P]),
        "q8o_quantize": (I, [S, S, P, P, P]),
        "q8o_dequantize": (None, [S, S, P, P, P]),
        "q8o_linear": (I, [P, P, S, P]),
        "q8o_linear_dynamic_int8": (I, [P, P, P]),
        "q8o_linear_dynamic_int8_rows": (I, [P, P, S, P]),
        "q8o_block_sums": (None, [P, P, S, P]),
        "q8o_softmax": (I, [P, S]),
        "q8o_route": (I, [P, S, S, I, F, P, P]),
        "q8o_silu": (None, [P, S]),
        "q8o_linear_bf16": (I, [P, S, S, P, S, P]),
        "q8o_feed_forward": (I, [P, P, S, I, P]),
        "q8o_experts": (I, [P, P, S, P, P, S, S, S, I, F, I, P, P, P]),
        "q8o_rms_norm": (I, [P, S, S, P, F, P]),
        "q8o_rope": (I, [P, S, S, S, F]),
        "q8o_attention_decode": (I, [P, S, P, S, P, S, S, P]),
        "q8o_attention": (I, [P, S, S, S, P, P, S, I, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _check(code: int):
    if code:
        raise OracleError(code)


def set_threads(n: int) -> None:
    lib().q8o_set_threads(int(n))


def get_threads() -> int:
    return int(lib().q8o_get_threads())


@dataclass
class Matrix:
    """Host copy of an Int8Matrix (src/cpu/quantized.rs:11-16)."""
    w: np.ndarray  # int8 [rows, cols]
    s: np.ndarray  # float32 [rows, ceil(cols/32)]

    @property
    def rows(self) -> int:
        return int(self.w.shape[0])

    @property
    def cols(self) -> int:
        return int(self.w.shape[1])

    def _c(self) -> _Mat:
        return _Mat(self.rows, self.cols, self.w.ctypes.data, self.s.ctypes.data)


def _contig(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def from_parts_check(rows, cols, w, s) -> int:
    w = _contig(w, np.int8)
    s = _contig(s, np.float32)
    return int(lib().q8o_from_parts_check(rows, cols, w.size, s.size, _ptr(s)))


def quantize(x) -> Matrix:
    x = _contig(x, np.float32)
    if x.ndim != 2:
        raise OracleError(4)
    rows, cols = x.shape
    w = np.zeros((rows, cols), np.int8)
    s = np.zeros((rows, (cols + BLOCK - 1) // BLOCK), np.float32)
    _check(lib().q8o_quantize(rows, cols, _ptr(x), _ptr(w), _ptr(s)))
    return Matrix(w, s)


def dequantize(m: Matrix) -> np.ndarray:
    out = np.empty((m.rows, m.cols), np.float32)
    lib().q8o_dequantize(m.rows, m.cols, _ptr(m.w), _ptr(m.s), _ptr(out))
    return out


def linear(m: Matrix, x) -> np.ndarray:
    x = _contig(x, np.float32)
    batch = x.size // m.cols
    y = np.empty((batch, m.rows), np.float32)
    c = m._c()
    _check(lib().q8o_linear(ctypes.byref(c), _ptr(x), batch, _ptr(y)))
    return y


def linear_dynamic_int8(m: Matrix, x) -> np.ndarray:
    x = _contig(x, np.float32).reshape(-1, m.cols)
    y = np.empty((x.shape[0], m.rows), np.float32)
    c = m._c()
    _check(lib().q8o_linear_dynamic_int8_rows(ctypes.byref(c), _ptr(x), x.shape[0], _ptr(y)))
    return y


def block_sums(w_row, xq) -> np.ndarray:
    w_row = _contig(w_row, np.int8)
    xq = _contig(xq, np.int8)
    out = np.empty(((w_row.size + BLOCK - 1) // BLOCK,), np.int32)
    lib().q8o_block_sums(_ptr(w_row), _ptr(xq), w_row.size, _ptr(out))
    return out


def softmax(v) -> np.ndarray:
    v = np.array(v, dtype=np.float32, copy=True)
    _check(lib().q8o_softmax(_ptr(v), v.size))
    return v


def route(logits, count: int, normalize: bool = False, scale: float = 1.0):
    logits = _contig(logits, np.float32)
    ids = np.empty((max(count, 0),), np.int32)
    wts = np.empty((max(count, 0),), np.float32)
    _check(lib().q8o_route(_ptr(logits), logits.size, count, int(bool(normalize)),
                           float(scale), _ptr(ids), _ptr(wts)))
    return [(int(i), float(w)) for i, w in zip(ids, wts)]


def silu(v) -> np.ndarray:
    v = np.array(v, dtype=np.float32, copy=True)
    lib().q8o_silu(_ptr(v), v.size)
    return v


def linear_bf16(w_bf16, x) -> np.ndarray:
    w = _contig(w_bf16, np.uint16)
    n, k = w.shape
    x = _contig(x, np.float32).reshape(-1, k)
    y = np.empty((x.shape[0], n), np.float32)
    _check(lib().q8o_linear_bf16(_ptr(w), n, k, _ptr(x), x.shape[0], _ptr(y)))
    return y


@dataclass
class Ffn:
    gate: Matrix
    up: Matrix
    down: Matrix

    def _c(self) -> _Ffn:
        return _Ffn(self.gate._c(), self.up._c(), self.down._c())


def feed_forward(f: Ffn, x, mode: int = WEIGHTS_ONLY) -> np.ndarray:
    x = _contig(x, np.float32).reshape(-1, f.gate.cols)
    out = np.empty((x.shape[0], f.down.rows), np.float32)
    c = f._c()
    _check(lib().q8o_feed_forward(ctypes.byref(c), _ptr(x), x.shape[0], mode, _ptr(out)))
    return out


def experts(shared: Ffn, routed: list, logits, x, top_k: int, mode: int = WEIGHTS_ONLY,
            normalize: bool = False, scale: float = 1.0):
    """Decoder::experts given router logits; returns (out, ids, weights)."""
    x = _contig(x, np.float32)
    tokens, hidden = x.shape
    logits = _contig(logits, np.float32).reshape(tokens, len(routed))
    arr = (_Ffn * len(routed))(*[f._c() for f in routed])
    sc = shared._c()
    out = np.empty((tokens, hidden), np.float32)
    ids = np.empty((tokens, top_k), np.int32)
    wts = np.empty((tokens, top_k), np.float32)
    _check(lib().q8o_experts(ctypes.byref(sc), arr, len(routed), _ptr(logits), _ptr(x), tokens,
                             hidden, top_k, int(bool(normalize)), float(scale), mode, _ptr(out),
                             _ptr(ids), _ptr(wts)))
    return out, ids, wts


def rms_norm(x, weight, eps: float = 1e-6) -> np.ndarray:
    """ops::rms_norm over the last dimension."""
    x = _contig(x, np.float32)
    w = _contig(weight, np.float32)
    width = x.shape[-1] if x.ndim else 0
    out = np.empty_like(x)
    rows = x.size // width if width else 0
    _check(lib().q8o_rms_norm(_ptr(x), rows, width, _ptr(w), float(eps), _ptr(out)))
    return out


def rope(values, head_dim: int, position: int, theta: float = 10000.0) -> np.ndarray:
    """ops::rope of one row (every head) at one position; returns a copy."""
    v = np.array(values, dtype=np.float32, copy=True)
    _check(lib().q8o_rope(_ptr(v), v.size, head_dim, position, float(theta)))
    return v


def attention_decode(q, keys, values, heads: int) -> np.ndarray:
    """ops::attention_decode: q [width] over token-major keys/values."""
    q = _contig(q, np.float32).reshape(-1)
    k = _contig(keys, np.float32).reshape(-1)
    v = _contig(values, np.float32).reshape(-1)
    out = np.empty_like(q)
    _check(lib().q8o_attention_decode(_ptr(q), q.size, _ptr(k), k.size, _ptr(v), v.size, heads,
                                      _ptr(out)))
    return out


def attention(q, k, v, causal: bool = True) -> np.ndarray:
    """ops::attention: q [heads, nq, dim] over k, v [heads, nk, dim]."""
    q = _contig(q, np.float32)
    k = _contig(k, np.float32)
    v = _contig(v, np.float32)
    heads, nq, dim = q.shape
    if k.shape != v.shape or k.ndim != 3 or k.shape[0] != heads or k.shape[2] != dim:
        raise OracleError(4)
    out = np.empty_like(q)
    _check(lib().q8o_attention(_ptr(q), heads, nq, dim, _ptr(k), _ptr(v), k.shape[1],
                               int(bool(causal)), _ptr(out)))
    return out


def attention_prefill(q, keys, values, heads: int) -> np.ndarray:
    """The prefill branch of Decoder::layer (src/decoder/mod.rs:313-338):
    token-major q, keys, values [tokens x width] split into heads, causal
    ops::attention, joined back to token-major rows."""
    q = _contig(q, np.float32)
    tokens, width = q.shape
    dim = width // heads

    def split(a):
        return np.ascontiguousarray(
            _contig(a, np.float32).reshape(-1, heads, dim).transpose(1, 0, 2))

    out = attention(split(q), split(keys), split(values), True)
    return np.ascontiguousarray(out.transpose(1, 0, 2).reshape(tokens, width))


class LayerCache:
    """LayerCache (src/decoder/cache.rs:3-95): token-major keys/values, an
    immutable prefix followed by a ring of `window` tokens."""

    def __init__(self, heads: int, head_dim: int, window: int):
        if heads * head_dim <= 0:
            raise OracleError(4)
        if window == 0:
            raise OracleError(4)
        self.width, self.window = heads * head_dim, window
        self.prefix = None
        self.generated = 0
        self.keys = np.zeros((0, self.width), np.float32)
        self.values = np.zeros((0, self.width), np.float32)

    def prefill(self, keys, values, tokens: int) -> None:
        keys = _contig(keys, np.float32).reshape(-1)
        values = _contig(values, np.float32).reshape(-1)
        if self.prefix is not None or tokens == 0 or tokens * self.width != keys.size or \
                keys.size != values.size:
            raise OracleError(4)
        self.keys = keys.reshape(tokens, self.width).copy()
        self.values = values.reshape(tokens, self.width).copy()
        self.prefix = tokens

    def push(self, key, value) -> None:
        if self.prefix is None:
            raise OracleError(4)
        key = _contig(key, np.float32).reshape(-1)
        value = _contig(value, np.float32).reshape(-1)
        if key.size != self.width or value.size != self.width:
            raise OracleError(4)
        if self.generated < self.window:
            self.keys = np.vstack([self.keys, key[None]])
            self.values = np.vstack([self.values, value[None]])
        else:
            slot = self.prefix + self.generated % self.window
            self.keys[slot] = key
            self.values[slot] = value
        self.generated += 1

    def tokens(self) -> int:
        return self.keys.shape[0]

    def position(self) -> int:
        return (self.prefix or 0) + self.generated
