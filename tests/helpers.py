"""Numeric helpers shared by the parity tests."""
import numpy as np

BLOCK = 32


def rel_err(y, ref, terms_abs):
    """Max relative error normalised by max(|ref|, sum|w'x| * 2^-10).

    The floor keeps outputs that cancel to nearly zero from turning an
    accumulation-order difference of ~1 ulp of the terms into a large ratio.
    """
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = np.maximum(np.abs(ref), np.asarray(terms_abs, np.float64) * 2.0 ** -10)
    denom = np.where(denom == 0, 1.0, denom)
    return float(np.max(np.abs(y - ref) / denom)) if y.size else 0.0


def dequant64(w, s):
    """Dequantized weights in float64 (exact products of the f32 values)."""
    w = np.asarray(w)
    rows, cols = w.shape
    sx = np.repeat(np.asarray(s, np.float64), BLOCK, axis=1)[:, :cols]
    return w.astype(np.float64) * sx


def terms_abs(w, s, x):
    """sum_k |w'_k x_k| per (batch row, output row)."""
    d = np.abs(dequant64(w, s))
    return np.abs(np.asarray(x, np.float64).reshape(-1, w.shape[1])) @ d.T


def bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and bool(np.all(a.view(np.uint32) == b.view(np.uint32)))


def random_q8(rng, rows, cols, lo=1e-4, hi=1e-2):
    """Config-0 style weights: int8 uniform in [-127, 127], scales U(lo, hi)."""
    w = rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)
    s = rng.uniform(lo, hi, size=(rows, (cols + BLOCK - 1) // BLOCK)).astype(np.float32)
    return w, s


def exact_linear(w, s, x):
    """The exact product of x with the fp32-dequantized weights (w * s rounded
    to fp32, as Int8Matrix::dequantize), computed in float64 and rounded once
    to fp32 (a result below fp32's range is 0, as any fp32 evaluation gives)."""
    w = np.asarray(w)
    wd = (w.astype(np.float32) * np.repeat(np.asarray(s, np.float32), BLOCK, axis=1)[:, :w.shape[1]]
          ).astype(np.float64)
    return (np.asarray(x, np.float64).reshape(-1, w.shape[1]) @ wd.T).astype(np.float32)
