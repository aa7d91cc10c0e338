"""Generate tests/golden/quantize_golden.npz from the reference's own quantizer.

The reference's Python tool ``tools/quantize.py`` (``quantize_blocks``,
tools/quantize.py:19-34) is the reference's executable statement of q8-block32
quantization: the same per-block max/127 scale, IEEE float32 division and
round-half-to-even as ``Int8Matrix::quantize`` (src/cpu/quantized.rs:43-74).
This script imports it from a checkout of the reference and records its
outputs for a set of seeded inputs, so the oracle and the CUDA kernels can be
pinned to it on machines where the reference is absent.

Usage:  python tests/golden/make_golden.py --reference <reference checkout>
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def cases(rng: np.random.Generator):
    """Seeded inputs: tails, zero rows, ties, denormals, extremes."""
    out = {}
    # tests/python/test_quantize.py:9-11
    x = np.arange(105, dtype=np.float32).reshape(3, 35) / 37 - 1
    x[0] = 0
    out["ref_test_tails"] = x
    for cols in (1, 15, 31, 32, 33, 131, 513, 1280):
        rows = 5 if cols > 200 else 7
        v = rng.standard_normal((rows, cols)) * rng.uniform(0.1, 10.0, (rows, 1))
        out[f"normal_cols{cols}"] = v.astype(np.float32)
    # exact ties: block max 127 gives scale 1, so k + 0.5 lands on a tie
    t = np.array([127.0, 2.5, -3.5, 0.5, -0.5, 1.5, -1.5, 126.5, -126.5] + [4.5] * 23,
                 np.float32)[None, :]
    out["ties"] = t
    # denormal block (scale stays nonzero), huge values, signed zeros
    d = np.zeros((3, 64), np.float32)
    d[0, :32] = np.float32(1e-38) * rng.uniform(-1, 1, 32).astype(np.float32)
    d[0, 32:] = np.float32(3e-43) * np.sign(rng.uniform(-1, 1, 32)).astype(np.float32)
    d[1, :] = rng.uniform(-3e38, 3e38, 64).astype(np.float32)
    d[2, :] = -0.0
    d[2, 5] = 1e-30
    out["extremes"] = d
    # config-3 style activation rows (N(0,1) * U(0.1,10)), K=1280
    a = rng.standard_normal((16, 1280)) * rng.uniform(0.1, 10.0, (16, 1))
    out["activations_k1280"] = a.astype(np.float32)
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, help="reference checkout (contains tools/)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from tools.quantize import quantize_blocks  # the reference's own implementation

    rng = np.random.default_rng(20261201)
    arrays = {}
    names = []
    for name, x in cases(rng).items():
        q, s = quantize_blocks(x)
        arrays[f"{name}__x"] = x
        arrays[f"{name}__q"] = q
        arrays[f"{name}__s"] = np.asarray(s, np.float32)
        names.append(name)
    # scale underflow: the reference quantizer must reject it
    under = np.full((1, 8), np.float32(1e-44))
    try:
        quantize_blocks(under)
        raise SystemExit("reference accepted an underflowing block")
    except ValueError:
        arrays["underflow__x"] = under
    arrays["names"] = np.array(names)
    path = os.path.join(HERE, "quantize_golden.npz")
    np.savez_compressed(path, **arrays)
    print(f"wrote {path}: {len(names)} cases")


if __name__ == "__main__":
    main()
