"""Tensor-core path of linear_dynamic_int8 for many rows (csrc/q8_tc.cu).

The reference applies Int8Matrix::linear_dynamic_int8 (src/cpu/quantized.rs:
155-236) row by row; the tensor-core kernel must reproduce it bit for bit:
exact int32 block sums, then ((float)S * ws) * xs added block by block from
-0.0.  Shapes: BASELINE config 3 (M in {1,16,128,512}, N in {896,1280,3840},
K = 1280) and ragged edges (M not a multiple of the 64-row tile, one 128-row
weight tile, K of one stage).
"""
import numpy as np
import pytest

import oracle
from helpers import bits_equal, random_q8

pytestmark = pytest.mark.gpu


def run_device(ctx, w, s, x):
    import torch

    import uocr_q8
    m = uocr_q8.Int8Matrix.from_parts(w.shape[0], w.shape[1], w, s, ctx)
    y = m.linear_device(torch.from_numpy(np.ascontiguousarray(x)).cuda(), dynamic=True)
    ctx.sync()
    return y.cpu().numpy()


@pytest.mark.parametrize("batch", [2, 16, 63, 64, 65, 128, 200])
@pytest.mark.parametrize("rows,cols", [(128, 128), (896, 1280), (256, 896)])
def test_tc_dynamic_bit_exact(ctx, rows, cols, batch):
    rng = np.random.default_rng(rows * 7 + cols + batch)
    w, s = random_q8(rng, rows, cols)
    x = (rng.standard_normal((batch, cols)) * rng.uniform(0.1, 10, (batch, 1))).astype(np.float32)
    assert bits_equal(run_device(ctx, w, s, x), oracle.linear_dynamic_int8(oracle.Matrix(w, s), x))


@pytest.mark.parametrize("rows", [896, 1280, 3840])
@pytest.mark.parametrize("batch", [16, 128, 512])
def test_tc_config3_shapes(ctx, rows, batch):
    rng = np.random.default_rng(rows + batch)
    w, s = random_q8(rng, rows, 1280)
    x = (rng.standard_normal((batch, 1280)) * rng.uniform(0.1, 10, (batch, 1))).astype(np.float32)
    assert bits_equal(run_device(ctx, w, s, x), oracle.linear_dynamic_int8(oracle.Matrix(w, s), x))


def test_tc_extremes_zero_rows_and_denormal_scales(ctx):
    """+-127 weight patterns (src/cpu/neon.rs:245-276), an all-zero activation
    row (zero scales: the sum stays -0.0 + ...), and 1e-20 weight scales whose
    products are subnormal (no flushing anywhere)."""
    rows, cols, batch = 256, 1280, 70
    i = np.arange(rows * cols).reshape(rows, cols)
    w = ((i * 53) % 255 - 127).astype(np.int8)
    s = np.full((rows, cols // 32), 1e-20, np.float32)
    s[::3] = 0.7
    s[1::7] = 17.0
    x = np.cos(np.arange(batch * cols, dtype=np.float64) * 0.37).reshape(batch, cols).astype(np.float32)
    x[5] = 0.0
    x[9] *= 1e-30
    assert bits_equal(run_device(ctx, w, s, x), oracle.linear_dynamic_int8(oracle.Matrix(w, s), x))
