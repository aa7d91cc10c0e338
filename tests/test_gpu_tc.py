"""Tensor-core paths of Int8Matrix for several rows (csrc/q8_tc.cu for more
than 16 rows, csrc/q8_small.cu for 2..16).

int8 activations: the reference applies Int8Matrix::linear_dynamic_int8
(src/cpu/quantized.rs:155-236) row by row; the tensor-core kernel must
reproduce it bit for bit: exact int32 block sums, then ((float)S * ws) * xs
added block by block from -0.0.  Shapes: the int8 micro-suite (M in
{1,16,128,512}, N in {896,1280,3840}, K = 1280) and ragged edges (M not a
multiple of the 64-row tile, one 128-row weight tile, K of one stage).

FP32 activations: Int8Matrix::linear (src/cpu/quantized.rs:101-153) for
batches of 8 rows or more runs on the tensor cores with exact bf16 pieces of
the activations.  Tolerance (helpers.rel_err: max relative error normalised
by max(|ref|, sum|w'x| * 2^-10)): <= 1e-4 against the exact (float64)
product of the reference's fp32-dequantized weights, and <= 2e-4 against the
oracle, whose own sequential FP32 sum is up to ~1e-4 from that product at
K = 1280 (two FP32 orders differ by up to the sum of their errors).
"""
import numpy as np
import pytest

import oracle
from helpers import bits_equal, exact_linear, random_q8, rel_err, terms_abs

FP32_REL_TOL = 1e-4      # vs the exact product
FP32_ORACLE_TOL = 2e-4   # vs the oracle's sequential FP32 sum

pytestmark = pytest.mark.gpu


def run_device(ctx, w, s, x):
    import torch

    import uocr_q8
    m = uocr_q8.Int8Matrix.from_parts(w.shape[0], w.shape[1], w, s, ctx)
    y = m.linear_device(torch.from_numpy(np.ascontiguousarray(x)).cuda(), dynamic=True)
    ctx.sync()
    return y.cpu().numpy()


@pytest.mark.parametrize("batch", [2, 3, 7, 9, 16, 17, 63, 64, 65, 128, 200])
@pytest.mark.parametrize("rows,cols", [(128, 128), (896, 1280), (256, 896), (1792, 1280), (1280, 1792)])
def test_tc_dynamic_bit_exact(ctx, rows, cols, batch):
    """2..16 rows: the warp-level kernel (s8 MMA per block); more: tcgen05."""
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


def run_device_f32(ctx, w, s, x):
    import torch

    import uocr_q8
    m = uocr_q8.Int8Matrix.from_parts(w.shape[0], w.shape[1], w, s, ctx)
    y = m.linear_device(torch.from_numpy(np.ascontiguousarray(x)).cuda())
    ctx.sync()
    return y.cpu().numpy(), m


@pytest.mark.parametrize("batch", [2, 5, 8, 16, 17, 63, 64, 65, 130, 512])
@pytest.mark.parametrize("rows,cols", [(128, 128), (896, 1280), (1280, 896), (3840, 1280), (1280, 1792)])
def test_tc_fp32_linear_tolerance(ctx, rows, cols, batch):
    rng = np.random.default_rng(rows * 5 + cols + batch)
    w, s = random_q8(rng, rows, cols)
    x = (rng.standard_normal((batch, cols)) * rng.uniform(0.1, 10, (batch, 1))).astype(np.float32)
    y, m = run_device_f32(ctx, w, s, x)
    ta = terms_abs(w, s, x)
    assert rel_err(y, exact_linear(w, s, x), ta) <= FP32_REL_TOL
    assert rel_err(y, oracle.linear(oracle.Matrix(w, s), x), ta) <= FP32_ORACLE_TOL
    # the host-buffer entry point takes the same path
    assert bits_equal(m.linear(x), y)


def test_tc_fp32_extremes(ctx):
    """Mixed magnitudes inside a block (the pieces are exact for every fp32
    value), subnormal activations, zero rows, +-127 weight patterns, large
    and subnormal scales."""
    rows, cols, batch = 256, 1280, 40
    rng = np.random.default_rng(77)
    # (the same inputs through the warp-level kernel: see test_small_fp32_extremes)
    i = np.arange(rows * cols).reshape(rows, cols)
    w = ((i * 53) % 255 - 127).astype(np.int8)
    s = rng.uniform(1e-4, 1e-2, (rows, cols // 32)).astype(np.float32)
    s[::5] = 1e-38
    s[1::7] = 3e3
    x = (rng.standard_normal((batch, cols)) * 10.0 ** rng.integers(-20, 20, (batch, cols))).astype(np.float32)
    x[3] = 0.0
    x[4] = np.float32(1e-41)  # subnormal
    x[5, ::2] = 1e25
    y, _ = run_device_f32(ctx, w, s, x)
    # magnitudes 10^-20 .. 10^20 within a row cancel: the oracle's sequential
    # sum is itself ~1e-2 from the exact product here, so only that is checked
    assert rel_err(y, exact_linear(w, s, x), terms_abs(w, s, x)) <= FP32_REL_TOL
    assert np.all(y[3] == 0)


def test_small_fp32_extremes(ctx):
    """The extremes of test_tc_fp32_extremes through the 2..16-row kernel."""
    rows, cols, batch = 256, 1280, 12
    rng = np.random.default_rng(78)
    i = np.arange(rows * cols).reshape(rows, cols)
    w = ((i * 53) % 255 - 127).astype(np.int8)
    s = rng.uniform(1e-4, 1e-2, (rows, cols // 32)).astype(np.float32)
    s[::5] = 1e-38
    s[1::7] = 3e3
    x = (rng.standard_normal((batch, cols)) * 10.0 ** rng.integers(-20, 20, (batch, cols))).astype(np.float32)
    x[3] = 0.0
    x[4] = np.float32(1e-41)
    x[5, ::2] = 1e25
    y, _ = run_device_f32(ctx, w, s, x)
    assert rel_err(y, exact_linear(w, s, x), terms_abs(w, s, x)) <= FP32_REL_TOL
    assert np.all(y[3] == 0)
