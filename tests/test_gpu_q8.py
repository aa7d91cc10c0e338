"""GPU parity of the q8-block32 operators against the oracle, through the C ABI.

Restates the reference's own operator tests (tests/quantized.rs,
tests/quantized_loader.rs, src/cpu/neon.rs:245-276) on the CUDA library:
bit-exact for dequantize, quantize and linear_dynamic_int8; within the
stated tolerance for FP32-activation linear.
"""
import numpy as np
import pytest

import oracle
from helpers import bits_equal, dequant64, exact_linear, random_q8, rel_err, terms_abs

pytestmark = pytest.mark.gpu

FP32_REL_TOL = 1e-4  # max relative error, normalised (helpers.rel_err)


def q8():
    import uocr_q8
    return uocr_q8


# ---------------------------------------------------------------- storage
def test_from_parts_validation(ctx):
    M = q8().Int8Matrix
    E = q8().OcrError
    # tests/quantized.rs:74-87
    with pytest.raises(E) as e:
        M.from_parts(1, 33, np.zeros(33), [1.0], ctx)
    assert e.value.kind == "Shape"
    with pytest.raises(E) as e:
        M.from_parts(1, 1, [0], [np.nan], ctx)
    assert e.value.kind == "Numerical"
    with pytest.raises(E) as e:
        M.from_parts(1, 1, [0], [-1.0], ctx)
    assert e.value.kind == "Numerical"
    with pytest.raises(E) as e:
        M.from_parts(0, 1, [], [], ctx)
    assert e.value.kind == "Shape"
    m = M.from_parts(1, 1, [1], [-0.0], ctx)  # -0.0 accepted
    assert m.storage_bytes() == 1 + 4
    with pytest.raises(E) as e:
        M.quantize(np.array([[np.inf]], np.float32), ctx)
    assert e.value.kind == "Numerical"
    m = M.from_parts(1, 1, [1], [1.0], ctx)
    with pytest.raises(E) as e:
        m.linear(np.ones((1, 2), np.float32))
    assert e.value.kind == "Shape"


def test_storage_bytes_of_expert_matrix(ctx):
    rng = np.random.default_rng(0)
    m = q8().Int8Matrix.from_parts(896, 1280, *random_q8(rng, 896, 1280), ctx=ctx)
    assert m.storage_bytes() == 1_290_240  # bench_int8's int8_bytes for gate_proj
    w, s = m.download()
    assert w.shape == (896, 1280) and s.shape == (896, 40)


def test_loader_known_answer(ctx):
    # tests/quantized_loader.rs:41-48
    m = q8().Int8Matrix.from_parts(1, 2, np.array([1, -2], np.int8), [1.0], ctx)
    assert m.linear(np.array([[3.0, 4.0]], np.float32)).tolist() == [[-5.0]]
    assert m.linear_dynamic_int8(np.array([[3.0, 4.0]], np.float32)).shape == (1, 1)


# ---------------------------------------------------------------- dequantize
@pytest.mark.parametrize("cols", [1, 31, 32, 33, 513, 1280])
def test_dequantize_correctly_rounded(ctx, cols):
    # tests/quantized.rs:7-30
    rows = 5
    w = ((np.arange(rows * cols) % 255) - 127).astype(np.int8).reshape(rows, cols)
    nb = (cols + 31) // 32
    s = np.array([[0.0, -0.0, 0.1234567, 1e-20, 1e20][i % 5] for i in range(rows * nb)],
                 np.float32).reshape(rows, nb)
    m = q8().Int8Matrix.from_parts(rows, cols, w, s, ctx)
    assert bits_equal(m.dequantize(), dequant64(w, s).astype(np.float32))


@pytest.mark.parametrize("shape", [(896, 1280), (1280, 896), (257, 513)])
def test_dequantize_bench_shapes(ctx, shape):
    # examples/bench_dequantize.rs shapes and patterns
    rows, cols = shape
    w = ((np.arange(rows * cols) % 255) - 127).astype(np.int8).reshape(rows, cols)
    nb = (cols + 31) // 32
    s = (((np.arange(rows * nb) % 19) + 1) / np.float32(127)).astype(np.float32).reshape(rows, nb)
    m = q8().Int8Matrix.from_parts(rows, cols, w, s, ctx)
    assert bits_equal(m.dequantize(), oracle.dequantize(oracle.Matrix(w, s)))


# ---------------------------------------------------------------- quantize
def test_quantize_matches_reference_tool(ctx, golden):
    for name in golden["names"]:
        x = golden[f"{name}__x"]
        m = q8().Int8Matrix.quantize(x, ctx)
        w, s = m.download()
        assert np.array_equal(w, golden[f"{name}__q"]), name
        assert bits_equal(s, golden[f"{name}__s"]), name


def test_quantize_underflow_is_numerical(ctx, golden):
    with pytest.raises(q8().OcrError) as e:
        q8().Int8Matrix.quantize(golden["underflow__x"], ctx)
    assert e.value.kind == "Numerical"
    ctx.sync()  # the error was consumed; the context stays usable


def test_quantize_rows_device(ctx):
    import torch
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((64, 1280)) * rng.uniform(0.1, 10, (64, 1))).astype(np.float32)
    q, s = q8().quantize_rows_device(ctx, torch.from_numpy(x).cuda())
    ctx.sync()
    ref = oracle.quantize(x)
    assert np.array_equal(q.cpu().numpy(), ref.w)
    assert bits_equal(s.cpu().numpy(), ref.s)


# ---------------------------------------------------------------- linear (FP32)
@pytest.mark.parametrize("cols", [1, 31, 32, 33, 131, 513])
def test_linear_reference_tolerance(ctx, cols):
    # tests/quantized.rs:31-73: abs error < 2e-5 vs the f64 product
    rows = 257 if cols == 513 else 7
    i = np.arange(rows * cols, dtype=np.float32)
    values = (np.sin(i * np.float32(0.37)) * np.float32(3.0)).astype(np.float32)
    values[:cols] = 0
    m = q8().Int8Matrix.quantize(values.reshape(rows, cols), ctx)
    restored = m.dequantize()
    assert np.all(restored[0] == 0)
    for batch in (1, 3):
        x = np.cos(np.arange(batch * cols, dtype=np.float32) * np.float32(0.13)).reshape(batch, cols)
        y = m.linear(x)
        want = x.astype(np.float64) @ restored.astype(np.float64).T
        assert np.max(np.abs(y - want)) < 2e-5


@pytest.mark.parametrize("rows,cols", [(896, 1280), (1280, 896), (1792, 1280), (1280, 1792),
                                       (129, 1280), (6, 128), (37, 513), (1000, 6848),
                                       (64, 6144), (32, 8192)])
@pytest.mark.parametrize("batch", [1, 4])
def test_linear_vs_oracle(ctx, rows, cols, batch):
    """(64, 6144) and (32, 8192): rows too wide for the streaming kernel's ring
    in shared memory take the generic kernel at batch 1."""
    rng = np.random.default_rng(rows * 7 + cols + batch)
    w, s = random_q8(rng, rows, cols)
    x = rng.standard_normal((batch, cols)).astype(np.float32)
    m = q8().Int8Matrix.from_parts(rows, cols, w, s, ctx)
    y = m.linear(x)
    ref = oracle.linear(oracle.Matrix(w, s), x)
    ta = terms_abs(w, s, x)
    # vs the exact product; vs the oracle, whose own sequential FP32 sum is up
    # to ~1e-4 from it at these sizes, twice that
    assert rel_err(y, exact_linear(w, s, x), ta) <= FP32_REL_TOL
    assert rel_err(y, ref, ta) <= 2 * FP32_REL_TOL


def test_linear_device_matches_host(ctx):
    import torch
    rng = np.random.default_rng(17)
    w, s = random_q8(rng, 896, 1280)
    x = rng.standard_normal((1, 1280)).astype(np.float32)
    m = q8().Int8Matrix.from_parts(896, 1280, w, s, ctx)
    yd = m.linear_device(torch.from_numpy(x).cuda())
    ctx.sync()
    assert bits_equal(yd.cpu().numpy(), m.linear(x))


def test_linear_multi_matches_single(ctx):
    import torch
    rng = np.random.default_rng(19)
    mats, ws = [], []
    for _ in range(20):  # more than one launch's worth of matrices
        w, s = random_q8(rng, 896, 1280)
        mats.append(q8().Int8Matrix.from_parts(896, 1280, w, s, ctx))
        ws.append((w, s))
    x = rng.standard_normal(1280).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    for mode in (0, 1):
        ys = [torch.empty(896, device="cuda") for _ in mats]
        q8().linear_multi_device(ctx, mats, xt, ys, mode)
        ctx.sync()
        for (w, s), y in zip(ws, ys):
            if mode == 0:
                ref = oracle.linear(oracle.Matrix(w, s), x)[0]
                assert rel_err(y.cpu().numpy(), ref, terms_abs(w, s, x)[0]) <= FP32_REL_TOL
            else:
                assert bits_equal(y.cpu().numpy(), oracle.linear_dynamic_int8(oracle.Matrix(w, s), x)[0])


# ---------------------------------------------------------------- linear (int8 activations)
@pytest.mark.parametrize("cols", [1, 15, 31, 32, 33, 131, 1280])
def test_dynamic_reference_tolerance_and_bits(ctx, cols):
    # tests/quantized.rs:89-120, plus bit equality with the oracle
    rows = 129 if cols == 1280 else 9
    wf = np.sin(np.arange(rows * cols, dtype=np.float32) * np.float32(0.41)).reshape(rows, cols)
    m = q8().Int8Matrix.quantize(wf, ctx)
    w, s = m.download()
    x = (np.cos(np.arange(cols, dtype=np.float32) * np.float32(0.17)) * np.float32(2.0))[None]
    y = m.linear_dynamic_int8(x)
    rounded = oracle.dequantize(oracle.quantize(x))
    want = rounded.astype(np.float64) @ dequant64(w, s).T
    assert np.max(np.abs(y - want)) < 2e-4
    assert bits_equal(y, oracle.linear_dynamic_int8(oracle.Matrix(w, s), x))


@pytest.mark.parametrize("rows,cols", [(896, 1280), (1280, 896), (3840, 1280), (1280, 1792),
                                       (64, 6848), (33, 100), (4, 32), (64, 6144), (32, 8192)])
def test_dynamic_bit_exact(ctx, rows, cols):
    rng = np.random.default_rng(rows + 3 * cols)
    w, s = random_q8(rng, rows, cols)
    x = (rng.standard_normal(cols) * rng.uniform(0.1, 10)).astype(np.float32)[None]
    m = q8().Int8Matrix.from_parts(rows, cols, w, s, ctx)
    assert bits_equal(m.linear_dynamic_int8(x), oracle.linear_dynamic_int8(oracle.Matrix(w, s), x))


@pytest.mark.parametrize("cols", [32, 64, 896, 1280])
def test_dynamic_four_row_patterns(ctx, cols):
    # src/cpu/neon.rs:245-276: -128 extremes, zero/tiny/huge scales
    rows = 4
    w = (((np.arange(cols * rows) * 53) % 256) - 128).astype(np.int8).reshape(rows, cols)
    s = np.array([[0.0, 0.00317, 0.7, 1e-10, 17.0][i % 5] for i in range(rows * cols // 32)],
                 np.float32).reshape(rows, cols // 32)
    x = (np.sin(np.arange(cols, dtype=np.float32)) * np.float32(5.0))[None]
    m = q8().Int8Matrix.from_parts(rows, cols, w, s, ctx)
    assert bits_equal(m.linear_dynamic_int8(x), oracle.linear_dynamic_int8(oracle.Matrix(w, s), x))


def test_dynamic_rowwise_device(ctx):
    import torch
    rng = np.random.default_rng(23)
    w, s = random_q8(rng, 1280, 1280)
    x = (rng.standard_normal((16, 1280)) * rng.uniform(0.1, 10, (16, 1))).astype(np.float32)
    m = q8().Int8Matrix.from_parts(1280, 1280, w, s, ctx)
    y = m.linear_device(torch.from_numpy(x).cuda(), dynamic=True)
    ctx.sync()
    assert bits_equal(y.cpu().numpy(), oracle.linear_dynamic_int8(oracle.Matrix(w, s), x))


def test_dynamic_rejects_multi_row_and_nonfinite(ctx):
    rng = np.random.default_rng(1)
    w, s = random_q8(rng, 8, 64)
    m = q8().Int8Matrix.from_parts(8, 64, w, s, ctx)
    with pytest.raises(q8().OcrError) as e:
        m.linear_dynamic_int8(np.zeros((2, 64), np.float32))
    assert e.value.kind == "Shape"
    x = np.zeros((1, 64), np.float32)
    x[0, 5] = np.nan
    with pytest.raises(q8().OcrError) as e:
        m.linear_dynamic_int8(x)
    assert e.value.kind == "Numerical"
    # the context keeps working after a device-detected error
    x[0, 5] = 1.0
    assert bits_equal(m.linear_dynamic_int8(x), oracle.linear_dynamic_int8(oracle.Matrix(w, s), x))


def test_scratch_limit_is_resource_error():
    import uocr_q8
    small = uocr_q8.GpuContext(0, scratch_limit=1024)
    rng = np.random.default_rng(2)
    w, s = random_q8(rng, 300, 64)
    m = uocr_q8.Int8Matrix.from_parts(300, 64, w, s, small)
    with pytest.raises(uocr_q8.OcrError) as e:  # 300 outputs * 4 B > 1024 B
        m.linear(np.zeros((1, 64), np.float32))
    assert e.value.kind == "Resource"
    small.close()
