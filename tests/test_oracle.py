"""CPU checks of the oracle against the reference's own known answers.

Pins: tools/quantize.py outputs (tests/golden), the loader known answer
(tests/quantized_loader.rs:41-48), routing known answers (tests/moe.rs:4-13),
and restatements of the reference's arithmetic tests (tests/quantized.rs).
"""
import numpy as np
import pytest

import oracle
from helpers import bits_equal, dequant64, random_q8


def test_quantizer_matches_reference_tool(golden):
    for name in golden["names"]:
        x = golden[f"{name}__x"]
        m = oracle.quantize(x)
        assert np.array_equal(m.w, golden[f"{name}__q"]), name
        assert bits_equal(m.s, golden[f"{name}__s"]), name


def test_quantizer_rejects_underflow_and_nonfinite(golden):
    with pytest.raises(oracle.OracleError) as e:
        oracle.quantize(golden["underflow__x"])
    assert e.value.kind == "Numerical"
    with pytest.raises(oracle.OracleError) as e:
        oracle.quantize(np.array([[np.inf]], np.float32))
    assert e.value.kind == "Numerical"


def test_loader_known_answer():
    # tests/quantized_loader.rs:24-48: W = [1, -2] (bytes 1, 254), scale 1, x = [3, 4]
    m = oracle.Matrix(np.array([[1, -2]], np.int8), np.array([[1.0]], np.float32))
    assert oracle.linear(m, [3.0, 4.0]).tolist() == [[-5.0]]


def test_route_known_answers():
    # tests/moe.rs:5-12
    assert oracle.route([0, 0, 0, 0], 2) == [(0, 0.25), (1, 0.25)]
    assert oracle.route([0, 0, 0, 0], 2, True, 2.0) == [(0, 1.0), (1, 1.0)]
    for bad in ([0.0, float("nan")], [0.0, float("inf")], [-np.inf, -np.inf]):
        with pytest.raises(oracle.OracleError) as e:
            oracle.route(bad, 1)
        assert e.value.kind == "Numerical"
    with pytest.raises(oracle.OracleError) as e:
        oracle.route([0.0], 2)
    assert e.value.kind == "Shape"


def test_from_parts_rules():
    # tests/quantized.rs:74-87
    assert oracle.from_parts_check(1, 33, np.zeros(33), [1.0]) == 4
    assert oracle.from_parts_check(1, 1, [0], [np.nan]) == 7
    assert oracle.from_parts_check(1, 1, [0], [-1.0]) == 7
    assert oracle.from_parts_check(0, 1, [], []) == 4
    assert oracle.from_parts_check(1, 1, [0], [-0.0]) == 0


@pytest.mark.parametrize("cols", [1, 31, 32, 33, 513, 1280])
def test_dequantize_is_correctly_rounded(cols):
    # tests/quantized.rs:7-30
    rows = 5
    w = ((np.arange(rows * cols) % 255) - 127).astype(np.int8).reshape(rows, cols)
    nb = (cols + 31) // 32
    s = np.array([[0.0, -0.0, 0.1234567, 1e-20, 1e20][i % 5] for i in range(rows * nb)],
                 np.float32).reshape(rows, nb)
    m = oracle.Matrix(w, s)
    want = dequant64(w, s).astype(np.float32)
    assert bits_equal(oracle.dequantize(m), want)


@pytest.mark.parametrize("cols", [1, 31, 32, 33, 131, 513])
def test_roundtrip_and_linear_tolerance(cols):
    # tests/quantized.rs:31-73
    rows = 257 if cols == 513 else 7
    i = np.arange(rows * cols, dtype=np.float32)
    values = (np.sin(i * np.float32(0.37)) * np.float32(3.0)).astype(np.float32)
    values[:cols] = 0
    values = values.reshape(rows, cols)
    m = oracle.quantize(values)
    restored = oracle.dequantize(m)
    assert np.all(np.abs(restored - values) <= 3.0 / 254.0 + 1e-6)
    assert np.all(restored[0] == 0)
    for batch in (1, 3):
        x = np.cos(np.arange(batch * cols, dtype=np.float32) * np.float32(0.13)).reshape(batch, cols)
        y = oracle.linear(m, x)
        want = x.astype(np.float64) @ restored.astype(np.float64).T
        assert np.max(np.abs(y - want)) < 2e-5


@pytest.mark.parametrize("cols", [1, 15, 31, 32, 33, 131, 1280])
def test_dynamic_tolerance(cols):
    # tests/quantized.rs:89-120
    rows = 129 if cols == 1280 else 9
    w = np.sin(np.arange(rows * cols, dtype=np.float32) * np.float32(0.41)).reshape(rows, cols)
    m = oracle.quantize(w)
    x = (np.cos(np.arange(cols, dtype=np.float32) * np.float32(0.17)) * np.float32(2.0))[None]
    rounded = oracle.dequantize(oracle.quantize(x))
    y = oracle.linear_dynamic_int8(m, x)
    want = rounded.astype(np.float64) @ oracle.dequantize(m).astype(np.float64).T
    assert np.max(np.abs(y - want)) < 2e-4


def _dynamic_python(w, s, x):
    """Independent pure-Python restatement of the scalar dynamic dot
    (src/cpu/quantized.rs:190-198) in numpy float32 scalars."""
    q = oracle.quantize(np.asarray(x, np.float32)[None])
    xq, xs = q.w[0].astype(np.int64), q.s[0]
    rows, cols = w.shape
    out = np.empty(rows, np.float32)
    for r in range(rows):
        acc = np.float32(-0.0)
        for b in range((cols + 31) // 32):
            S = int(np.dot(w[r, b * 32:(b + 1) * 32].astype(np.int64), xq[b * 32:(b + 1) * 32]))
            acc = np.float32(acc + np.float32(np.float32(np.float32(S) * s[r, b]) * xs[b]))
        out[r] = acc
    return out


def test_dynamic_matches_independent_restatement():
    rng = np.random.default_rng(5)
    w, s = random_q8(rng, 24, 96)
    x = rng.standard_normal(96).astype(np.float32)
    got = oracle.linear_dynamic_int8(oracle.Matrix(w, s), x)[0]
    assert bits_equal(got, _dynamic_python(w, s, x))


def test_four_row_patterns_block_sums():
    # src/cpu/neon.rs:245-276 patterns, including -128 extremes
    for cols in (32, 64, 896, 1280):
        w = (((np.arange(cols * 4) * 53) % 256) - 128).astype(np.int8).reshape(4, cols)
        xq = (((np.arange(cols) * 71) % 256) - 128).astype(np.int8)
        for r in range(4):
            sums = oracle.block_sums(w[r], xq)
            want = (w[r].astype(np.int64).reshape(-1, 32) * xq.astype(np.int64).reshape(-1, 32)).sum(1)
            assert np.array_equal(sums, want)


def test_linear_is_thread_count_invariant():
    rng = np.random.default_rng(9)
    w, s = random_q8(rng, 300, 1280)
    m = oracle.Matrix(w, s)
    x = rng.standard_normal((2, 1280)).astype(np.float32)
    oracle.set_threads(1)
    a = oracle.linear(m, x)
    b = oracle.linear_dynamic_int8(m, x)
    oracle.set_threads(4)
    assert bits_equal(a, oracle.linear(m, x))
    assert bits_equal(b, oracle.linear_dynamic_int8(m, x))
    oracle.set_threads(0)


def test_experts_order_and_modes():
    """Decoder::experts: shared first, routed experts added in ascending id."""
    rng = np.random.default_rng(11)
    H, F, FS, E, k, T = 64, 32, 64, 8, 3, 5

    def ffn(width):
        g = oracle.Matrix(*random_q8(rng, width, H))
        u = oracle.Matrix(*random_q8(rng, width, H))
        d = oracle.Matrix(*random_q8(rng, H, width))
        return oracle.Ffn(g, u, d)

    shared = ffn(FS)
    routed = [ffn(F) for _ in range(E)]
    x = rng.standard_normal((T, H)).astype(np.float32)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    for mode in (oracle.WEIGHTS_ONLY, oracle.DYNAMIC, oracle.DYNAMIC_ROWWISE):
        out, ids, wts = oracle.experts(shared, routed, logits, x, k, mode)
        # restate the combine per token with single-row feed_forward calls
        for t in range(T):
            m1 = oracle.DYNAMIC_ROWWISE if mode == oracle.DYNAMIC_ROWWISE else mode
            sh_mode = m1 if (mode != oracle.DYNAMIC or T == 1) else oracle.WEIGHTS_ONLY
            r = oracle.feed_forward(shared, x[t:t + 1], sh_mode)[0]
            order = np.argsort(ids[t], kind="stable")
            for j in order:
                e = int(ids[t, j])
                cnt = int((ids == e).sum())
                e_mode = mode
                if mode == oracle.DYNAMIC:
                    e_mode = oracle.DYNAMIC if cnt == 1 else oracle.WEIGHTS_ONLY
                o = oracle.feed_forward(routed[e], x[t:t + 1], e_mode)[0]
                r = (r + np.float32(wts[t, j]) * o).astype(np.float32)
            assert bits_equal(out[t], r), (mode, t)
