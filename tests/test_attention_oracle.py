"""CPU checks of the oracle's decode-attention ops against the reference's
own tests: RMSNorm and rope known answers (tests/ops.rs:33-73), decode
attention against an f64 restatement (tests/decode_attention.rs:6-47) and its
layout rejections (:50-64), causal prefill attention (tests/ops.rs:89-99,
166-202), and the KV cache ring (tests/cache.rs).
"""
import numpy as np
import pytest

import oracle


def test_rms_norm_known_answer():
    """tests/ops.rs:43-50."""
    y = oracle.rms_norm(np.array([[1.0, 3.0]], np.float32), np.array([1.0, 1.0], np.float32), 1e-6)
    assert abs(float(y[0, 0]) - 0.44721355) < 1e-6
    assert abs(float(y[0, 1]) - 1.3416406) < 1e-6


def test_rms_norm_rejections():
    w = np.ones(4, np.float32)
    with pytest.raises(oracle.OracleError) as e:
        oracle.rms_norm(np.array([[1, np.nan, 0, 0]], np.float32), w)
    assert e.value.kind == "Numerical"
    with pytest.raises(oracle.OracleError) as e:
        oracle.rms_norm(np.ones((1, 4), np.float32), np.array([1, 1, np.inf, 1], np.float32))
    assert e.value.kind == "Numerical"
    with pytest.raises(oracle.OracleError) as e:
        oracle.rms_norm(np.ones((1, 4), np.float32), w, eps=0.0)
    assert e.value.kind == "Shape"


def test_rms_norm_is_the_sequential_f32_sum():
    """The oracle's variance is the left-to-right float32 sum (differs from a
    float64 sum in the last bits for wide rows)."""
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((4, 1280)) * 3).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 1280).astype(np.float32)
    y = oracle.rms_norm(x, w, 1e-6)
    for r in range(4):
        acc = np.float32(-0.0)
        for v in x[r]:
            acc = np.float32(acc + np.float32(v * v))
        var = np.float32(acc / np.float32(1280))
        scale = np.float32(np.float32(1.0) / np.sqrt(np.float32(var + np.float32(1e-6))))
        ref = ((x[r] * scale).astype(np.float32) * w).astype(np.float32) + np.float32(0.0)
        assert np.array_equal(ref.view(np.uint32), y[r].view(np.uint32))


def test_rope_known_answers():
    """tests/ops.rs:63-73: position 0 is the identity; position 1 of [1,2,3,4]."""
    v = oracle.rope([1.0, 2.0, 3.0, 4.0], 4, 0, 10000.0)
    assert v.tolist() == [1.0, 2.0, 3.0, 4.0]
    v = oracle.rope(v, 4, 1, 10000.0)
    want = [-1.9841106, 1.9599007, 2.462378, 4.0197997]
    assert np.max(np.abs(v - np.array(want, np.float32))) < 1e-5


def test_rope_rejections():
    for values, dim, theta in (([1.0] * 4, 0, 1e4), ([1.0] * 6, 3, 1e4), ([1.0] * 6, 4, 1e4),
                               ([1.0] * 4, 4, 0.0), ([1.0] * 4, 4, np.inf)):
        with pytest.raises(oracle.OracleError) as e:
            oracle.rope(values, dim, 1, theta)
        assert e.value.kind == "Shape"


def f64_attention(q, k, v, heads):
    """The reference test's f64 oracle (tests/decode_attention.rs:22-38)."""
    width = q.size
    dim = width // heads
    tokens = k.size // width
    k = k.reshape(tokens, width).astype(np.float64)
    v = v.reshape(tokens, width).astype(np.float64)
    out = np.zeros(width)
    for h in range(heads):
        sl = slice(h * dim, (h + 1) * dim)
        s = np.exp((k[:, sl] @ q[sl].astype(np.float64)) / np.sqrt(dim))
        out[sl] = (s / s.sum()) @ v[:, sl]
    return out


def reference_case(tokens, heads=3, dim=5):
    """tests/decode_attention.rs:8-20 inputs."""
    width = heads * dim
    q = np.sin(np.arange(width, dtype=np.float32) * np.float32(0.7)).astype(np.float32)
    i = np.arange(tokens * width, dtype=np.float32)
    k = np.cos(i * np.float32(0.13)).astype(np.float32)
    v = np.sin(i * np.float32(0.31)).astype(np.float32)
    return q, k, v


@pytest.mark.parametrize("tokens", [1, 7, 139, 1641])
def test_attention_matches_f64(tokens):
    q, k, v = reference_case(tokens)
    out = oracle.attention_decode(q, k, v, 3)
    assert np.max(np.abs(out.astype(np.float64) - f64_attention(q, k, v, 3))) < 2e-6


def test_attention_rejects_layouts():
    """tests/decode_attention.rs:50-64."""
    q = np.zeros(6, np.float32)
    for keys, values, heads in (([], [], 2), ([0.0] * 7, [0.0] * 7, 2), ([0.0] * 6, [0.0] * 5, 2),
                                ([0.0] * 6, [0.0] * 6, 4), ([0.0] * 6, [0.0] * 6, 0)):
        with pytest.raises(oracle.OracleError) as e:
            oracle.attention_decode(q, np.array(keys, np.float32), np.array(values, np.float32),
                                    heads)
        assert e.value.kind == "Shape"


def test_causal_attention_excludes_future_values():
    """tests/ops.rs:89-99."""
    q = np.zeros((1, 2, 2), np.float32)
    v = np.array([2.0, 4.0, 6.0, 8.0], np.float32).reshape(1, 2, 2)
    assert oracle.attention(q, q, v, True).ravel().tolist() == [2.0, 4.0, 4.0, 6.0]
    assert oracle.attention(q, q, v, False).ravel().tolist() == [4.0, 6.0, 4.0, 6.0]


def causal_block_case(heads=2, tokens=129, dim=3):
    """tests/ops.rs:167-181 inputs: zero queries and keys, values
    head * 100 + token + channel."""
    q = np.zeros((heads, tokens, dim), np.float32)
    i = np.arange(heads * tokens * dim)
    v = ((i // (tokens * dim)) * 100 + (i // dim) % tokens + i % dim).astype(np.float32)
    return q, v.reshape(heads, tokens, dim)


def test_causal_attention_masks_across_query_block_boundaries():
    """tests/ops.rs:166-194: uniform weights over the first token + 1 values."""
    heads, tokens, dim = 2, 129, 3
    q, v = causal_block_case(heads, tokens, dim)
    out = oracle.attention(q, q, v, True)
    h, t, c = np.meshgrid(np.arange(heads), np.arange(tokens), np.arange(dim), indexing="ij")
    want = (h * 100 + c).astype(np.float32) + t.astype(np.float32) / 2
    assert np.max(np.abs(out - want)) < 2e-4


def test_causal_attention_of_zeros_is_zero():
    """tests/ops.rs:196-202 (a zero input gives a zero output)."""
    q = np.zeros((1, 129, 3), np.float32)
    assert np.array_equal(oracle.attention(q, q, q, True), q)


def test_causal_row_equals_decode_over_its_prefix():
    """Row i of the causal prefill attention is attention_decode over tokens
    0..i: the masked keys only add +0.0 products after the real ones, so every
    nonzero output is bit-identical."""
    rng = np.random.default_rng(5)
    tokens, heads, dim = 23, 3, 8
    width = heads * dim
    q, k, v = (rng.standard_normal((tokens, width)).astype(np.float32) for _ in range(3))
    out = oracle.attention_prefill(q, k, v, heads)
    for i in range(tokens):
        ref = oracle.attention_decode(q[i], k[:i + 1], v[:i + 1], heads)
        assert np.array_equal(out[i], ref)
        nz = ref != 0
        assert np.array_equal(out[i][nz].view(np.uint32), ref[nz].view(np.uint32))


def test_causal_attention_rejects_layouts():
    q = np.zeros((1, 2, 2), np.float32)
    with pytest.raises(oracle.OracleError) as e:
        oracle.attention(q, np.zeros((1, 3, 2), np.float32), np.zeros((1, 3, 2), np.float32), True)
    assert e.value.kind == "Shape"
    bad = q.copy()
    bad[0, 0, 0] = np.nan
    with pytest.raises(oracle.OracleError) as e:
        oracle.attention(bad, q, q, True)
    assert e.value.kind == "Numerical"


def test_cache_prefix_survives_ring_wraps():
    """tests/cache.rs:4-19."""
    c = oracle.LayerCache(1, 1, 3)
    c.prefill([10.0, 20.0], [100.0, 200.0], 2)
    for i in range(10):
        c.push([float(i)], [float(i * 10)])
        assert c.keys[:2, 0].tolist() == [10.0, 20.0]
        assert c.values[:2, 0].tolist() == [100.0, 200.0]
        assert c.tokens() == 2 + min(i + 1, 3)
    assert sorted(c.keys[2:, 0].tolist()) == [7.0, 8.0, 9.0]
    assert c.position() == 12


def test_cache_bad_push_does_not_advance():
    """tests/cache.rs:21-29."""
    c = oracle.LayerCache(2, 2, 128)
    with pytest.raises(oracle.OracleError):
        c.push([1.0] * 4, [1.0] * 4)
    c.prefill([0.0] * 8, [0.0] * 8, 2)
    with pytest.raises(oracle.OracleError):
        c.push([1.0] * 3, [1.0] * 4)
    assert c.position() == 2
    with pytest.raises(oracle.OracleError):
        c.prefill([0.0] * 8, [0.0] * 8, 2)
