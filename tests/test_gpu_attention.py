"""GPU parity of the decode-attention ops (RMSNorm, rope, decode attention,
KV cache, the attention half of a decoder layer) against the CPU oracle,
through the C ABI.

Bit-exact: RMSNorm, rope and the cache contents.  The causal attention of a
prefill runs the decode kernels with one query per row, so it is held to the
same bounds.  Attention follows the
reference's order, so it is bit-identical wherever every exp rounds the same
(checked exactly with uniform scores, where exp is exact); otherwise the
device's exp (double, rounded once) and the C library's expf (within 0.502
ulp) can differ by one ulp in a few of thousands of softmax terms, which
moves a head's sum and so the last bits of that head's outputs.  Those cases
are held to the reference's own bound: 2e-6 against its f64 oracle
(tests/decode_attention.rs:44), and 1e-5 relative against the oracle.
"""
import numpy as np
import pytest

import oracle
from helpers import bits_equal
from test_attention_oracle import f64_attention, reference_case

pytestmark = pytest.mark.gpu


def A():
    import uocr_q8.attention as attention
    return attention


def dev(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.cuda() if dtype is None else t.to(dtype).cuda()


def host(t):
    return t.detach().cpu().numpy()


# ---------------------------------------------------------------- RMSNorm
@pytest.mark.parametrize("rows,width", [(1, 2), (3, 7), (64, 1280), (2, 4096), (5, 33)])
def test_rms_norm_bit_exact(ctx, rows, width):
    rng = np.random.default_rng(rows * 1000 + width)
    x = (rng.standard_normal((rows, width)) * rng.uniform(0.01, 30, (rows, 1))).astype(np.float32)
    w = rng.uniform(-2, 2, width).astype(np.float32)
    y = A().rms_norm_device(ctx, dev(x), dev(w), 1e-6)
    ctx.sync()
    assert bits_equal(host(y), oracle.rms_norm(x, w, 1e-6))


def test_rms_norm_known_answer_and_in_place(ctx):
    x = dev(np.array([[1.0, 3.0]], np.float32))
    A().rms_norm_device(ctx, x, dev(np.ones(2, np.float32)), 1e-6, out_t=x)
    ctx.sync()
    y = host(x)
    assert abs(float(y[0, 0]) - 0.44721355) < 1e-6 and abs(float(y[0, 1]) - 1.3416406) < 1e-6


def test_rms_norm_errors(ctx):
    import uocr_q8
    x = np.ones((2, 8), np.float32)
    x[1, 3] = np.nan
    A().rms_norm_device(ctx, dev(x), dev(np.ones(8, np.float32)))
    with pytest.raises(uocr_q8.OcrError) as e:
        ctx.sync()
    assert e.value.kind == "Numerical"
    with pytest.raises(uocr_q8.OcrError) as e:
        A().rms_norm_device(ctx, dev(np.ones((1, 8), np.float32)), dev(np.ones(8, np.float32)), 0.0)
    assert e.value.kind == "Shape"


@pytest.mark.parametrize("alias", ["none", "x", "res"])
@pytest.mark.parametrize("rows,width", [(64, 1280), (3, 7)])
def test_add_rms_norm_equals_add_then_norm(ctx, alias, rows, width):
    """uocr_add_rms_norm: the residual sum bit for bit as x + res (one
    rounding), the output as rms_norm of it (the oracle's), with the sum
    written to a separate buffer or over either input."""
    rng = np.random.default_rng(rows + width + len(alias))
    x = (rng.standard_normal((rows, width)) * 3).astype(np.float32)
    r = (rng.standard_normal((rows, width)) * 2).astype(np.float32)
    w = rng.uniform(-2, 2, width).astype(np.float32)
    xt, rt = dev(x), dev(r)
    st = {"none": None, "x": xt, "res": rt}[alias]
    out = A().add_rms_norm_device(ctx, xt, rt, dev(w), 1e-6, sum_t=st)
    ctx.sync()
    s_ref = (x + r).astype(np.float32)
    if st is not None:
        assert bits_equal(host(st), s_ref)
    assert bits_equal(host(out), oracle.rms_norm(s_ref, w, 1e-6))


def test_add_rms_norm_errors(ctx):
    import uocr_q8
    x = np.full((2, 8), 3e38, np.float32)  # the sum overflows: a nonfinite norm input
    A().add_rms_norm_device(ctx, dev(x), dev(x), dev(np.ones(8, np.float32)))
    with pytest.raises(uocr_q8.OcrError) as e:
        ctx.sync()
    assert e.value.kind == "Numerical"


# ---------------------------------------------------------------- rope
def test_rope_known_answer(ctx):
    r = A().Rope(ctx, 4, 10000.0, 16)
    q = dev(np.array([[1.0, 2.0, 3.0, 4.0], [1.0, 2.0, 3.0, 4.0]], np.float32))
    r.apply(q, None, dev(np.array([0, 1], np.int32)))
    ctx.sync()
    y = host(q)
    assert y[0].tolist() == [1.0, 2.0, 3.0, 4.0]
    assert np.max(np.abs(y[1] - np.array([-1.9841106, 1.9599007, 2.462378, 4.0197997]))) < 1e-5
    r.free()


def test_rope_bit_exact(ctx):
    rng = np.random.default_rng(4)
    heads, dim, rows = 10, 128, 12
    pos = np.array([0, 1, 2, 3, 127, 128, 2047, 2048, 2175, 5000, 32766, 32767], np.int32)
    q = rng.standard_normal((rows, heads * dim)).astype(np.float32)
    k = rng.standard_normal((rows, heads * dim)).astype(np.float32)
    r = A().Rope(ctx, dim, 10000.0, 32768)
    qt, kt = dev(q), dev(k)
    r.apply(qt, kt, dev(pos))
    ctx.sync()
    for i in range(rows):
        assert bits_equal(host(qt)[i], oracle.rope(q[i], dim, int(pos[i]))), i
        assert bits_equal(host(kt)[i], oracle.rope(k[i], dim, int(pos[i]))), i
    r.free()


def test_rope_position_past_table(ctx):
    import uocr_q8
    r = A().Rope(ctx, 4, 10000.0, 8)
    r.apply(dev(np.ones((1, 4), np.float32)), None, dev(np.array([8], np.int32)))
    with pytest.raises(uocr_q8.OcrError) as e:
        ctx.sync()
    assert e.value.kind == "Resource"
    with pytest.raises(uocr_q8.OcrError) as e:
        A().Rope(ctx, 3, 10000.0, 8)
    assert e.value.kind == "Shape"
    r.free()


# ---------------------------------------------------------------- attention
@pytest.mark.parametrize("tokens", [1, 7, 139, 1641])
def test_attention_reference_cases(ctx, tokens):
    """tests/decode_attention.rs:6-47 (3 heads of 5: the scalar-load path)."""
    q, k, v = reference_case(tokens)
    out = host(A().attention_decode_device(ctx, dev(q), dev(k), dev(v), 3))
    ctx.sync()
    assert np.max(np.abs(out.astype(np.float64) - f64_attention(q, k, v, 3))) < 2e-6
    ref = oracle.attention_decode(q, k, v, 3)
    assert np.max(np.abs(out - ref)) <= 1e-5 * max(1.0, float(np.max(np.abs(ref))))


@pytest.mark.parametrize("tokens", [129, 1641, 2176])
def test_attention_decoder_shape(ctx, tokens):
    """10 heads of 128 (tests/decode_attention.rs:66-96 shapes): vector path."""
    heads, dim = 10, 128
    width = heads * dim
    q = np.sin(np.arange(width, dtype=np.float32) * np.float32(0.17)).astype(np.float32)
    i = np.arange(tokens * width, dtype=np.float32)
    k = np.cos(i * np.float32(0.013)).astype(np.float32)
    v = np.sin(i * np.float32(0.031)).astype(np.float32)
    out = host(A().attention_decode_device(ctx, dev(q), dev(k), dev(v), heads))
    ctx.sync()
    ref = oracle.attention_decode(q, k, v, heads)
    assert np.max(np.abs(out - ref)) <= 1e-5 * max(1.0, float(np.max(np.abs(ref))))
    assert np.max(np.abs(out.astype(np.float64) - f64_attention(q, k, v, heads))) < 2e-6


@pytest.mark.parametrize("heads,dim,tokens", [(10, 128, 2176), (3, 5, 1641), (2, 64, 33)])
def test_attention_order_bit_exact_with_exact_exp(ctx, heads, dim, tokens):
    """Keys equal within each head make every score equal, so every exp is
    exp(0) = 1 exactly and the softmax is 1/T on both sides: the outputs are
    then the left-to-right value sums of the reference, bit for bit."""
    rng = np.random.default_rng(tokens)
    width = heads * dim
    q = rng.standard_normal(width).astype(np.float32)
    k = np.tile(rng.standard_normal(width).astype(np.float32), (tokens, 1))
    v = (rng.standard_normal((tokens, width)) * rng.uniform(0.1, 10, (tokens, 1))).astype(np.float32)
    out = host(A().attention_decode_device(ctx, dev(q), dev(k), dev(v), heads))
    ctx.sync()
    assert bits_equal(out, oracle.attention_decode(q, k, v, heads))


def test_attention_layout_errors(ctx):
    import torch
    import uocr_q8
    q = torch.zeros(6, device="cuda")
    for keys, values, heads in ((7, 7, 2), (6, 5, 2), (6, 6, 4), (6, 6, 0)):
        with pytest.raises(uocr_q8.OcrError) as e:
            A().attention_decode_device(ctx, q, torch.zeros(keys, device="cuda"),
                                        torch.zeros(values, device="cuda"), heads)
        assert e.value.kind == "Shape"
    bad = torch.zeros(6, device="cuda")
    bad[0] = float("nan")
    A().attention_decode_device(ctx, bad, torch.ones(12, device="cuda"), torch.ones(12, device="cuda"), 2)
    with pytest.raises(uocr_q8.OcrError) as e:
        ctx.sync()
    assert e.value.kind == "Numerical"


# ---------------------------------------------------------------- KV cache
@pytest.mark.parametrize("heads,dim", [(2, 8), (2, 64), (3, 128)])
def test_cache_ring_matches_layer_cache(ctx, heads, dim):
    """Prefill + pushes across ring wraps (tests/cache.rs shapes scaled up):
    the device cache holds the reference's physical token order (plain layout
    for head_dim 8, 32-slot tiles for 64 and 128), and the attention over it
    equals the oracle's over LayerCache contents."""
    rng = np.random.default_rng(11 + dim)
    batch, window = 3, 5
    width = heads * dim
    prefixes = [4, 1, 7]
    kv = A().KvCache(ctx, batch, heads, dim, window, max_prefix=8)
    refs = [oracle.LayerCache(heads, dim, window) for _ in range(batch)]
    for b in range(batch):
        k = rng.standard_normal((prefixes[b], width)).astype(np.float32)
        v = rng.standard_normal((prefixes[b], width)).astype(np.float32)
        kv.prefill(b, dev(k), dev(v))
        refs[b].prefill(k, v, prefixes[b])
    for step in range(13):
        k = rng.standard_normal((batch, width)).astype(np.float32)
        v = rng.standard_normal((batch, width)).astype(np.float32)
        q = rng.standard_normal((batch, width)).astype(np.float32)
        kv.push(dev(k), dev(v))
        for b in range(batch):
            refs[b].push(k[b], v[b])
        out = host(kv.attention(dev(q)))
        ctx.sync()
        for b in range(batch):
            n = refs[b].tokens()
            assert kv.state(b) == (n, refs[b].position())
            keys, values = (host(t) for t in kv.export(b))
            assert bits_equal(keys, refs[b].keys) and bits_equal(values, refs[b].values)
            ref = oracle.attention_decode(q[b], refs[b].keys, refs[b].values, heads)
            assert np.max(np.abs(out[b] - ref)) <= 1e-5 * max(1.0, float(np.max(np.abs(ref))))
    kv.free()


def test_cache_rope_uses_positions(ctx):
    rng = np.random.default_rng(12)
    batch, heads, dim, window = 2, 2, 4, 3
    width = heads * dim
    kv = A().KvCache(ctx, batch, heads, dim, window, max_prefix=6)
    r = A().Rope(ctx, dim, 10000.0, 64)
    for b, n in enumerate((6, 2)):
        z = np.zeros((n, width), np.float32)
        kv.prefill(b, dev(z), dev(z))
    pos = [6, 2]
    for step in range(5):
        q = rng.standard_normal((batch, width)).astype(np.float32)
        k = rng.standard_normal((batch, width)).astype(np.float32)
        qt, kt = dev(q), dev(k)
        kv.rope(r, qt, kt)
        kv.push(kt, kt)
        ctx.sync()
        for b in range(batch):
            assert bits_equal(host(qt)[b], oracle.rope(q[b], dim, pos[b]))
            assert bits_equal(host(kt)[b], oracle.rope(k[b], dim, pos[b]))
            pos[b] += 1
    kv.free()
    r.free()


def test_cache_errors(ctx):
    import torch
    import uocr_q8
    kv = A().KvCache(ctx, 2, 2, 2, 4, max_prefix=3)
    z = torch.zeros((3, 4), device="cuda")
    with pytest.raises(uocr_q8.OcrError) as e:
        kv.push(z[:2], z[:2])
    assert e.value.kind == "Shape"  # not prefilled
    kv.prefill(0, z, z)
    with pytest.raises(uocr_q8.OcrError) as e:
        kv.prefill(0, z, z)
    assert e.value.kind == "Shape"  # twice
    with pytest.raises(uocr_q8.OcrError) as e:
        kv.attention(z[:2])
    assert e.value.kind == "Shape"  # sequence 1 not prefilled
    with pytest.raises(uocr_q8.OcrError) as e:
        kv.prefill(1, torch.zeros((4, 4), device="cuda"), torch.zeros((4, 4), device="cuda"))
    assert e.value.kind == "Resource"  # longer than max_prefix
    for args in ((1, 0, 2, 4, 3), (1, 2, 2, 0, 3)):
        with pytest.raises(uocr_q8.OcrError) as e:
            A().KvCache(ctx, *args)
        assert e.value.kind == "Shape"
    kv.free()


@pytest.mark.parametrize("batch,heads,dim,prefix", [(1, 10, 128, 1517), (3, 2, 64, 100),
                                                     (2, 1, 256, 33), (5, 10, 128, 300)])
def test_split_attention_equals_one_cta_per_head(ctx, batch, heads, dim, prefix):
    """The split form (scores over token chunks, then softmax and value sums
    per 32-column slice) gives the one-CTA-per-head kernel's bits, across
    ragged prefixes and ring wraps, and matches the oracle."""
    import torch
    rng = np.random.default_rng(prefix + batch)
    width = heads * dim
    kv = A().KvCache(ctx, batch, heads, dim, 8, max_prefix=prefix)
    for b in range(batch):
        n = prefix - b
        kv.prefill(b, dev(rng.standard_normal((n, width)).astype(np.float32)),
                   dev(rng.standard_normal((n, width)).astype(np.float32)))
    for _ in range(11):  # the 8-token ring wraps
        kv.push(dev(rng.standard_normal((batch, width)).astype(np.float32)),
                dev(rng.standard_normal((batch, width)).astype(np.float32)))
    q = dev((rng.standard_normal((batch, width)) * 0.2).astype(np.float32))
    kv.set_attention_form(1)
    one = host(kv.attention(q))
    kv.set_attention_form(2)
    split = host(kv.attention(q))
    kv.set_attention_form(0)
    auto = host(kv.attention(q))
    ctx.sync()
    assert bits_equal(split, one)
    assert bits_equal(auto, one)
    for b in range(batch):
        k, v = (host(t) for t in kv.export(b))
        ref = oracle.attention_decode(host(q)[b], k, v, heads)
        assert np.max(np.abs(split[b] - ref)) <= 1e-5 * max(1.0, float(np.max(np.abs(ref))))
    bad = q.clone()
    bad[0, 0] = float("nan")
    kv.set_attention_form(2)
    kv.attention(bad)
    import uocr_q8
    with pytest.raises(uocr_q8.OcrError) as e:
        ctx.sync()
    assert e.value.kind == "Numerical"
    kv.free()
    small = A().KvCache(ctx, 1, 2, 8, 4, max_prefix=4)  # head_dim 8: no split form
    with pytest.raises(uocr_q8.OcrError) as e:
        small.set_attention_form(2)
    assert e.value.kind == "Unsupported"
    small.free()


# ---------------------------------------------------------------- prefill attention
def _token_major(a):
    """[heads, tokens, dim] -> token-major [tokens, heads * dim]."""
    return np.ascontiguousarray(np.transpose(a, (1, 0, 2)).reshape(a.shape[1], -1))


def _equal_values(a, b):
    """Bit-identical except for the sign of zeros (ops::attention sums its
    masked +0.0 products after the real ones; the device sums only the real
    ones)."""
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nz = b != 0
    return np.array_equal(a, b) and np.array_equal(a[nz].view(np.uint32), b[nz].view(np.uint32))


def test_prefill_attention_reference_cases(ctx):
    """tests/ops.rs:89-99 (future values excluded), :166-194 (masks across
    the reference's 128-query blocks: uniform weights, so every exp is exact
    and the outputs are the oracle's bit for bit) and :196-202 (zeros)."""
    from test_attention_oracle import causal_block_case
    q = np.zeros((2, 2), np.float32)
    v = np.array([[2.0, 4.0], [6.0, 8.0]], np.float32)
    out = host(A().attention_prefill_device(ctx, dev(q), dev(q), dev(v), 1))
    ctx.sync()
    assert out.ravel().tolist() == [2.0, 4.0, 4.0, 6.0]
    heads, tokens, dim = 2, 129, 3
    qh, vh = causal_block_case(heads, tokens, dim)
    out = host(A().attention_prefill_device(ctx, dev(_token_major(qh)), dev(_token_major(qh)),
                                            dev(_token_major(vh)), heads))
    ctx.sync()
    ref = _token_major(oracle.attention(qh, qh, vh, True))
    assert _equal_values(out, ref)
    h, t, c = np.meshgrid(np.arange(heads), np.arange(tokens), np.arange(dim), indexing="ij")
    want = _token_major(((h * 100 + c).astype(np.float32) + t.astype(np.float32) / 2))
    assert np.max(np.abs(out - want)) < 2e-4
    z = np.zeros((129, 3), np.float32)
    out = host(A().attention_prefill_device(ctx, dev(z), dev(z), dev(z), 1))
    ctx.sync()
    assert np.array_equal(out, z)


@pytest.mark.parametrize("heads,dim,tokens", [(3, 5, 37), (2, 64, 300), (10, 128, 257)])
def test_prefill_attention_matches_oracle(ctx, heads, dim, tokens):
    """Random inputs (the generic kernel for 3 x 5, the TMA kernel otherwise)
    against the oracle's causal ops::attention: 1e-5 relative (exp may round
    differently by one ulp); with keys equal within each head every exp is
    exact and the outputs are bit-identical up to the sign of zeros."""
    rng = np.random.default_rng(tokens)
    width = heads * dim
    q, k, v = (rng.standard_normal((tokens, width)).astype(np.float32) for _ in range(3))
    out = host(A().attention_prefill_device(ctx, dev(q), dev(k), dev(v), heads))
    ctx.sync()
    ref = oracle.attention_prefill(q, k, v, heads)
    assert np.max(np.abs(out - ref)) <= 1e-5 * max(1.0, float(np.max(np.abs(ref))))
    k = np.tile(rng.standard_normal(width).astype(np.float32), (tokens, 1))
    out = host(A().attention_prefill_device(ctx, dev(q), dev(k), dev(v), heads))
    ctx.sync()
    assert _equal_values(out, oracle.attention_prefill(q, k, v, heads))


def test_prefill_attention_full_prefix_sampled_rows(ctx):
    """The benchmark's prefill (1517 tokens, 10 heads of 128): sampled rows
    against the oracle's attention_decode over each row's prefix, which is the
    same arithmetic as its causal row."""
    rng = np.random.default_rng(1517)
    tokens, heads, dim = 1517, 10, 128
    width = heads * dim
    q, k, v = (rng.standard_normal((tokens, width)).astype(np.float32) for _ in range(3))
    out = host(A().attention_prefill_device(ctx, dev(q), dev(k), dev(v), heads))
    ctx.sync()
    for i in (0, 1, 31, 32, 33, 700, 1023, 1024, 1516):
        ref = oracle.attention_decode(q[i], k[:i + 1], v[:i + 1], heads)
        assert np.max(np.abs(out[i] - ref)) <= 1e-5 * max(1.0, float(np.max(np.abs(ref)))), i


@pytest.mark.parametrize("heads,dim", [(2, 8), (10, 128)])
def test_kv_prefill_attention_equals_token_major(ctx, heads, dim):
    """uocr_kv_attention_prefill over the cache (head-major or tiled layout)
    gives the token-major entry point's outputs bit for bit; rows other than
    the prefilled ones are Shape."""
    import uocr_q8
    rng = np.random.default_rng(dim)
    width, tokens = heads * dim, 45
    kv = A().KvCache(ctx, 2, heads, dim, 4, max_prefix=64)
    q, k, v = (rng.standard_normal((tokens, width)).astype(np.float32) for _ in range(3))
    kv.prefill(0, dev(rng.standard_normal((7, width)).astype(np.float32)),
               dev(rng.standard_normal((7, width)).astype(np.float32)))
    kv.prefill(1, dev(k), dev(v))
    out = host(kv.attention_prefill(1, dev(q)))
    ref = host(A().attention_prefill_device(ctx, dev(q), dev(k), dev(v), heads))
    ctx.sync()
    assert bits_equal(out, ref)
    with pytest.raises(uocr_q8.OcrError) as e:
        kv.attention_prefill(0, dev(q))
    assert e.value.kind == "Shape"
    kv.free()


@pytest.mark.parametrize("heads,tokens", [(10, 1517), (2, 33), (3, 16), (1, 17)])
def test_blocked_prefill_attention_equals_row_per_cta(ctx, heads, tokens):
    """The 16-rows-per-CTA causal prefill (head_dim 128, the default form)
    gives the one-row-per-CTA form's bits (forced with attention form 1),
    including the last partial block of rows; sampled rows against the oracle."""
    rng = np.random.default_rng(tokens + heads)
    dim = 128
    width = heads * dim
    q, k, v = (rng.standard_normal((tokens, width)).astype(np.float32) for _ in range(3))
    outs = []
    for form in (0, 1):
        kv = A().KvCache(ctx, 2, heads, dim, 8, max_prefix=tokens)
        kv.prefill(0, dev(rng.standard_normal((3, width)).astype(np.float32)),
                   dev(rng.standard_normal((3, width)).astype(np.float32)))
        kv.prefill(1, dev(k), dev(v))
        kv.set_attention_form(form)
        outs.append(host(kv.attention_prefill(1, dev(q))))
        ctx.sync()
        kv.free()
    assert bits_equal(outs[0], outs[1])
    for i in sorted({0, 1, 15, 16, tokens // 2, tokens - 1} & set(range(tokens))):
        ref = oracle.attention_decode(q[i], k[:i + 1], v[:i + 1], heads)
        assert np.max(np.abs(outs[0][i] - ref)) <= 1e-5 * max(1.0, float(np.max(np.abs(ref)))), i


def test_prefill_attention_errors(ctx):
    import torch
    import uocr_q8
    z = torch.zeros((4, 6), device="cuda")
    with pytest.raises(uocr_q8.OcrError) as e:
        A().attention_prefill_device(ctx, z, z, z, 4)
    assert e.value.kind == "Shape"
    bad = z.clone()
    bad[1, 0] = float("nan")
    A().attention_prefill_device(ctx, bad, z, z, 2)
    with pytest.raises(uocr_q8.OcrError) as e:
        ctx.sync()
    assert e.value.kind == "Numerical"


# ---------------------------------------------------------------- attention block
@pytest.mark.parametrize("mode", [0, 1])
def test_attention_block_matches_oracle(ctx, mode):
    """The attention half of Decoder::layer (src/decoder/mod.rs:241-341) for a
    batch of sequences at decode, three steps, vs the oracle composition."""
    import torch
    import uocr_q8
    from helpers import random_q8
    rng = np.random.default_rng(20 + mode)
    batch, heads, dim, window, prefix = 4, 10, 128, 4, 37
    H = heads * dim
    mats = [oracle.Matrix(*random_q8(rng, H, H, 1e-3, 2e-3)) for _ in range(4)]
    dmats = [uocr_q8.Int8Matrix.from_parts(H, H, m.w, m.s, ctx) for m in mats]
    norm = rng.uniform(0.5, 1.5, H).astype(np.float32)
    kv = A().KvCache(ctx, batch, heads, dim, window, max_prefix=prefix)
    rope = A().Rope(ctx, dim, 10000.0, 4096)
    refs = []
    for b in range(batch):
        k = rng.standard_normal((prefix, H)).astype(np.float32)
        v = rng.standard_normal((prefix, H)).astype(np.float32)
        kv.prefill(b, dev(k), dev(v))
        c = oracle.LayerCache(heads, dim, window)
        c.prefill(k, v, prefix)
        refs.append(c)
    block = A().AttentionBlock(ctx, dev(norm), *dmats, kv, rope)
    lin = oracle.linear_dynamic_int8 if mode == 1 else oracle.linear
    for step in range(3):
        x = rng.standard_normal((batch, H)).astype(np.float32)
        y = host(block.forward_device(dev(x), mode))
        ctx.sync()
        for b in range(batch):
            c = refs[b]
            n = oracle.rms_norm(x[b:b + 1], norm)
            q, k, v = (lin(m, n)[0] for m in mats[:3])
            pos = c.position()
            q, k = oracle.rope(q, dim, pos), oracle.rope(k, dim, pos)
            c.push(k, v)
            a = oracle.attention_decode(q, c.keys, c.values, heads)
            ref = lin(mats[3], a[None])[0] + x[b]
            err = np.max(np.abs(y[b].astype(np.float64) - ref))
            # int8 mode: a one-ulp attention difference can move one activation
            # quantization step of the o projection (the MoE layer tolerance)
            tol = 1e-3 if mode == 1 else 1e-4
            assert err <= tol * float(np.max(np.abs(ref))), (step, b, err)
    kv.free()
    rope.free()


@pytest.mark.parametrize("heads,dim", [(2, 8), (10, 128)])
def test_rope_push_qkv_equals_rope_then_push(ctx, heads, dim):
    """uocr_kv_rope_push_qkv on fused [q | k | v] rows equals uocr_kv_rope
    followed by uocr_kv_push on the separate rows, bit for bit (q and the
    cache contents), across ring wraps, for the plain and tiled layouts."""
    import torch
    rng = np.random.default_rng(31 + dim)
    batch, window, prefix = 3, 4, 5
    width = heads * dim
    a = A().KvCache(ctx, batch, heads, dim, window, prefix)
    b = A().KvCache(ctx, batch, heads, dim, window, prefix)
    rope = A().Rope(ctx, dim, 10000.0, 64)
    for s in range(batch):
        k = dev(rng.standard_normal((prefix - s, width)).astype(np.float32))
        a.prefill(s, k, k)
        b.prefill(s, k, k)
    for step in range(6):
        qkv = dev(rng.standard_normal((batch, 3 * width)).astype(np.float32))
        q1 = a.rope_push_qkv(rope, qkv)
        q2, k2, v2 = (qkv[:, i * width:(i + 1) * width].contiguous() for i in range(3))
        b.rope(rope, q2, k2)
        b.push(k2, v2)
        ctx.sync()
        assert bits_equal(host(q1), host(q2)), step
        for s in range(batch):
            assert a.state(s) == b.state(s)
            for x, y in zip(a.export(s), b.export(s)):
                assert bits_equal(host(x), host(y)), (step, s)
    a.free()
    b.free()
    rope.free()
