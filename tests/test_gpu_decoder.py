"""GPU parity of a batched decode step (Decoder::step, src/decoder/mod.rs:
241-420) against the oracle's composition of the same reference operations,
on a small decoder with a dense layer and an MoE layer, across ring wraps of
the KV cache; and the pieces the step adds: Decoder::feed_forward and the
BF16 router linear."""
import numpy as np
import pytest

import oracle
from helpers import bits_equal, random_q8

pytestmark = pytest.mark.gpu


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def test_linear_bf16_bit_exact(ctx):
    from uocr_q8.decoder import linear_bf16_device
    rng = np.random.default_rng(1)
    for n, k, rows in ((64, 1280, 64), (7, 33, 3), (130, 256, 1)):
        # bf16 bit patterns of N(0, 1) * 2^[-20, 20] weights (tail bits kept)
        wf = (rng.standard_normal((n, k)) * 2.0 ** rng.integers(-20, 21, (n, k))).astype(np.float32)
        w = (wf.view(np.uint32) >> 16).astype(np.uint16)
        x = rng.standard_normal((rows, k)).astype(np.float32)
        y = host(linear_bf16_device(ctx, dev(w.view(np.int16)), dev(x)))
        ctx.sync()
        assert bits_equal(y, oracle.linear_bf16(w, x)), (n, k, rows)


def _bf16_bits(rng, shape, scale):
    w = (rng.standard_normal(shape) * scale).astype(np.float32)
    return (w.view(np.uint32) >> 16).astype(np.uint16)


def _check_fp32(y, w_bits, x, rows_idx=None):
    """FP32 tolerance, as the tensor-core FP32 tests: normalised by
    max(|ref|, sum |w x| * 2^-10), <= 1e-4 against the exact product (float64
    of the bf16 weights) and <= 2e-4 against the reference's left-to-right
    sums (oracle), whose own order has an error of the same size."""
    idx = np.arange(w_bits.shape[0]) if rows_idx is None else rows_idx
    ws = w_bits[idx]
    wf = (ws.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    x64 = x.astype(np.float64)
    exact = x64 @ wf.T
    terms = np.abs(x64) @ np.abs(wf).T
    got = y[:, idx].astype(np.float64)
    floor = terms * 2.0 ** -10

    def err(ref):
        denom = np.maximum(np.abs(ref), floor)
        return float(np.max(np.abs(got - ref) / np.where(denom == 0, 1, denom)))

    e_exact, e_oracle = err(exact), err(oracle.linear_bf16(ws, x).astype(np.float64))
    assert e_exact <= 1e-4, e_exact
    assert e_oracle <= 2e-4, e_oracle
    return e_exact


@pytest.mark.parametrize("n,k,rows", [(130, 64, 1), (1000, 256, 17), (300, 128, 65),
                                      (517, 1280, 64)])
def test_linear_bf16_tc_matches_oracle(ctx, n, k, rows):
    """The tensor-core BF16 linear (exact products, FP32 accumulation) against
    the reference's sequential sums: ragged weight tiles (n not a multiple of
    128), one row, two row tiles, the lm_head's K."""
    from uocr_q8.decoder import linear_bf16_tc_device
    rng = np.random.default_rng(n + k + rows)
    w = _bf16_bits(rng, (n, k), 0.05)
    x = (rng.standard_normal((rows, k)) * rng.uniform(0.1, 10, (rows, 1))).astype(np.float32)
    y = host(linear_bf16_tc_device(ctx, dev(w.view(np.int16)), dev(x)))
    ctx.sync()
    _check_fp32(y, w, x)


@pytest.mark.slow
def test_linear_bf16_tc_lm_head_size(ctx):
    """The BF16 lm_head at its full size, 129,280 x 1280, batch 64: sampled
    output rows against the oracle (the whole product is 10.6 G sequential
    multiply-adds on the host)."""
    from uocr_q8.decoder import linear_bf16_tc_device
    rng = np.random.default_rng(129280)
    w = _bf16_bits(rng, (129280, 1280), 0.03)
    x = rng.standard_normal((64, 1280)).astype(np.float32)
    y = host(linear_bf16_tc_device(ctx, dev(w.view(np.int16)), dev(x)))
    ctx.sync()
    idx = np.concatenate([np.arange(0, 256), rng.choice(129280, 512, replace=False),
                          np.arange(129280 - 128, 129280)])
    _check_fp32(y, w, x, idx)


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("rows", [1, 5, 40])
def test_feed_forward_matches_oracle(ctx, mode, rows):
    import uocr_q8
    from uocr_q8.decoder import feed_forward_device
    rng = np.random.default_rng(10 * mode + rows)
    H, F = 256, 384
    g, u, d = (oracle.Matrix(*random_q8(rng, *shape)) for shape in ((F, H), (F, H), (H, F)))
    dm = [uocr_q8.Int8Matrix.from_parts(m.rows, m.cols, m.w, m.s, ctx) for m in (g, u, d)]
    x = rng.standard_normal((rows, H)).astype(np.float32)
    y = host(feed_forward_device(ctx, *dm, dev(x), mode))
    ctx.sync()
    ref = oracle.feed_forward(oracle.Ffn(g, u, d), x, mode)
    if mode == 2 or (mode == 1 and rows == 1):
        # int8 projections are bit-exact; silu's exp may differ by an ulp
        assert float(np.mean(y.view(np.uint32) == ref.view(np.uint32))) >= 0.99
        assert np.max(np.abs(y - ref)) <= 1e-3 * float(np.max(np.abs(ref)))
    else:
        assert np.max(np.abs(y.astype(np.float64) - ref)) <= 1e-4 * float(np.max(np.abs(ref)))


def small_config():
    """Two layers: a dense FFN of width 352 (padded to 384 on the device) and
    an MoE layer of 8 experts."""
    from uocr_q8.decoder import DecoderConfig
    return DecoderConfig(hidden=256, heads=2, layers=2, first_dense=1, experts=8, top_k=2,
                         expert_width=128, shared_width=256, dense_width=352, vocab=384, window=4)


def host_decoder(dec):
    """The device weights as oracle objects."""
    import torch

    def m(x):
        w, s = x.download()
        return oracle.Matrix(w, s)

    layers = []
    for L in dec.layers:
        w, s = L.qkv.download()
        H = w.shape[1]
        d = {"in": host(L.input_norm), "post": host(L.post_norm), "o": m(L.o)}
        for i, key in enumerate(("q", "k", "v")):
            d[key] = oracle.Matrix(w[i * H:(i + 1) * H].copy(), s[i * H:(i + 1) * H].copy())
        if L.moe is not None:
            shared, experts = L.moe._keep
            d["shared"] = oracle.Ffn(*[m(x) for x in shared])
            d["experts"] = [oracle.Ffn(*[m(x) for x in e]) for e in experts]
            d["router"] = host(L.router.view(torch.int16)).view(np.uint16)
        else:
            # the unpadded FFN (the device one is zero-padded to a multiple of 128)
            F = L.dense_width
            (gw, gs), (uw, us), (dw, ds) = (x.download() for x in L.dense)
            d["dense"] = oracle.Ffn(oracle.Matrix(gw[:F].copy(), gs[:F].copy()),
                                    oracle.Matrix(uw[:F].copy(), us[:F].copy()),
                                    oracle.Matrix(dw[:, :F].copy(), ds[:, :F // 32].copy()))
        layers.append(d)
    emb = (host(dec.embedding.view(torch.int16)).view(np.uint16).astype(np.uint32) << 16).view(
        np.float32)
    if isinstance(dec.lm_head, torch.Tensor):  # BF16 head: its bit patterns
        head = host(dec.lm_head.view(torch.int16)).view(np.uint16)
    else:
        head = m(dec.lm_head)
    return layers, emb, host(dec.final_norm), head


def oracle_step(cfg, layers, emb, final_norm, head, caches, token, mode):
    """Decoder::step for one sequence with the oracle's operations."""
    int8 = mode != 0
    proj = (lambda mat, v: oracle.linear_dynamic_int8(mat, v)) if int8 else \
        (lambda mat, v: oracle.linear(mat, v))
    x = emb[token][None]
    for L, c in zip(layers, caches):
        n = oracle.rms_norm(x, L["in"], cfg.eps)
        q, k, v = (proj(L[key], n)[0] for key in ("q", "k", "v"))
        pos = c.position()
        q, k = oracle.rope(q, cfg.head_dim, pos, cfg.theta), oracle.rope(k, cfg.head_dim, pos, cfg.theta)
        c.push(k, v)
        a = oracle.attention_decode(q, c.keys, c.values, cfg.heads)
        r = proj(L["o"], a[None])[0] + x[0]
        n2 = oracle.rms_norm(r[None], L["post"], cfg.eps)
        if "dense" in L:
            y = oracle.feed_forward(L["dense"], n2, 1 if int8 else 0)
        else:
            logits = oracle.linear_bf16(L["router"], n2)
            y, _, _ = oracle.experts(L["shared"], L["experts"], logits, n2, cfg.top_k, 1 if int8 else 0)
        x = (r + y[0])[None]
    h = oracle.rms_norm(x, final_norm, cfg.eps)
    if isinstance(head, np.ndarray):  # BF16 head (ops::linear_weight)
        return oracle.linear_bf16(head, h)[0]
    return proj(head, h)[0]


@pytest.mark.parametrize("mode,head", [(0, "q8"), (2, "q8"), (0, "bf16")])
def test_decode_step_matches_oracle(ctx, mode, head):
    import torch
    from uocr_q8.decoder import DecodeState, Decoder, decode_step
    cfg = small_config()
    dec = Decoder.random(ctx, cfg, seed=5 + mode, lm_head=head)
    layers, emb, final_norm, head = host_decoder(dec)
    batch, prefix = 3, 6
    state = DecodeState(dec, batch, prefix)
    rng = np.random.default_rng(7)
    caches = []
    for b in range(batch):
        seq = []
        for li, cache in enumerate(state.caches):
            k = rng.standard_normal((prefix - b, cfg.hidden)).astype(np.float32)
            v = rng.standard_normal((prefix - b, cfg.hidden)).astype(np.float32)
            cache.prefill(b, dev(k), dev(v))
            c = oracle.LayerCache(cfg.heads, cfg.head_dim, cfg.window)
            c.prefill(k, v, prefix - b)
            seq.append(c)
        caches.append(seq)
    for step in range(6):  # the 4-token ring wraps
        tokens = rng.integers(0, cfg.vocab, batch)
        logits = host(decode_step(dec, state, dev(tokens.astype(np.int64)), mode))
        ctx.sync()
        for b in range(batch):
            ref = oracle_step(cfg, layers, emb, final_norm, head, caches[b], int(tokens[b]), mode)
            scale = float(np.max(np.abs(ref)))
            err = float(np.max(np.abs(logits[b].astype(np.float64) - ref)))
            assert err <= (1e-3 if mode == 0 else 1e-2) * scale, (step, b, err, scale)
            assert int(np.argmax(logits[b])) == int(np.argmax(ref)) or \
                np.sort(ref)[-1] - np.sort(ref)[-2] < 2 * err
    for b in range(batch):
        assert state.caches[0].state(b) == (caches[b][0].tokens(), caches[b][0].position())
    state.free()


def oracle_prefill(cfg, layers, final_norm, head, x, mode):
    """Decoder::prefill (src/decoder/mod.rs:382-398) of embedding rows x with
    the oracle's operations; returns the layer caches and the logits."""
    T = x.shape[0]
    dyn = mode == 2 or (mode == 1 and T == 1)
    proj = (lambda mat, v: oracle.linear_dynamic_int8(mat, v)) if dyn else \
        (lambda mat, v: oracle.linear(mat, v))
    caches = []
    for L in layers:
        n = oracle.rms_norm(x, L["in"], cfg.eps)
        q, k, v = (proj(L[key], n) for key in ("q", "k", "v"))
        q = np.stack([oracle.rope(q[i], cfg.head_dim, i, cfg.theta) for i in range(T)])
        k = np.stack([oracle.rope(k[i], cfg.head_dim, i, cfg.theta) for i in range(T)])
        c = oracle.LayerCache(cfg.heads, cfg.head_dim, cfg.window)
        c.prefill(k, v, T)
        caches.append(c)
        a = oracle.attention_prefill(q, k, v, cfg.heads)
        r = proj(L["o"], a) + x
        n2 = oracle.rms_norm(r, L["post"], cfg.eps)
        if "dense" in L:
            y = oracle.feed_forward(L["dense"], n2, mode)
        else:
            logits = oracle.linear_bf16(L["router"], n2)
            y, _, _ = oracle.experts(L["shared"], L["experts"], logits, n2, cfg.top_k, mode)
        x = r + y
    h = oracle.rms_norm(x[T - 1:], final_norm, cfg.eps)
    if isinstance(head, np.ndarray):
        return caches, oracle.linear_bf16(head, h)[0]
    lin = oracle.linear_dynamic_int8 if mode != 0 else oracle.linear
    return caches, lin(head, h)[0]


def _close(got, ref, tol):
    scale = float(np.max(np.abs(ref)))
    err = float(np.max(np.abs(got.astype(np.float64) - ref)))
    assert err <= tol * scale, (err, scale)
    assert int(np.argmax(got)) == int(np.argmax(ref)) or \
        np.sort(ref)[-1] - np.sort(ref)[-2] < 2 * err


@pytest.mark.parametrize("mode,head,tokens", [(0, "q8", 37), (1, "q8", 37), (1, "q8", 1),
                                              (2, "q8", 20), (0, "bf16", 70)])
def test_prefill_then_decode_matches_oracle(ctx, mode, head, tokens):
    """Decoder::prefill of one sequence (causal attention over its rows, the
    MoE over all rows with the reference's per-group arithmetic) and then
    teacher-forced Decoder::step calls, as in the fixed-work benchmark
    (src/model/benchmark.rs:37-50), against the oracle: the prefill logits,
    the caches' contents and every step's logits.  DynamicActivations runs a
    multi-row prefill with FP32 activations and every decode projection with
    int8 ones."""
    import torch
    from uocr_q8.decoder import DecodeState, Decoder, decode_step, prefill
    cfg = small_config()
    dec = Decoder.random(ctx, cfg, seed=40 + mode, lm_head=head)
    layers, emb, final_norm, head_h = host_decoder(dec)
    rng = np.random.default_rng(41 + tokens)
    x = rng.standard_normal((tokens, cfg.hidden)).astype(np.float32)
    state = DecodeState(dec, 1, tokens)
    logits = host(prefill(dec, state, dev(x), mode))
    ctx.sync()
    caches, ref = oracle_prefill(cfg, layers, final_norm, head_h, x, mode)
    tol = 1e-3 if mode == 0 else 1e-2
    _close(logits[0], ref, tol)
    for cache, c in zip(state.caches, caches):
        keys, values = (host(t) for t in cache.export(0)[:2])
        kerr = float(np.max(np.abs(keys - c.keys)))
        assert kerr <= tol * float(np.max(np.abs(c.keys)))
        assert float(np.max(np.abs(values - c.values))) <= tol * float(np.max(np.abs(c.values)))
    # continue from the oracle's own caches: each side follows its own state
    for step in range(6):  # the 4-token ring wraps
        token = int(rng.integers(0, cfg.vocab))
        got = host(decode_step(dec, state, dev(np.array([token], np.int64)), mode))
        ctx.sync()
        ref = oracle_step(cfg, layers, emb, final_norm, head_h, caches, token, mode)
        _close(got[0], ref, tol)
    assert state.caches[0].state(0) == (caches[0].tokens(), caches[0].position())
    state.free()


@pytest.mark.parametrize("mode", [0, 2])
def test_decode_step_with_peer_experts_matches_plain(ctx, mode):
    """The decode step with its MoE layers through the expert-parallel
    exchange (uocr_ep_*, a world of this GPU alone) against the plain step on
    the same state: int8 activations bit for bit, FP32 activations within the
    decode tolerance, over steps that wrap the cache ring."""
    from uocr_q8.decoder import DecodeState, Decoder, decode_step
    from uocr_q8.expert_parallel import decoder_peer_experts
    cfg = small_config()
    dec = Decoder.random(ctx, cfg, seed=60 + mode)
    batch, prefix = 3, 5
    states = [DecodeState(dec, batch, prefix) for _ in range(2)]
    rng = np.random.default_rng(61)
    for b in range(batch):
        for li in range(cfg.layers):
            k = dev(rng.standard_normal((prefix, cfg.hidden)).astype(np.float32))
            v = dev(rng.standard_normal((prefix, cfg.hidden)).astype(np.float32))
            for st in states:
                st.caches[li].prefill(b, k, v)
    eps = decoder_peer_experts(dec, batch)
    assert sum(e is not None for e in eps) == cfg.layers - cfg.first_dense
    for step in range(6):
        tokens = dev(rng.integers(0, cfg.vocab, batch).astype(np.int64))
        plain = host(decode_step(dec, states[0], tokens, mode))
        peer = host(decode_step(dec, states[1], tokens, mode, experts=eps))
        ctx.sync()
        if mode == 2:
            assert bits_equal(peer, plain), step
        else:
            scale = float(np.max(np.abs(plain)))
            assert float(np.max(np.abs(peer.astype(np.float64) - plain))) <= 1e-3 * scale, step
    for e in eps:
        if e is not None:
            e.free()
    for st in states:
        st.free()


def test_logits_checksum_wraps_like_the_reference(ctx):
    """uocr_bits_checksum: the u64 wrapping sum of the logits' bit patterns
    (src/model/benchmark.rs:43-47), accumulated over calls."""
    import torch
    from uocr_q8.decoder import logits_checksum_device
    rng = np.random.default_rng(3)
    acc = torch.zeros(1, dtype=torch.int64, device="cuda")
    want = 0
    for n in (1, 129280, 1000003):
        x = rng.standard_normal(n).astype(np.float32)
        x[: n // 3] = -x[: n // 3]
        logits_checksum_device(ctx, dev(x), acc)
        want = (want + int(x.view(np.uint32).astype(np.uint64).sum())) % (1 << 64)
    # push the sum across 2^64 to check the wrap
    big = np.full(1 << 20, np.uint32(0xFFFFFFFF)).view(np.float32)
    for _ in range(3):
        logits_checksum_device(ctx, dev(big), acc)
        want = (want + (1 << 20) * 0xFFFFFFFF) % (1 << 64)
    ctx.sync()
    got = int(host(acc).view(np.uint64)[0])
    assert got == want


def test_cache_reset_then_prefill_again(ctx):
    """uocr_kv_reset empties a sequence: attention before the new prefill is
    Shape, and the new prefill gives a fresh cache."""
    import torch
    import uocr_q8
    from uocr_q8.attention import KvCache
    kv = KvCache(ctx, 1, 2, 8, 4, max_prefix=10)
    a = torch.randn((10, 16), device="cuda")
    kv.prefill(0, a, a)
    kv.push(a[:1], a[:1])
    kv.reset(0)
    with pytest.raises(uocr_q8.OcrError) as e:
        kv.attention(a[:1])
    assert e.value.kind == "Shape"
    b = torch.randn((6, 16), device="cuda")
    kv.prefill(0, b, b * 2)
    k, v, _ = (kv.export(0) + (None,))
    ctx.sync()
    assert kv.state(0) == (6, 6)
    assert torch.equal(k, b) and torch.equal(v, b * 2)
    kv.free()


@pytest.mark.slow
@pytest.mark.parametrize("mode", [0, 2])
def test_decode_step_config4_shapes(ctx, mode):
    """The decode step at the upstream decoder's shapes: hidden 1280, 10 heads
    of 128, a dense FFN of width 6848 and an MoE layer of 64 experts (top-6,
    width 896) plus the 1792-wide shared expert, the q8 lm_head over the full
    129,280-token vocabulary; 8 sequences with 2048-token prefixes (ragged),
    five steps.  Two layers (one of each kind) and a 4-token ring, so that the
    ring wraps within the steps; the 12-layer step repeats these layers."""
    from uocr_q8.decoder import DecodeState, Decoder, DecoderConfig, decode_step
    cfg = DecoderConfig(layers=2, window=4)
    dec = Decoder.random(ctx, cfg, seed=31 + mode)
    layers, emb, final_norm, head = host_decoder(dec)
    batch, prefix = 8, 2048
    state = DecodeState(dec, batch, prefix)
    rng = np.random.default_rng(17 + mode)
    caches = []
    for b in range(batch):
        seq = []
        for cache in state.caches:
            n = prefix - 3 * b
            k = rng.standard_normal((n, cfg.hidden)).astype(np.float32)
            v = rng.standard_normal((n, cfg.hidden)).astype(np.float32)
            cache.prefill(b, dev(k), dev(v))
            c = oracle.LayerCache(cfg.heads, cfg.head_dim, cfg.window)
            c.prefill(k, v, n)
            seq.append(c)
        caches.append(seq)
    for step in range(5):
        tokens = rng.integers(0, cfg.vocab, batch)
        logits = host(decode_step(dec, state, dev(tokens.astype(np.int64)), mode))
        ctx.sync()
        for b in range(batch):
            ref = oracle_step(cfg, layers, emb, final_norm, head, caches[b], int(tokens[b]), mode)
            scale = float(np.max(np.abs(ref)))
            err = float(np.max(np.abs(logits[b].astype(np.float64) - ref)))
            assert err <= (1e-3 if mode == 0 else 1e-2) * scale, (step, b, err, scale)
            assert int(np.argmax(logits[b])) == int(np.argmax(ref)) or \
                np.sort(ref)[-1] - np.sort(ref)[-2] < 2 * err
    for b in range(batch):
        assert state.caches[1].state(b) == (caches[b][1].tokens(), caches[b][1].position())
    state.free()
