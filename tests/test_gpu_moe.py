"""GPU parity of routing and the MoE FFN layer (Decoder::experts) vs the oracle.

Routing: selected ids exact, weights bit-exact (exp is evaluated so that it
rounds like libm's expf except in rare boundary cases; a one-ulp difference
is tolerated and counted).  FP32-activation layer: max |y - ref| <=
1e-4 * max |ref|.  int8-activation layer: every projection is bit-exact given
identical inputs; end to end, a silu value that rounds differently can flip
one activation rounding, so >= 99% of outputs must be bit-identical and the
rest within 1e-3 * max |ref|.
"""
import numpy as np
import pytest

import oracle
from helpers import bits_equal, random_q8

pytestmark = pytest.mark.gpu

LAYER_FP32_TOL = 1e-4
LAYER_INT8_TOL = 1e-3


def q8():
    import uocr_q8
    return uocr_q8


def make_layer(ctx, rng, H, F, FS, E, k, normalize=False, scale=1.0):
    M = q8().Int8Matrix

    def ffn(width):
        mats, host = [], []
        for r, c in ((width, H), (width, H), (H, width)):
            w, s = random_q8(rng, r, c)
            mats.append(M.from_parts(r, c, w, s, ctx))
            host.append(oracle.Matrix(w, s))
        return mats, oracle.Ffn(*host)

    shared, shared_o = ffn(FS)
    experts, experts_o = zip(*[ffn(F) for _ in range(E)])
    layer = q8().MoeLayer(ctx, shared, experts, k, normalize, scale)
    return layer, shared_o, list(experts_o)


def ulps(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


# ---------------------------------------------------------------- routing
def test_route_known_answers(ctx):
    import torch
    logits = torch.zeros((1, 4), device="cuda")
    ids, w = q8().route_device(ctx, logits, 2)
    ctx.sync()
    assert ids.cpu().tolist() == [[0, 1]] and w.cpu().tolist() == [[0.25, 0.25]]
    ids, w = q8().route_device(ctx, logits, 2, True, 2.0)
    ctx.sync()
    assert ids.cpu().tolist() == [[0, 1]] and w.cpu().tolist() == [[1.0, 1.0]]


@pytest.mark.parametrize("normalize,scale", [(False, 1.0), (True, 2.5)])
def test_route_vs_oracle(ctx, normalize, scale):
    import torch
    rng = np.random.default_rng(7)
    logits = rng.standard_normal((300, 64)).astype(np.float32)
    ids, w = q8().route_device(ctx, torch.from_numpy(logits).cuda(), 6, normalize, scale)
    ctx.sync()
    ids, w = ids.cpu().numpy(), w.cpu().numpy()
    for t in range(300):
        ref = oracle.route(logits[t], 6, normalize, scale)
        assert ids[t].tolist() == [i for i, _ in ref]
        assert ulps(w[t], [p for _, p in ref]).max() <= 1


def test_route_errors(ctx):
    import torch
    bad = torch.zeros((2, 8), device="cuda")
    bad[1, 3] = float("nan")
    q8().route_device(ctx, bad, 2)
    with pytest.raises(q8().OcrError) as e:
        ctx.sync()
    assert e.value.kind == "Numerical"
    with pytest.raises(q8().OcrError) as e:
        q8().route_device(ctx, bad, 9)
    assert e.value.kind == "Shape"
    with pytest.raises(q8().OcrError) as e:
        q8().route_device(ctx, bad, 2, False, 0.0)
    assert e.value.kind == "Shape"


# ---------------------------------------------------------------- decode (1 token)
@pytest.fixture(scope="module")
def config1(ctx):
    """The MoE layer of the upstream decoder: hidden 1280, 64 experts of width
    896, top-6, a fused shared expert of width 1792."""
    rng = np.random.default_rng(1)
    return make_layer(ctx, rng, 1280, 896, 1792, 64, 6)


def _check_layer(y, ref, ids, ids_ref, wts, wts_ref, int8):
    assert np.array_equal(ids, ids_ref)
    assert ulps(wts, wts_ref).max() <= 1
    scale = float(np.max(np.abs(ref)))
    err = float(np.max(np.abs(y.astype(np.float64) - ref)))
    if int8:
        same = float(np.mean(y.view(np.uint32) == ref.view(np.uint32)))
        print(f"int8 layer outputs bit-identical to the oracle: {same:.5f}")
        assert same >= 0.99, same
        assert err <= LAYER_INT8_TOL * scale
    else:
        assert err <= LAYER_FP32_TOL * scale


@pytest.mark.parametrize("mode", [0, 1])
def test_decode_config1(ctx, config1, mode):
    layer, sh, ex = config1
    rng = np.random.default_rng(100 + mode)
    for trial in range(3):
        x = rng.standard_normal((1, 1280)).astype(np.float32)
        logits = rng.standard_normal((1, 64)).astype(np.float32)
        y, ids, wts = layer.forward(x, logits, mode)
        ref, ids_ref, wts_ref = oracle.experts(sh, ex, logits, x, 6, mode)
        _check_layer(y, ref, ids, ids_ref, wts, wts_ref, mode != 0)


def test_decode_device_repeatable(ctx, config1):
    import torch
    layer = config1[0]
    rng = np.random.default_rng(5)
    x = torch.from_numpy(rng.standard_normal((1, 1280)).astype(np.float32)).cuda()
    lg = torch.from_numpy(rng.standard_normal((1, 64)).astype(np.float32)).cuda()
    a = torch.empty_like(x)
    b = torch.empty_like(x)
    torch.cuda.synchronize()
    layer.forward_device(x, lg, 0, y_t=a)
    for _ in range(5):
        layer.forward_device(x, lg, 0, y_t=b)
    ctx.sync()
    assert torch.equal(a, b)


def test_decode_host_calls_replay_graphs(ctx, config1):
    """The host-buffer decode call runs eagerly for the first call of a
    (layer, mode) and from a captured graph afterwards: every call equals
    the device-pointer call bit for bit, across two layers and both modes
    interleaved, and an error raised inside a replayed graph is reported and
    cleared."""
    import torch
    from uocr_q8 import _ptr, lib, _check
    layer_a = config1[0]
    rng = np.random.default_rng(9)
    layer_b = make_layer(ctx, rng, 1280, 896, 1792, 64, 6)[0]
    for call in range(6):
        for layer in (layer_a, layer_b):
            for mode in (0, 1):
                x = rng.standard_normal((1, 1280)).astype(np.float32)
                lg = rng.standard_normal((1, 64)).astype(np.float32)
                y, ids, wts = layer.forward(x, lg, mode)
                yd = layer.forward_device(torch.from_numpy(x).cuda(), torch.from_numpy(lg).cuda(),
                                          mode)
                ctx.sync()
                assert bits_equal(y, yd.cpu().numpy()), (call, mode)
                # y only (no routing outputs): the same graph family, other key
                y2 = np.empty_like(x)
                _check(lib().uocr_moe_forward_host(ctx.handle, layer._h, mode, _ptr(x), _ptr(lg),
                                                   1, _ptr(y2), None, None))
                assert bits_equal(y2, y)
    bad = np.zeros((1, 64), np.float32)
    bad[0, 5] = np.nan
    with pytest.raises(q8().OcrError) as e:
        layer_a.forward(np.zeros((1, 1280), np.float32), bad, 0)
    assert e.value.kind == "Numerical"
    x = rng.standard_normal((1, 1280)).astype(np.float32)
    lg = rng.standard_normal((1, 64)).astype(np.float32)
    y, _, _ = layer_a.forward(x, lg, 0)  # the status was cleared
    yd = layer_a.forward_device(torch.from_numpy(x).cuda(), torch.from_numpy(lg).cuda(), 0)
    ctx.sync()
    assert bits_equal(y, yd.cpu().numpy())
    layer_b.free()


def test_decode_rejects_bad_logits(ctx, config1):
    layer = config1[0]
    x = np.zeros((1, 1280), np.float32)
    logits = np.zeros((1, 64), np.float32)
    logits[0, 3] = np.inf
    with pytest.raises(q8().OcrError) as e:
        layer.forward(x, logits, 0)
    assert e.value.kind == "Numerical"


# ---------------------------------------------------------------- prefill (many tokens)
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_prefill_small(ctx, mode):
    rng = np.random.default_rng(40 + mode)
    layer, sh, ex = make_layer(ctx, rng, 128, 64, 128, 8, 3)
    T = 37
    x = rng.standard_normal((T, 128)).astype(np.float32)
    logits = rng.standard_normal((T, 8)).astype(np.float32)
    logits[5, 2] += 4.0  # a group of size one for expert 2 is likely
    y, ids, wts = layer.forward(x, logits, mode)
    ref, ids_ref, wts_ref = oracle.experts(sh, ex, logits, x, 3, mode)
    # mode 1 (the reference's dispatch) runs every multi-row group, and the
    # shared expert, with FP32 activations: FP32 tolerance applies.
    _check_layer(y, ref, ids, ids_ref, wts, wts_ref, mode == 2)


@pytest.mark.parametrize("T", [2, 65, 150])
def test_prefill_tensor_core_fp32(ctx, T):
    """FP32 activations on the tensor cores (exact bf16 pieces): gathered
    rows per expert, grouped projections, ragged groups and tiles."""
    rng = np.random.default_rng(800 + T)
    layer, sh, ex = make_layer(ctx, rng, 256, 128, 256, 8, 2)
    x = rng.standard_normal((T, 256)).astype(np.float32)
    logits = rng.standard_normal((T, 8)).astype(np.float32)
    logits[:, 5] += 1.5
    y, ids, wts = layer.forward(x, logits, 0)
    ref, ids_ref, wts_ref = oracle.experts(sh, ex, logits, x, 2, 0)
    _check_layer(y, ref, ids, ids_ref, wts, wts_ref, False)


@pytest.mark.parametrize("T", [2, 3, 65, 150])
def test_prefill_tensor_core_dynamic(ctx, T):
    """QuantizationMode::DynamicActivations on tensor-core shapes: groups of
    one row take the bit-exact int8 kernel, the others the FP32 kernel (the
    reference's dispatch, src/decoder/mod.rs:103-106); the shared expert runs
    FP32 for more than one token.  FP32 tolerance end to end; a layer whose
    tokens each choose distinct experts (every group one row) is checked
    against the all-int8 layer bit for bit in the routed part."""
    rng = np.random.default_rng(700 + T)
    layer, sh, ex = make_layer(ctx, rng, 256, 128, 256, 8, 2)
    x = rng.standard_normal((T, 256)).astype(np.float32)
    logits = rng.standard_normal((T, 8)).astype(np.float32)
    if T > 3:
        logits[:, 5] += 1.5
    y, ids, wts = layer.forward(x, logits, 1)
    ref, ids_ref, wts_ref = oracle.experts(sh, ex, logits, x, 2, 1)
    _check_layer(y, ref, ids, ids_ref, wts, wts_ref, False)


def test_prefill_dynamic_single_row_groups_are_int8(ctx):
    """Tokens routed to disjoint experts: every routed group has one row, so
    the routed part equals int8 activations; with the shared expert's FP32
    part identical in both runs, mode 1 and mode 2 differ only through it."""
    import torch
    rng = np.random.default_rng(71)
    layer, sh, ex = make_layer(ctx, rng, 256, 128, 256, 8, 2)
    x = rng.standard_normal((3, 256)).astype(np.float32)
    logits = np.full((3, 8), -5.0, np.float32)
    for t, (e0, e1) in enumerate([(0, 1), (2, 3), (4, 5)]):
        logits[t, e0] = 3.0
        logits[t, e1] = 2.0
    xt = torch.from_numpy(x).cuda()
    lt = torch.from_numpy(logits).cuda()
    ids, wts = q8().route_device(ctx, lt, 2)
    rows = xt.repeat_interleave(2, dim=0)
    eids = ids.reshape(-1).contiguous()
    out1 = layer.expert_rows_device(rows, eids, 1)
    out2 = layer.expert_rows_device(rows, eids, 2)
    ctx.sync()
    assert bits_equal(out1.cpu().numpy(), out2.cpu().numpy())


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("T,skew", [(24, False), (64, False), (64, True)])
def test_decode_batch_groups(ctx, mode, T, skew):
    """Up to 64 tokens every routed group runs on the warp-level kernel as
    8-row chunks listed by the pair grouping, gate and up in one launch: groups
    of several chunks, single-row groups and empty experts; with `skew` every
    token picks expert 3 (one 64-row group of eight chunks)."""
    rng = np.random.default_rng(1100 + 10 * T + mode + (5 if skew else 0))
    layer, sh, ex = make_layer(ctx, rng, 256, 128, 256, 8, 2)
    x = rng.standard_normal((T, 256)).astype(np.float32)
    logits = rng.standard_normal((T, 8)).astype(np.float32)
    logits[:, 6] -= 6.0  # expert 6 nearly empty
    if skew:
        logits[:, 3] += 8.0
    y, ids, wts = layer.forward(x, logits, mode)
    ref, ids_ref, wts_ref = oracle.experts(sh, ex, logits, x, 2, mode)
    _check_layer(y, ref, ids, ids_ref, wts, wts_ref, mode == 2)


@pytest.mark.parametrize("T", [2, 65, 150])
def test_prefill_tensor_core_int8(ctx, T):
    """Int8 activations for every row on shapes the tensor-core path takes
    (every dimension a multiple of 128): gathered rows per expert, grouped
    projections, ragged groups and tiles."""
    rng = np.random.default_rng(900 + T)
    layer, sh, ex = make_layer(ctx, rng, 256, 128, 256, 8, 2)
    x = rng.standard_normal((T, 256)).astype(np.float32)
    logits = rng.standard_normal((T, 8)).astype(np.float32)
    logits[:, 5] += 1.5  # one popular expert: a group of several tiles
    y, ids, wts = layer.forward(x, logits, 2)
    ref, ids_ref, wts_ref = oracle.experts(sh, ex, logits, x, 2, 2)
    _check_layer(y, ref, ids, ids_ref, wts, wts_ref, True)


@pytest.mark.slow
@pytest.mark.parametrize("mode", [0, 2])
def test_prefill_config2_shape(ctx, config1, mode):
    """Config-2 shapes with Zipf-skewed routing, 192 tokens (oracle-sized)."""
    layer, sh, ex = config1
    rng = np.random.default_rng(77)
    T = 192
    x = rng.standard_normal((T, 1280)).astype(np.float32)
    bias = (1.0 / np.arange(1, 65) ** 1.1).astype(np.float32) * 4.0
    logits = (rng.standard_normal((T, 64)).astype(np.float32) + rng.permutation(bias)).astype(np.float32)
    y, ids, wts = layer.forward(x, logits, mode)
    ref, ids_ref, wts_ref = oracle.experts(sh, ex, logits, x, 6, mode)
    _check_layer(y, ref, ids, ids_ref, wts, wts_ref, mode != 0)


def zipf_logits(rng, tokens, experts, s=1.1):
    """Router logits of a prefill with skewed expert popularity: N(0, 1) noise
    plus a Zipf(s) bias, -s * log(rank), over a random order of the experts."""
    bias = np.empty(experts, np.float32)
    bias[rng.permutation(experts)] = -s * np.log(np.arange(1, experts + 1, dtype=np.float64))
    return (rng.standard_normal((tokens, experts)) + bias).astype(np.float32)


@pytest.mark.slow
@pytest.mark.parametrize("mode", [0, 2])
def test_prefill_config2_full(ctx, config1, mode):
    """The grouped prefill at its full size: 1024 tokens, top-6 of 64 experts
    with Zipf(1.1)-skewed routing (groups from a few rows to several hundred:
    warp-level chunks and tensor-core tiles in one layer), FP32 activations
    and int8 activations for every row."""
    layer, sh, ex = config1
    rng = np.random.default_rng(2024)
    T = 1024
    x = rng.standard_normal((T, 1280)).astype(np.float32)
    logits = zipf_logits(rng, T, 64)
    y, ids, wts = layer.forward(x, logits, mode)
    ref, ids_ref, wts_ref = oracle.experts(sh, ex, logits, x, 6, mode)
    sizes = np.bincount(ids_ref.reshape(-1), minlength=64)
    assert sizes.max() > 256 and sizes.min() < 64, sizes  # both kernels reached
    _check_layer(y, ref, ids, ids_ref, wts, wts_ref, mode != 0)


# ------------------------------------------------- the layer in parts (expert parallelism)
def _parts_forward(ctx, layer, x_t, lg_t, mode, top_k, per_source=None):
    """uocr_moe_forward rebuilt from route, expert_rows, shared_rows and
    combine on one GPU; `per_source` splits the routed rows into that many
    consecutive calls (the grouping a multi-GPU dispatch produces)."""
    import torch
    q = q8()
    ids, wts = q.route_device(ctx, lg_t, top_k)
    T = x_t.shape[0]
    rows = x_t.repeat_interleave(top_k, dim=0)
    eids = ids.reshape(-1).contiguous()
    out = torch.empty_like(rows)
    cuts = [0, T * top_k] if not per_source else \
        [round(i * T * top_k / per_source) for i in range(per_source + 1)]
    for a, b in zip(cuts[:-1], cuts[1:]):
        if b > a:
            layer.expert_rows_device(rows[a:b], eids[a:b], mode, out[a:b])
    y = layer.shared_rows_device(x_t, mode)
    q.combine_device(ctx, ids, wts, out, y)
    return y, ids, wts


@pytest.mark.parametrize("mode", [0, 2])
@pytest.mark.parametrize("shape", [(128, 64, 128, 8, 3), (256, 128, 256, 8, 2)])
def test_parts_equal_forward(ctx, mode, shape):
    """route + expert_rows + shared_rows + combine == uocr_moe_forward, bit for
    bit in one call; split over three calls (as a multi-GPU dispatch), bit for
    bit with int8 activations and within the FP32 tolerance otherwise."""
    import torch
    H, F, FS, E, k = shape
    rng = np.random.default_rng(300 + mode + H)
    layer, sh, ex = make_layer(ctx, rng, H, F, FS, E, k)
    x = torch.from_numpy(rng.standard_normal((41, H)).astype(np.float32)).cuda()
    lg = torch.from_numpy(rng.standard_normal((41, E)).astype(np.float32)).cuda()
    y1 = layer.forward_device(x, lg, mode)
    y2, _, _ = _parts_forward(ctx, layer, x, lg, mode, k, per_source=3)
    y3, _, _ = _parts_forward(ctx, layer, x, lg, mode, k)
    ctx.sync()
    y1, y2, y3 = y1.cpu().numpy(), y2.cpu().numpy(), y3.cpu().numpy()
    assert bits_equal(y1, y3)
    if mode == 2:
        assert bits_equal(y1, y2)
    else:  # the split changes group sizes, hence kernels and FP32 order
        assert float(np.max(np.abs(y1.astype(np.float64) - y2))) <= 1e-4 * float(np.max(np.abs(y1)))


def test_parts_dynamic_groups_per_source(ctx):
    """DynamicActivations picks int8 for a one-row group: the parts reproduce
    the single-device layer when each source's rows are one call."""
    import torch
    rng = np.random.default_rng(311)
    layer, sh, ex = make_layer(ctx, rng, 128, 64, 128, 8, 3)
    x = rng.standard_normal((2, 128)).astype(np.float32)
    lg = rng.standard_normal((2, 8)).astype(np.float32)
    y1, _, _ = layer.forward(x, lg, 1)
    y2, _, _ = _parts_forward(ctx, layer, torch.from_numpy(x).cuda(), torch.from_numpy(lg).cuda(),
                              1, 3)
    ctx.sync()
    assert bits_equal(y1, y2.cpu().numpy())


def test_parts_errors(ctx):
    import torch
    q = q8()
    rng = np.random.default_rng(312)
    layer, _, _ = make_layer(ctx, rng, 128, 64, 128, 4, 2)
    x = torch.zeros((3, 128), device="cuda")
    bad = torch.tensor([0, 4, 1], dtype=torch.int32, device="cuda")
    layer.expert_rows_device(x, bad, 0)
    with pytest.raises(q.OcrError) as e:
        ctx.sync()
    assert e.value.kind == "Shape"
    ids = torch.zeros((3, 9), dtype=torch.int32, device="cuda")
    with pytest.raises(q.OcrError) as e:
        q.combine_device(ctx, ids, ids.float(), torch.zeros((27, 128), device="cuda"), x)
    assert e.value.kind == "Unsupported"
    # empty inputs are no-ops
    layer.expert_rows_device(x[:0], bad[:0], 2)
    layer.shared_rows_device(x[:0], 2)
    ctx.sync()
