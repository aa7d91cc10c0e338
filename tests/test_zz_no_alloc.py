"""GPU test of the allocation-free decode entry point.

uocr_moe_forward_decode_noalloc exists for callers that may not allocate
device memory once inference is running — serving loops that reserve every
buffer at start-up because a late cudaMalloc can stall the device, and hosts
whose own pool allocator must own all device memory.  It keeps its scratch in
a fixed array inside the library instead of the context's growable workspace.

The test calls it through the C ABI on a fresh context: once for the per-device
set-up, then twice in a row (two different tokens, so the second call reuses
the scratch the first one left behind), checks that the device's free memory
did not change across the two calls, and compares
each output with the regular entry point, uocr_moe_forward, on the same token
(on a second context), in all three modes.  The tolerance is the MoE layer
tolerance of the other parity tests
(max |y - ref| <= 1e-4 * max |ref|); the two paths run the same kernels, so the
outputs are expected to be bit-identical as well.  This file is named so that
pytest collects it last, and it builds everything it needs itself, so it passes
alone in a fresh process as well as after the other tests.
"""
import numpy as np
import pytest

from helpers import random_q8

pytestmark = pytest.mark.gpu

LAYER_TOL = 1e-4


def _layer(ctx, rng, H, F, FS, E, k):
    import uocr_q8
    M = uocr_q8.Int8Matrix

    def ffn(width):
        return [M.from_parts(r, c, *random_q8(rng, r, c), ctx=ctx)
                for r, c in ((width, H), (width, H), (H, width))]

    return uocr_q8.MoeLayer(ctx, ffn(FS), [ffn(F) for _ in range(E)], k)


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_noalloc_matches_regular_entry_point(mode):
    import torch

    import uocr_q8
    rng = np.random.default_rng(2024 + mode)
    # two fresh contexts: the no-allocation calls run first on one that has
    # never grown a workspace, the regular calls on the other
    ctx = uocr_q8.GpuContext(0)
    ref_ctx = uocr_q8.GpuContext(0)
    layer = _layer(ctx, rng, 1280, 896, 1792, 16, 6)
    ref_layer = uocr_q8.MoeLayer(ref_ctx, *layer._keep, 6)
    tokens = [(torch.from_numpy(rng.standard_normal((1, 1280)).astype(np.float32)).cuda(),
               torch.from_numpy(rng.standard_normal((1, 16)).astype(np.float32)).cuda())
              for _ in range(2)]
    refs = [torch.empty_like(x) for x, _ in tokens]
    outs = [torch.empty_like(x) for x, _ in tokens]
    # the library runs on the context's own stream: synchronise it before
    # torch touches the outputs on its stream
    torch.cuda.synchronize()
    # the first call on a device is the set-up: it looks up the scratch
    # array, which may load the library's device code (and with it the array)
    layer.forward_decode_noalloc(tokens[0][0], tokens[0][1], mode, y_t=outs[1])
    ctx.sync()
    free_before = torch.cuda.mem_get_info(0)[0]
    for (x, lg), y in zip(tokens, outs):  # two calls in a row
        layer.forward_decode_noalloc(x, lg, mode, y_t=y)
    ctx.sync()
    assert torch.cuda.mem_get_info(0)[0] == free_before  # nothing was allocated
    for (x, lg), y in zip(tokens, refs):
        ref_layer.forward_device(x, lg, mode, y_t=y)
    ref_ctx.sync()
    for y, ref in zip(outs, refs):
        y, ref = y.cpu().numpy(), ref.cpu().numpy()
        scale = float(np.max(np.abs(ref)))
        assert float(np.max(np.abs(y.astype(np.float64) - ref))) <= LAYER_TOL * scale
        assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))
    ref_layer.free()
    layer.free()
    ref_ctx.close()
    ctx.close()


def test_noalloc_rejects_layers_beyond_its_scratch(ctx):
    import torch

    import uocr_q8
    rng = np.random.default_rng(7)
    layer = _layer(ctx, rng, 128, 8192, 8192, 2, 2)  # h needs 8192 + 2*8192 floats
    x = torch.zeros((1, 128), device="cuda")
    lg = torch.zeros((1, 2), device="cuda")
    with pytest.raises(uocr_q8.OcrError) as e:
        layer.forward_decode_noalloc(x, lg, 0)
    assert e.value.kind == "Resource"
