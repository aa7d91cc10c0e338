"""Failure detection on the GPU without a GPU fault.

The one-token decode kernel synchronises its CTAs with a bounded grid barrier.
A host-side hook (uocr_ctx_hold_decode_barrier) makes the barrier wait for one
arrival more than the grid makes; with a short wait limit
(uocr_ctx_set_wait_limit) every CTA gives up, the launch returns, and the next
synchronising call reports Timeout.  Nothing traps or faults: the context stays
usable, and once the hold is released the barrier's words are valid again, so
the next launch is bit-identical to the one before the fault.  (The
expert-parallel waits are driven to expiry in test_gpu_ep_peer.py.)
"""
import numpy as np
import pytest

from helpers import random_q8

pytestmark = pytest.mark.gpu


def test_decode_barrier_timeout_and_recovery():
    import torch

    import uocr_q8
    ctx = uocr_q8.GpuContext(0)
    rng = np.random.default_rng(21)
    M = uocr_q8.Int8Matrix

    def ffn(width):
        return [M.from_parts(r, c, *random_q8(rng, r, c), ctx=ctx)
                for r, c in ((width, 1280), (width, 1280), (1280, width))]

    layer = uocr_q8.MoeLayer(ctx, ffn(1792), [ffn(896) for _ in range(16)], 6)
    x = torch.from_numpy(rng.standard_normal((1, 1280)).astype(np.float32)).cuda()
    lg = torch.from_numpy(rng.standard_normal((1, 16)).astype(np.float32)).cuda()
    torch.cuda.synchronize()
    for mode in (0, 1):
        before = layer.forward_device(x, lg, mode)
        ctx.sync()
        ctx.set_wait_limit(0.002)
        ctx.hold_decode_barrier(True)
        layer.forward_device(x, lg, mode)
        with pytest.raises(uocr_q8.OcrError) as e:
            ctx.sync()
        assert e.value.kind == "Timeout"
        ctx.hold_decode_barrier(False)
        ctx.set_wait_limit(0)
        after = layer.forward_device(x, lg, mode)
        ctx.sync()
        assert np.array_equal(before.cpu().numpy().view(np.uint32),
                              after.cpu().numpy().view(np.uint32))
    layer.free()
    ctx.close()
