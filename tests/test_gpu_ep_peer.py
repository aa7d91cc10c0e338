"""Expert parallelism over NVLink peer memory (uocr_ep_*, PeerExpertParallel).

No counterpart in the reference, which runs Decoder::experts
(src/decoder/mod.rs:124-220) on one device.  The routed experts of a layer
are split over the ranks in contiguous blocks and rows move as stores into
the other ranks' memory.  Each rank's result must equal the single-GPU layer
(uocr_moe_forward over all experts, which the MoE parity tests tie to the
oracle) on that rank's tokens over consecutive steps (the step numbers that
pair each dispatch with its wait advance): routing bit for bit, outputs bit
for bit in the int8-activation modes and within the FP32 layer tolerance
(max |y - ref| <= 1e-4 * max |ref|) with FP32 activations, where an owner's
group (rows from several ranks) can take another projection kernel, with
another FP32 summation order, than the same rows on one GPU.

Several ranks are emulated on one GPU: one process, one context and so one
stream, the ranks driven through the three-part API in the order
dispatch(all ranks), experts(all ranks), combine(all ranks), so that every
bounded wait finds what it waits for already written (no kernel waits on
work queued behind it).  Two real GPUs (CUDA IPC mappings) are covered by the
last test when the box has them.
"""
import os
import socket

import numpy as np
import pytest

from helpers import random_q8

pytestmark = pytest.mark.gpu

H, F, FS, E, K = 1280, 896, 1792, 64, 6


def q8():
    import uocr_q8
    return uocr_q8


def bounds_of(n, world):
    from uocr_q8.expert_parallel import expert_bounds
    return expert_bounds(n, world)


def build(ctx, seed, H=H, F=F, FS=FS, E=E, k=K):
    rng = np.random.default_rng(seed)
    M = q8().Int8Matrix

    def ffn(width):
        return [M.from_parts(r, c, *random_q8(rng, r, c), ctx=ctx)
                for r, c in ((width, H), (width, H), (H, width))]

    shared = ffn(FS)
    experts = [ffn(F) for _ in range(E)]
    return shared, experts, q8().MoeLayer(ctx, shared, experts, k)


@pytest.fixture(scope="module")
def layer4(ctx):
    """The MoE layer shapes of the 12-layer decoder: hidden 1280, 64 experts of
    width 896, top-6, a fused shared expert of width 1792."""
    return build(ctx, 41)


def make_ranks(ctx, shared, experts, world, max_tokens, n=E, k=K):
    b = bounds_of(n, world)
    locs = [q8().MoeLayer(ctx, shared, experts[b[r]:b[r + 1]], 1) for r in range(world)]
    eps = [q8().PeerExpertParallel(ctx, locs[r], n, k, b, r, max_tokens) for r in range(world)]
    q8().PeerExpertParallel.connect_local(eps)
    return eps, locs


def emulated_step(ctx, eps, xs, lgs, mode):
    import torch
    ys = [torch.empty_like(x) for x in xs]
    ids = [torch.empty((x.shape[0], eps[0].top_k), dtype=torch.int32, device="cuda") for x in xs]
    wts = [torch.empty((x.shape[0], eps[0].top_k), dtype=torch.float32, device="cuda") for x in xs]
    for ep, x, lg, y in zip(eps, xs, lgs, ys):
        ep.dispatch_device(x, lg, mode, y)
    for ep in eps:
        ep.experts_device()
    for ep, y, i, w in zip(eps, ys, ids, wts):
        ep.combine_device(y, i, w)
    ctx.sync()
    return ys, ids, wts


def reference(ctx, full, x, lg, mode):
    import torch
    t = x.shape[0]
    y = torch.empty_like(x)
    i = torch.empty((t, full.top_k), dtype=torch.int32, device="cuda")
    w = torch.empty((t, full.top_k), dtype=torch.float32, device="cuda")
    if t:
        full.forward_device(x, lg, mode, y, i, w)
    ctx.sync()
    return y, i, w


def assert_same(got, ref, exact=True):
    """(y, ids, weights) against the single-GPU layer: routing identical;
    outputs identical, or (exact=False, FP32 activations) within the FP32
    layer tolerance, max |y - ref| <= 1e-4 * max |ref|, with the fraction of
    bit-identical outputs printed."""
    for n, (a, b) in enumerate(zip(got, ref)):
        a, b = a.cpu().numpy(), b.cpu().numpy()
        assert a.shape == b.shape
        if exact or n > 0:
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        elif a.size:
            err = float(np.max(np.abs(a.astype(np.float64) - b)))
            same = float(np.mean(a.view(np.uint32) == b.view(np.uint32)))
            print(f"fp32 outputs: {same:.4f} bit-identical, max |diff| / max |ref| = "
                  f"{err / float(np.max(np.abs(b))):.2e}")
            assert err <= 1e-4 * float(np.max(np.abs(b)))


def inputs(rng, tokens, n=E, hidden=H, bias=None):
    import torch
    xs, lgs = [], []
    for t in tokens:
        x = rng.standard_normal((t, hidden)).astype(np.float32)
        lg = rng.standard_normal((t, n)).astype(np.float32)
        if bias is not None:
            lg = lg + bias
        xs.append(torch.from_numpy(x).cuda())
        lgs.append(torch.from_numpy(lg).cuda())
    return xs, lgs


@pytest.mark.parametrize("tokens", [[64], [64, 17], [64, 0, 1, 33],
                                    [64, 64, 0, 5, 64, 1, 12, 64]],
                         ids=["w1", "w2", "w4", "w8"])
def test_emulated_ranks_match_single_gpu(ctx, layer4, tokens):
    shared, experts, full = layer4
    eps, locs = make_ranks(ctx, shared, experts, len(tokens), 64)
    rng = np.random.default_rng(len(tokens))
    for mode in (0, 1, 2, 0):  # four consecutive steps
        xs, lgs = inputs(rng, tokens)
        got = emulated_step(ctx, eps, xs, lgs, mode)
        for r in range(len(tokens)):
            ref = reference(ctx, full, xs[r], lgs[r], mode)
            assert_same([g[r] for g in got], ref, exact=mode != 0)
    for ep in eps:
        ep.free()


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_emulated_skewed_routing(ctx, layer4, mode):
    """Every rank routes to the experts of rank 2 only: one owner receives all
    pairs (groups of up to 256 rows take the tensor-core GEMMs)."""
    shared, experts, full = layer4
    world = 4
    eps, locs = make_ranks(ctx, shared, experts, world, 64)
    bias = np.zeros(E, np.float32)
    b = bounds_of(E, world)
    bias[b[2]:b[3]] = 30.0
    rng = np.random.default_rng(77 + mode)
    xs, lgs = inputs(rng, [64, 64, 64, 64], bias=bias)
    got = emulated_step(ctx, eps, xs, lgs, mode)
    for r in range(world):
        assert_same([g[r] for g in got], reference(ctx, full, xs[r], lgs[r], mode),
                    exact=mode != 0)
    for ep in eps:
        ep.free()


def test_forward_single_rank_and_graph(ctx, layer4):
    """uocr_ep_forward (the exchange on its own high-priority stream, joined
    back) at world 1, eagerly and replayed from a CUDA graph."""
    import torch
    shared, experts, full = layer4
    eps, locs = make_ranks(ctx, shared, experts, 1, 64)
    ep = eps[0]
    rng = np.random.default_rng(5)
    xs, lgs = inputs(rng, [64, 64, 64])
    for mode in (0, 2):
        y = torch.empty_like(xs[0])
        ep.forward_device(xs[0], lgs[0], mode, y)
        ctx.sync()
        assert_same([y], [reference(ctx, full, xs[0], lgs[0], mode)[0]], exact=mode != 0)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    ctx.set_stream(side)
    outs = [torch.empty_like(x) for x in xs]
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for x, lg, y in zip(xs, lgs, outs):
            ep.forward_device(x, lg, 0, y)
    ctx.set_stream(torch.cuda.current_stream())
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    ctx.sync()
    for x, lg, y in zip(xs, lgs, outs):
        assert_same([y], [reference(ctx, full, x, lg, 0)[0]], exact=False)
    del g
    ep.free()


@pytest.mark.parametrize("mode", [0, 2])
def test_forward_host_matches_device(ctx, layer4, mode):
    """uocr_ep_forward_host at world 1, several calls in a row (different tokens
    each time, pinned buffers copied directly or ordinary ones through the
    staging mirror, two token counts): every call equals the device-buffer
    forward on the same tokens, bit for bit."""
    import torch
    shared, experts, full = layer4
    eps, locs = make_ranks(ctx, shared, experts, 1, 64)
    ep = eps[0]
    rng = np.random.default_rng(9 + mode)
    for tokens, pinned in ((64, True), (64, True), (64, False), (64, True), (17, False), (17, True),
                           (17, True)):
        x = rng.standard_normal((tokens, 1280)).astype(np.float32)
        lg = rng.standard_normal((tokens, 64)).astype(np.float32)
        if pinned:
            xh = torch.from_numpy(x).pin_memory()
            lh = torch.from_numpy(lg).pin_memory()
            yh = torch.empty_like(xh).pin_memory()
            ep.forward_host_ptrs(xh.data_ptr(), lh.data_ptr(), tokens, yh.data_ptr(), mode)
            y = yh.numpy()
        else:
            y = ep.forward(x, lg, mode)
        ref = torch.empty((tokens, 1280), device="cuda")
        ep.forward_device(torch.from_numpy(x).cuda(), torch.from_numpy(lg).cuda(), mode, ref)
        ctx.sync()
        assert np.array_equal(y.view(np.uint32), ref.cpu().numpy().view(np.uint32)), (tokens, pinned)
    ep.free()


def test_timeout_when_a_rank_never_dispatches(ctx):
    """A bounded wait that expires: rank 1 never dispatches, so rank 0's
    wait for its rows gives up after the limit and the next synchronising
    call reports Timeout (no GPU fault; the context stays usable)."""
    import torch
    shared, experts, full = build(ctx, 9, H=256, F=128, FS=256, E=8, k=2)
    eps, locs = make_ranks(ctx, shared, experts, 2, 8, n=8, k=2)
    eps[0].set_wait_limit(0.05)
    rng = np.random.default_rng(3)
    xs, lgs = inputs(rng, [8], n=8, hidden=256)
    y = torch.empty_like(xs[0])
    eps[0].dispatch_device(xs[0], lgs[0], 0, y)
    eps[0].experts_device()
    with pytest.raises(q8().OcrError) as e:
        ctx.sync()
    assert e.value.kind == "Timeout"
    for ep in eps:
        ep.free()
    # the context still works
    ref = reference(ctx, full, xs[0], lgs[0], 0)
    assert np.all(np.isfinite(ref[0].cpu().numpy()))


def test_rejections(ctx):
    import torch
    shared, experts, full = build(ctx, 10, H=256, F=128, FS=256, E=8, k=2)
    b = bounds_of(8, 2)
    loc = q8().MoeLayer(ctx, shared, experts[b[0]:b[1]], 1)
    with pytest.raises(q8().OcrError) as e:  # bounds do not cover the experts
        q8().PeerExpertParallel(ctx, loc, 8, 2, [0, 4, 7], 0, 8)
    assert e.value.kind == "Shape"
    with pytest.raises(q8().OcrError) as e:  # local layer is not rank 1's block size
        q8().PeerExpertParallel(ctx, loc, 8, 2, [0, 2, 8], 1, 8)
    assert e.value.kind == "Shape"
    ep = q8().PeerExpertParallel(ctx, loc, 8, 2, b, 0, 8)
    x = torch.zeros((4, 256), device="cuda")
    lg = torch.zeros((4, 8), device="cuda")
    with pytest.raises(q8().OcrError) as e:  # not connected
        ep.forward_device(x, lg, 0)
    assert e.value.kind == "Invalid"
    other = q8().PeerExpertParallel(ctx, loc, 8, 2, b, 0, 8)
    with pytest.raises(q8().OcrError) as e:  # two rank-0 ends
        q8().PeerExpertParallel.connect_local([ep, other])
    assert e.value.kind == "Shape"
    solo_b = [0, 8]
    full_loc = q8().MoeLayer(ctx, shared, experts, 1)
    solo = q8().PeerExpertParallel(ctx, full_loc, 8, 2, solo_b, 0, 8)
    q8().PeerExpertParallel.connect_local([solo])
    big = torch.zeros((9, 256), device="cuda")
    with pytest.raises(q8().OcrError) as e:
        solo.forward_device(big, torch.zeros((9, 8), device="cuda"), 0)
    assert e.value.kind == "Resource"
    with pytest.raises(q8().OcrError) as e:
        solo.connect([solo.handle()])
    assert e.value.kind == "Invalid"
    for p in (ep, other, solo):
        p.free()


# ---------------------------------------------------------------- two GPUs
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_rank(rank, world, port, result_dir):
    import datetime
    import sys

    import torch
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "unlimited-ocr-kernel_b200"), os.path.join(root, "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import uocr_q8
    from uocr_q8.expert_parallel import peer_expert_parallel
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    ctx = uocr_q8.GpuContext(rank)
    shared, experts, full = build(ctx, 41)
    b = bounds_of(E, world)
    loc = uocr_q8.MoeLayer(ctx, shared, experts[b[rank]:b[rank + 1]], 1)
    ep = peer_expert_parallel(ctx, loc, E, K, 64)
    rng = np.random.default_rng(100 + rank)
    ok = True
    dist.barrier()
    for step, mode in enumerate((0, 1, 2, 0)):
        t = [64, 23][rank] if step != 3 else [0, 64][rank]
        x = torch.from_numpy(rng.standard_normal((t, H)).astype(np.float32)).cuda()
        lg = torch.from_numpy(rng.standard_normal((t, E)).astype(np.float32)).cuda()
        y = torch.empty_like(x)
        ep.forward_device(x, lg, mode, y)
        ctx.sync()
        ref = reference(ctx, full, x, lg, mode)[0].cpu().numpy()
        got = y.cpu().numpy()
        if mode != 0:
            ok = ok and np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        elif t:
            ok = ok and float(np.max(np.abs(got.astype(np.float64) - ref))) <= \
                1e-4 * float(np.max(np.abs(ref)))
    dist.barrier()
    ep.free()
    with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
        f.write("ok" if ok else "mismatch")
    dist.destroy_process_group()


def test_two_gpus_ipc(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_two_gpu_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert (tmp_path / f"rank{r}").read_text() == "ok"
