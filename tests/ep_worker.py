"""Rank bodies for the expert-parallel tests (spawned processes).

CPU ranks use gloo and an oracle backend; GPU ranks use NCCL and the CUDA
library.  Either way each rank checks its own output against the oracle's
Decoder::experts of its tokens (src/decoder/mod.rs:124-220).
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "unlimited-ocr-kernel_b200"), os.path.dirname(__file__)):
    if p not in sys.path:
        sys.path.insert(0, p)

import oracle  # noqa: E402
from helpers import random_q8  # noqa: E402


def make_layer(seed, hidden, width, shared_width, n_experts):
    """Random q8 shared FFN and routed FFNs as oracle matrices."""
    rng = np.random.default_rng(seed)

    def ffn(f):
        g = oracle.Matrix(*random_q8(rng, f, hidden))
        u = oracle.Matrix(*random_q8(rng, f, hidden))
        d = oracle.Matrix(*random_q8(rng, hidden, f))
        return oracle.Ffn(g, u, d)

    return ffn(shared_width), [ffn(width) for _ in range(n_experts)]


def rank_inputs(seed, rank, tokens, hidden, n_experts):
    rng = np.random.default_rng(seed * 101 + rank)
    x = (rng.standard_normal((tokens, hidden)) * rng.uniform(0.2, 4, (tokens, 1))).astype(np.float32)
    logits = (rng.standard_normal((tokens, n_experts)) * 2).astype(np.float32)
    return x, logits


class OracleBackend:
    """The CPU oracle behind ExpertParallelMoe (test-only checker)."""

    def __init__(self, shared, local_experts, top_k, normalize, scale):
        self.shared = shared
        self.local = local_experts
        self.top_k = top_k
        self.normalize = normalize
        self.scale = scale

    def route(self, logits):
        import torch
        lg = logits.numpy()
        ids = np.empty((lg.shape[0], self.top_k), np.int32)
        wts = np.empty((lg.shape[0], self.top_k), np.float32)
        for t in range(lg.shape[0]):
            sel = oracle.route(lg[t], self.top_k, self.normalize, self.scale)
            ids[t] = [i for i, _ in sel]
            wts[t] = [w for _, w in sel]
        return torch.from_numpy(ids), torch.from_numpy(wts)

    def expert_rows(self, x, local_ids, mode, out):
        import torch
        xn, ids = x.numpy(), local_ids.numpy()
        for e in np.unique(ids[ids >= 0]):  # negative: unused slot
            rows = np.nonzero(ids == e)[0]
            out[torch.from_numpy(rows)] = torch.from_numpy(
                oracle.feed_forward(self.local[int(e)], xn[rows], mode))

    def shared_rows(self, x, mode):
        import torch
        if x.shape[0] == 0:
            return x.clone()
        return torch.from_numpy(oracle.feed_forward(self.shared, x.numpy(), mode))

    def combine(self, ids, wts, pair_out, y):
        k = ids.shape[1]
        idn, wn, po, yn = ids.numpy(), wts.numpy(), pair_out.numpy(), y.numpy()
        for t in range(idn.shape[0]):
            for j in np.argsort(idn[t], kind="stable"):
                yn[t] = yn[t] + np.float32(wn[t, j]) * po[t * k + j]

    def dispatch(self, x, ids, bounds, capacity):
        """uocr_moe_dispatch restated: slot = earlier pairs for the same rank."""
        import torch
        world = len(bounds) - 1
        xn, idn = x.numpy(), ids.numpy().reshape(-1)
        k = ids.shape[1]
        send_x = np.zeros((world * capacity, xn.shape[1]), np.float32)
        send_ids = np.full((world * capacity,), -1, np.int32)
        pair_rows = np.empty((idn.size,), np.int32)
        used = [0] * world
        for i, e in enumerate(idn):
            r = next(r for r in range(world) if bounds[r] <= e < bounds[r + 1])
            slot = used[r]
            used[r] += 1
            assert slot < capacity
            send_x[r * capacity + slot] = xn[i // k]
            send_ids[r * capacity + slot] = e - bounds[r]
            pair_rows[i] = r * capacity + slot
        return torch.from_numpy(send_x), torch.from_numpy(send_ids), torch.from_numpy(pair_rows)

    def combine_rows(self, ids, wts, rows, pair_rows, y):
        import torch
        self.combine(ids, wts, rows[torch.from_numpy(pair_rows.numpy().astype(np.int64))], y)


def _init(rank, world, port, backend):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=60))


def cpu_rank(rank, world, port, case):
    """gloo rank: ExpertParallelMoe over the oracle backend vs oracle.experts."""
    import torch
    import torch.distributed as dist
    from uocr_q8.expert_parallel import ExpertParallelMoe, expert_bounds
    _init(rank, world, port, "gloo")
    try:
        H, F, FS, E, k = case["hidden"], case["width"], case["shared_width"], case["experts"], case["top_k"]
        shared, experts = make_layer(case["seed"], H, F, FS, E)
        b = expert_bounds(E, world)
        be = OracleBackend(shared, experts[b[rank]:b[rank + 1]], k, case["normalize"], case["scale"])
        cap = case.get("capacity")
        ep = ExpertParallelMoe(be, E, k, H, capacity=cap)
        x, logits = rank_inputs(case["seed"], rank, case["tokens"][rank], H, E)
        for mode in case["modes"]:
            y, ids, wts = ep.forward(torch.from_numpy(x), torch.from_numpy(logits), mode)
            if x.shape[0] == 0:
                assert y.shape == (0, H)
                continue
            ry, rids, rw = oracle.experts(shared, experts, logits, x, k, mode, case["normalize"],
                                          case["scale"])
            assert np.array_equal(ids.numpy(), rids), (rank, mode)
            assert np.array_equal(wts.numpy().view(np.uint32), rw.view(np.uint32)), (rank, mode)
            assert np.array_equal(y.numpy().view(np.uint32), ry.view(np.uint32)), (rank, mode)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def cpu_rank_leaves(rank, world, port, case):
    """gloo ranks: both run one step, then the last rank leaves (returns
    between steps, none of its collectives in flight); the others' next step
    must fail with OcrError "Nccl" within the process group's timeout instead
    of waiting for ever.  Each rank writes its outcome to case["out"]."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from uocr_q8 import OcrError
    from uocr_q8.expert_parallel import ExpertParallelMoe, expert_bounds
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    H, F, FS, E, k = case["hidden"], case["width"], case["shared_width"], case["experts"], case["top_k"]
    shared, experts = make_layer(case["seed"], H, F, FS, E)
    b = expert_bounds(E, world)
    be = OracleBackend(shared, experts[b[rank]:b[rank + 1]], k, False, 1.0)
    ep = ExpertParallelMoe(be, E, k, H, capacity=case.get("capacity"))
    x, logits = rank_inputs(case["seed"], rank, 4, H, E)
    ep.forward(torch.from_numpy(x), torch.from_numpy(logits), 0)
    outcome = "left"
    if rank != world - 1:
        try:
            ep.forward(torch.from_numpy(x), torch.from_numpy(logits), 0)
            outcome = "no error"
        except OcrError as exc:
            outcome = exc.kind
    with open(os.path.join(case["out"], f"rank{rank}"), "w") as f:
        f.write(outcome)
    if rank == world - 1:
        os._exit(0)  # leave without a goodbye: the others learn it from the transport


def gpu_rank(rank, world, port, case):
    """NCCL rank: ExpertParallelMoe over the CUDA library, each rank on its own
    GPU.  Its output must equal the single-GPU layer's (uocr_moe_forward over
    all experts on this rank's tokens) bit for bit with int8 activations and
    within the FP32 tolerance with FP32 activations, and the oracle's within
    the MoE layer tolerances of the single-GPU tests."""
    import torch
    import torch.distributed as dist
    import uocr_q8
    from uocr_q8.expert_parallel import ExpertParallelMoe, LibraryBackend, expert_bounds, local_layer
    from helpers import bits_equal
    torch.cuda.set_device(rank)
    _init(rank, world, port, "nccl")
    try:
        H, F, FS, E, k = case["hidden"], case["width"], case["shared_width"], case["experts"], case["top_k"]
        norm, scale = case["normalize"], case["scale"]
        shared, experts = make_layer(case["seed"], H, F, FS, E)
        ctx = uocr_q8.GpuContext(rank)
        dev = lambda m: uocr_q8.Int8Matrix.from_parts(m.rows, m.cols, m.w, m.s, ctx)
        sh = [dev(shared.gate), dev(shared.up), dev(shared.down)]
        ex = [[dev(f.gate), dev(f.up), dev(f.down)] for f in experts]
        b = expert_bounds(E, world)
        layer = local_layer(ctx, sh, ex, b, rank)
        full = uocr_q8.MoeLayer(ctx, sh, ex, k, norm, scale)
        be = LibraryBackend(ctx, layer, E, k, norm, scale)
        ep = ExpertParallelMoe(be, E, k, H, capacity=case.get("capacity"))
        x, logits = rank_inputs(case["seed"], rank, case["tokens"][rank], H, E)
        xt = torch.from_numpy(x).cuda()
        lt = torch.from_numpy(logits).cuda()
        for mode in case["modes"]:
            y, ids, wts = ep.forward(xt, lt, mode)
            y1 = full.forward_device(xt, lt, mode)
            torch.cuda.synchronize()
            ctx.sync()
            y, ids, wts, y1 = y.cpu().numpy(), ids.cpu().numpy(), wts.cpu().numpy(), y1.cpu().numpy()
            if mode == 0:
                # FP32 activations: an expert's kernel depends on its group's
                # size, which differs between the owner's groups (rows of all
                # ranks) and the single-GPU ones, so the FP32 order may too
                scale0 = float(np.max(np.abs(y1)))
                assert float(np.max(np.abs(y.astype(np.float64) - y1))) <= 1e-4 * scale0, rank
            else:
                assert bits_equal(y, y1), (rank, mode)
            ry, rids, rw = oracle.experts(shared, experts, logits, x, k, mode, norm, scale)
            assert np.array_equal(ids, rids), (rank, mode)
            d = np.abs(wts.view(np.int32).astype(np.int64) - rw.view(np.int32).astype(np.int64))
            assert d.max() <= 1, (rank, mode)
            err = float(np.max(np.abs(y.astype(np.float64) - ry)))
            ref_scale = float(np.max(np.abs(ry)))
            # mode 1 runs multi-row groups and the shared expert with FP32 activations
            if mode == 0 or (mode == 1 and x.shape[0] > 1):
                assert err <= 1e-4 * ref_scale, (rank, mode, err)
            else:
                assert float(np.mean(y.view(np.uint32) == ry.view(np.uint32))) >= 0.99, (rank, mode)
                assert err <= 1e-3 * ref_scale, (rank, mode, err)
        dist.barrier()
        full.free()
        layer.free()
    finally:
        dist.destroy_process_group()
