"""Expert parallelism for Decoder::experts (src/decoder/mod.rs:124-220).

The reference runs every expert of a MoE layer where the layer's tokens are.
Here the routed experts of one layer are split over the ranks of a
torch.distributed process group in contiguous blocks (rank r holds experts
[bounds[r], bounds[r + 1]) ), the shared expert and the router are on every
rank, and every rank brings its own tokens.  One forward:

  route     every rank routes its tokens (moe::route): top_k (expert, weight)
            pairs per token, in the reference's order.
  dispatch  the pairs, sorted by owning rank (stable: (token, j) order within
            a rank); one all_to_all of the per-rank counts, then two of the
            payload: the pair's row of x, and its expert id local to the owner.
  experts   the owner applies its experts to the rows it received.
  return    one all_to_all of the expert outputs back to the source rank,
            where they are put back in pair order (t * top_k + j).
  combine   the shared expert over the local tokens into y, then
            y[t] += weight * output over t's pairs in ascending expert id.

The result on each rank is Decoder::experts of that rank's tokens, bit for
bit.  The rows an expert receives are applied in one group per source rank
under QuantizationMode::DynamicActivations, whose arithmetic depends on the
group's row count (src/decoder/mod.rs:103-106: int8 for a single row); in the
other modes every row's result is independent of its group, so one call
covers all received rows.

Two forms of the exchange.  With counts (``capacity=None``) the per-rank
counts are exchanged first and the rows travel in variable-size chunks, which
needs the counts on the host.  With a fixed ``capacity`` (rows per rank pair,
``tokens * top_k`` always suffices) every rank sends ``capacity`` rows to every
rank, unused slots marked by expert id -1 and skipped by the experts: no
host synchronisation, so a whole step can be captured in a CUDA graph; the
dispatch (slot assignment and row gather) and the combine (reading the
returned rows by slot) run on the device.

This module's exchange runs torch.distributed's all_to_all_single: NCCL over
NVLink on GPUs, gloo on the CPU.  The library's own exchange
(``uocr_q8.PeerExpertParallel``, uocr_ep_* in the C ABI) moves only the rows
in use, as stores into the other GPUs' memory, and needs no collective;
``peer_expert_parallel`` below builds it over a process group.

The compute is a backend with the methods ``route``, ``expert_rows``,
``shared_rows``, ``combine`` (counts form) and ``dispatch``, ``combine_rows``
(fixed form); on GPUs it is ``LibraryBackend``, the CUDA
library's C ABI (uocr_moe_route, uocr_moe_expert_rows, uocr_moe_shared_rows,
uocr_moe_combine, uocr_moe_dispatch, uocr_moe_combine_rows), which runs on the
torch stream current at construction so that collectives and kernels are
ordered on one stream.  A failed collective (a rank that left, a
process-group timeout) raises OcrError "Nccl" instead of hanging.
"""
from __future__ import annotations

from typing import List, Sequence

import torch
import torch.distributed as dist

DYNAMIC_ACTIVATIONS = 1
EXCHANGE_ERROR = 9  # uocr_status UOCR_ERR_NCCL: the collective exchange failed


def _exchange(fn, *args, **kwargs):
    """One collective of the exchange; a failure (a rank that left, a
    process-group timeout, a transport error) becomes OcrError "Nccl"."""
    try:
        return fn(*args, **kwargs)
    except Exception as exc:
        from . import OcrError
        raise OcrError(EXCHANGE_ERROR, f"expert-parallel exchange failed: {exc}") from exc


def expert_bounds(n_experts: int, world: int) -> List[int]:
    """Contiguous expert blocks: the first n_experts % world ranks hold one more."""
    if world <= 0 or n_experts < world:
        raise ValueError(f"{n_experts} experts cannot be split over {world} ranks")
    base, extra = divmod(n_experts, world)
    bounds = [0]
    for r in range(world):
        bounds.append(bounds[-1] + base + (1 if r < extra else 0))
    return bounds


class ExpertParallelMoe:
    """One MoE layer whose routed experts are spread over a process group."""

    def __init__(self, backend, n_experts: int, top_k: int, hidden: int, group=None,
                 capacity=None):
        self.backend = backend
        self.capacity = capacity
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_experts = n_experts
        self.top_k = top_k
        self.hidden = hidden
        self.bounds = expert_bounds(n_experts, self.world)
        owner = torch.empty(n_experts, dtype=torch.int64)
        first = torch.empty(n_experts, dtype=torch.int64)
        for r in range(self.world):
            owner[self.bounds[r]:self.bounds[r + 1]] = r
            first[self.bounds[r]:self.bounds[r + 1]] = self.bounds[r]
        self._owner_cpu, self._first_cpu = owner, first
        self._tables = {}

    @property
    def local_experts(self) -> range:
        return range(self.bounds[self.rank], self.bounds[self.rank + 1])

    def _table(self, device):
        key = str(device)
        if key not in self._tables:
            self._tables[key] = (self._owner_cpu.to(device), self._first_cpu.to(device))
        return self._tables[key]

    def dispatch_plan(self, ids):
        """Send order of the pairs, their owners and the per-rank counts."""
        owner, first = self._table(ids.device)
        flat = ids.reshape(-1).to(torch.int64)
        dest = owner[flat]
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=self.world)
        local_ids = (flat - first[flat]).index_select(0, order).to(torch.int32)
        return order, local_ids, send_counts

    def forward(self, x, logits, mode: int):
        """(y, ids, weights) for this rank's tokens x [T, hidden] with router
        logits [T, n_experts]."""
        if self.capacity is not None:
            return self._forward_fixed(x, logits, mode)
        k, H = self.top_k, self.hidden
        T = x.shape[0]
        ids, wts = self.backend.route(logits)
        order, local_ids, send_counts = self.dispatch_plan(ids)
        recv_counts = torch.empty_like(send_counts)
        _exchange(dist.all_to_all_single, recv_counts, send_counts, group=self.group)
        sc = send_counts.tolist()
        rc = recv_counts.tolist()
        n_recv = sum(rc)
        send_x = x.index_select(0, torch.div(order, k, rounding_mode="floor"))
        recv_x = x.new_empty((n_recv, H))
        recv_ids = local_ids.new_empty((n_recv,))
        _exchange(dist.all_to_all_single, recv_x, send_x, rc, sc, group=self.group)
        _exchange(dist.all_to_all_single, recv_ids, local_ids, rc, sc, group=self.group)
        out = x.new_empty((n_recv, H))
        if mode == DYNAMIC_ACTIVATIONS:
            pos = 0
            for c in rc:
                if c:
                    self.backend.expert_rows(recv_x[pos:pos + c], recv_ids[pos:pos + c], mode,
                                             out[pos:pos + c])
                pos += c
        elif n_recv:
            self.backend.expert_rows(recv_x, recv_ids, mode, out)
        back = x.new_empty((T * k, H))
        _exchange(dist.all_to_all_single, back, out, sc, rc, group=self.group)
        pair_out = torch.empty_like(back)
        pair_out.index_copy_(0, order, back)
        y = self.backend.shared_rows(x, mode)
        self.backend.combine(ids, wts, pair_out, y)
        return y, ids, wts

    def _forward_fixed(self, x, logits, mode: int):
        C, W = self.capacity, self.world
        if x.shape[0] * self.top_k > C:
            raise ValueError(f"{x.shape[0]} tokens x top-{self.top_k} exceed capacity {C}")
        ids, wts = self.backend.route(logits)
        send_x, send_ids, pair_rows = self.backend.dispatch(x, ids, self.bounds, C)
        recv_x = torch.empty_like(send_x)
        recv_ids = torch.empty_like(send_ids)
        _exchange(dist.all_to_all_single, recv_x, send_x, group=self.group)
        _exchange(dist.all_to_all_single, recv_ids, send_ids, group=self.group)
        out = torch.empty_like(recv_x)
        if mode == DYNAMIC_ACTIVATIONS:
            for r in range(W):
                seg = slice(r * C, (r + 1) * C)
                self.backend.expert_rows(recv_x[seg], recv_ids[seg], mode, out[seg])
        else:
            self.backend.expert_rows(recv_x, recv_ids, mode, out)
        back = torch.empty_like(out)
        _exchange(dist.all_to_all_single, back, out, group=self.group)
        y = self.backend.shared_rows(x, mode)
        self.backend.combine_rows(ids, wts, back, pair_rows, y)
        return y, ids, wts


class LibraryBackend:
    """The CUDA library behind ExpertParallelMoe on one GPU.

    ``layer`` is a uocr_q8.MoeLayer holding this rank's experts (ids local to
    it) and the shared expert; routing uses the whole layer's expert count."""

    def __init__(self, ctx, layer, n_experts: int, top_k: int, normalize: bool = False,
                 scale: float = 1.0):
        import uocr_q8
        self._q8 = uocr_q8
        self.ctx = ctx
        self.layer = layer
        self.n_experts = n_experts
        self.top_k = top_k
        self.normalize = normalize
        self.scale = scale
        ctx.set_stream(torch.cuda.current_stream(ctx.device))

    def route(self, logits):
        return self._q8.route_device(self.ctx, logits, self.top_k, self.normalize, self.scale)

    def expert_rows(self, x, local_ids, mode, out):
        self.layer.expert_rows_device(x, local_ids, mode, out)

    def shared_rows(self, x, mode):
        return self.layer.shared_rows_device(x, mode)

    def combine(self, ids, wts, pair_out, y):
        self._q8.combine_device(self.ctx, ids, wts, pair_out, y)

    def dispatch(self, x, ids, bounds, capacity):
        return self._q8.dispatch_device(self.ctx, x, ids, bounds, capacity)

    def combine_rows(self, ids, wts, rows, pair_rows, y):
        self._q8.combine_rows_device(self.ctx, ids, wts, rows, pair_rows, y)


def local_layer(ctx, shared: Sequence, experts: Sequence[Sequence], bounds: Sequence[int],
                rank: int):
    """The MoeLayer of rank ``rank``: the shared expert and experts
    [bounds[rank], bounds[rank + 1]) of ``experts`` (gate, up, down each)."""
    import uocr_q8
    mine = list(experts[bounds[rank]:bounds[rank + 1]])
    # top_k and the routing arguments are not used by the per-part calls
    return uocr_q8.MoeLayer(ctx, shared, mine, top_k=1)


def peer_expert_parallel(ctx, local_layer, n_experts: int, top_k: int, max_tokens: int,
                         group=None, normalize: bool = False, scale: float = 1.0):
    """This rank's uocr_q8.PeerExpertParallel over the ranks of a process
    group (one GPU each), connected: the handles of all ranks are gathered
    with all_gather_object (any backend)."""
    import uocr_q8
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    ep = uocr_q8.PeerExpertParallel(ctx, local_layer, n_experts, top_k,
                                    expert_bounds(n_experts, world), rank, max_tokens,
                                    normalize, scale)
    handles = [None] * world
    dist.all_gather_object(handles, ep.handle(), group=group)
    ep.connect(handles)
    return ep


def decoder_peer_experts(decoder, max_tokens: int, group=None):
    """Per layer of ``decoder``, this rank's connected PeerExpertParallel over
    the ranks of ``group`` (None for dense layers), built from the layer's
    shared expert and this rank's share of its routed experts (the decoder's
    weights are the same on every rank).  Without an initialised process
    group the world is this GPU alone (connected locally)."""
    import uocr_q8
    world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
    rank = dist.get_rank(group) if world > 1 else 0
    cfg = decoder.cfg
    bounds = expert_bounds(cfg.experts, world)
    out = []
    for layer in decoder.layers:
        if layer.moe is None:
            out.append(None)
            continue
        shared, experts = layer.moe._keep
        local = uocr_q8.MoeLayer(decoder.ctx, shared, experts[bounds[rank]:bounds[rank + 1]], 1)
        ep = uocr_q8.PeerExpertParallel(decoder.ctx, local, cfg.experts, cfg.top_k, bounds, rank,
                                        max_tokens, cfg.normalize, cfg.routed_scale)
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, ep.handle(), group=group)
            ep.connect(handles)
        else:
            uocr_q8.PeerExpertParallel.connect_local([ep])
        out.append(ep)
    return out

