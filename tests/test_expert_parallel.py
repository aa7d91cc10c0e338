"""Expert parallelism of the MoE layer (uocr_q8.expert_parallel).

No counterpart in the reference, which runs Decoder::experts
(src/decoder/mod.rs:124-220) on one device: the routed experts are split over
the ranks in contiguous blocks and rows travel by all_to_all.  On the CPU,
world_size-2 gloo ranks run the dispatch/combine logic over an oracle backend
and must reproduce oracle.experts of their own tokens bit for bit in every
mode (ragged token counts, an empty rank, uneven expert blocks, renormalised
and scaled routing).  On two GPUs, NCCL ranks run the CUDA library and must
equal the single-GPU layer bit for bit.
"""
import os
import socket

import pytest

import ep_worker


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def spawn(fn, world, case):
    import torch.multiprocessing as mp
    mp.spawn(fn, args=(world, free_port(), case), nprocs=world, join=True)


BASE = dict(seed=3, hidden=64, width=32, shared_width=64, experts=8, top_k=3,
            normalize=False, scale=1.0, modes=[0, 1, 2])


def test_expert_bounds():
    from uocr_q8.expert_parallel import expert_bounds
    assert expert_bounds(64, 8) == [0, 8, 16, 24, 32, 40, 48, 56, 64]
    assert expert_bounds(7, 2) == [0, 4, 7]
    assert expert_bounds(5, 5) == [0, 1, 2, 3, 4, 5]
    with pytest.raises(ValueError):
        expert_bounds(3, 4)


@pytest.mark.parametrize("tokens", [(5, 7), (1, 1), (0, 6)])
def test_ep_gloo_matches_oracle(tokens):
    spawn(ep_worker.cpu_rank, 2, dict(BASE, tokens=list(tokens)))


@pytest.mark.parametrize("tokens", [(5, 7), (0, 6)])
def test_ep_gloo_fixed_capacity(tokens):
    """The fixed-capacity exchange (no counts on the host): same results."""
    spawn(ep_worker.cpu_rank, 2, dict(BASE, seed=6, tokens=list(tokens), capacity=7 * 3))


def test_ep_gloo_uneven_blocks_renormalised():
    spawn(ep_worker.cpu_rank, 2, dict(BASE, seed=9, experts=7, top_k=4, normalize=True,
                                      scale=2.5, tokens=[9, 4]))


@pytest.mark.parametrize("capacity", [None, 4 * 3])
def test_ep_gloo_rank_leaves_between_steps(tmp_path, capacity):
    """Failure detection on the host: after one step the last rank exits; the
    other rank's next exchange raises OcrError "Nccl" (a dropped peer is an
    error, not a hang), within the 10 s process-group timeout."""
    import time
    t0 = time.time()
    spawn(ep_worker.cpu_rank_leaves, 2, dict(BASE, seed=12, tokens=[4, 4], capacity=capacity,
                                              out=str(tmp_path)))
    assert (tmp_path / "rank0").read_text() == "Nccl"
    assert (tmp_path / "rank1").read_text() == "left"
    assert time.time() - t0 < 60


@pytest.mark.gpu
@pytest.mark.parametrize("case", [
    dict(BASE, hidden=256, width=128, shared_width=256, tokens=[37, 20]),
    dict(BASE, seed=4, hidden=1280, width=896, shared_width=1792, experts=64, top_k=6,
         tokens=[64, 64], modes=[1, 2]),
    dict(BASE, seed=5, hidden=1280, width=896, shared_width=1792, experts=64, top_k=6,
         tokens=[32, 20], modes=[0, 1, 2], capacity=32 * 6),
])
def test_ep_two_gpus_matches_single_gpu(case):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    spawn(ep_worker.gpu_rank, 2, case)
