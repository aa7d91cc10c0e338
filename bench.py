"""Benchmark of the B200 q8-block32 MoE path.

Default workload (the one the multi-GPU scaling runs measure): the 12-layer
decoder's MoE FFN layer at decode with its routed experts split over the GPUs
(expert parallelism).  Every GPU brings a decode batch of 64 tokens (weak
scaling) and holds 64/N of the 64 routed experts (gate/up [896x1280], down
[1280x896], q8-block32) plus the fused shared expert (width 1792).  One layer
forward: router logits -> top-6 (moe::route) -> dispatch of every (token,
expert) row into the owning GPU's memory (stores over NVLink, the library's
own kernels) -> the owners' grouped SwiGLU projections -> return of the
outputs -> ordered combine with the shared expert's output.  FP32
activations by default (--ep-mode 2: int8 activations for every row).

metric  : decode tok/s = tokens of all GPUs / device time (max over ranks).
value   : device-resident inputs; a step replays a CUDA graph of R
          consecutive layer forwards over distinct layers (weights from HBM),
          R sized so that the K timed steps last >= 0.6 s.
e2e     : the same metric through uocr_ep_forward_host (pinned host x and
          logits copied in, y copied out, synchronous per layer forward).
ep_parity: one step of the sharded layer against the single-GPU layer on rank
          0's tokens (FP32 activations within the FP32 tolerance, int8
          activations bit for bit).
secondary (one GPU only): every other configuration, bounded: the one-token
          MoE decode layer (GB/s), the GEMV stream (GB/s), grouped prefill at
          1024 tokens in both modes (TOP/s), the int8 micro-suite, decode
          attention and the whole 12-layer decode step.
--impl reference: the reference's scalar CPU path (oracle port, all host
          threads) on the default workload, rank 0 only.
Inputs are seeded synthetic data with the configurations' distributions
(x ~ N(0,1), logits ~ N(0,1), int8 weights uniform in [-127,127], scales ~
U(1e-4,1e-2)).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "unlimited-ocr-kernel_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

H, F, FS, E, TOPK = 1280, 896, 1792, 64, 6
MAT_BYTES = lambda r, c: r * c + r * ((c + 31) // 32) * 4
STEP_WEIGHT_BYTES = TOPK * 3 * MAT_BYTES(F, H) + 3 * MAT_BYTES(FS, H)  # 30,965,760
STEP_BYTES = STEP_WEIGHT_BYTES + H * 4 + E * 4 + H * 4
METRIC = "q8-block32 expert GEMV GB/s (MoE decode layer, one token)"
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch, from the
# ncu captures summarised in profiles/moe_decode_kernel_one_token_layer.md and
# profiles/gemv_tma_kernel_896x1280_stream.md (16 matrices per GEMV launch).
DECODE_TRAFFIC = 31_045_632
GEMV_TRAFFIC = 4 * 20_668_928  # the 16-matrix capture scaled to a 64-matrix launch
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM = 6650.0


def kept_graph():
    """A CUDA graph whose cudaGraph_t is kept after capture, so that its
    kernel nodes can be counted (graph_launches); replay instantiates it."""
    import torch
    return torch.cuda.CUDAGraph(keep_graph=True)


def graph_launches(graph):
    """Kernel launches of one replay of a kept graph that are this library's
    own kernels: the graph's kernel nodes whose function (driver API name,
    mangled) is in namespace uocr; torch's copies and index kernels are not
    counted.  None if the graph cannot be inspected."""
    try:
        from cuda.bindings import driver as drv
        h = graph.raw_cuda_graph()
        h = h if isinstance(h, drv.CUgraph) else drv.CUgraph(init_value=int(h))
        err, _, n = drv.cuGraphGetNodes(h, 0)
        if err != drv.CUresult.CUDA_SUCCESS:
            return None
        err, nodes, n = drv.cuGraphGetNodes(h, n)
        ours = 0
        for nd in nodes[:n]:
            err, t = drv.cuGraphNodeGetType(nd)
            if t != drv.CUgraphNodeType.CU_GRAPH_NODE_TYPE_KERNEL:
                continue
            err, prm = drv.cuGraphKernelNodeGetParams(nd)
            if err != drv.CUresult.CUDA_SUCCESS:
                return None
            name = None
            if int(prm.func):
                err, name = drv.cuFuncGetName(prm.func)
            elif int(getattr(prm, "kern", 0) or 0):
                err, name = drv.cuKernelGetName(prm.kern)
            if name is None or err != drv.CUresult.CUDA_SUCCESS:
                return None
            name = name.decode() if isinstance(name, bytes) else str(name)
            ours += "uocr" in name
        return ours
    except Exception as exc:  # an inspection failure leaves the count unknown
        print(f"graph_launches: {exc}", file=sys.stderr)
        return None


def _launches(per_replay, replays):
    return None if per_replay is None else per_replay * replays


def peak_hbm():
    try:
        with open(PEAKS_PATH) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            parts = [p.strip() for p in l.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl" if os.environ.get("BENCH_BACKEND") != "gloo" else "gloo",
                                timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def build_layers(ctx, n_layers, device, seed):
    """n_layers MoE layers of the upstream decoder's shapes (64 experts of width
    896, top-6, shared expert 1792, hidden 1280), generated on the device."""
    import torch

    import uocr_q8
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    layers = []

    def mat(r, c):
        w = torch.randint(-127, 128, (r, c), dtype=torch.int8, device=device, generator=g)
        s = (torch.rand((r, (c + 31) // 32), device=device, generator=g) * (1e-2 - 1e-4) + 1e-4)
        return uocr_q8.Int8Matrix.from_device(r, c, w, s.float().contiguous(), ctx)

    for _ in range(n_layers):
        shared = [mat(FS, H), mat(FS, H), mat(H, FS)]
        experts = [[mat(F, H), mat(F, H), mat(H, F)] for _ in range(E)]
        layers.append(uocr_q8.MoeLayer(ctx, shared, experts, TOPK))
    return layers


def run_ours(args):
    import torch

    import uocr_q8
    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    ctx = uocr_q8.GpuContext(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    n_layers = args.layers
    layers = build_layers(ctx, n_layers, dev, 1234 + rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(99 + rank)
    chunk = args.graph_steps
    n_inputs = chunk
    xs = torch.randn((n_inputs, 1, H), device=dev, generator=gen)
    lg = torch.randn((n_inputs, 1, E), device=dev, generator=gen)
    ys = torch.empty((n_inputs, 1, H), device=dev)
    torch.cuda.synchronize()

    def enqueue(i):
        layers[i % n_layers].forward_device(xs[i % n_inputs], lg[i % n_inputs], 0, ys[i % n_inputs])

    with torch.cuda.stream(stream):  # eager pass: sizes the context workspace
        for i in range(chunk):
            enqueue(i)
    ctx.sync()
    # capture `chunk` consecutive steps (distinct layers and tokens) in a graph
    graph = kept_graph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(chunk):
            enqueue(i)
    per_replay = graph_launches(graph)
    reps = max(1, args.steps // chunk)
    steps = reps * chunk
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    ctx.sync()

    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(reps):
                graph.replay()
            stop.record(stream)
        stop.synchronize()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop)
    ctx.sync()
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_step = ms / steps
    value = world * STEP_BYTES * steps / (ms * 1e-3) / 1e9

    # ---- end to end: host buffers through the C ABI, one call per step
    e2e_steps = min(steps, args.e2e_steps)
    hx = torch.empty((n_inputs, 1, H), pin_memory=True)
    hl = torch.empty((n_inputs, 1, E), pin_memory=True)
    hy = torch.empty((n_inputs, 1, H), pin_memory=True)
    hx.copy_(xs.cpu())
    hl.copy_(lg.cpu())
    for i in range(3):
        layers[i % n_layers].forward_host_ptrs(hx[i].data_ptr(), hl[i].data_ptr(), 1, hy[i].data_ptr())
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        j = i % n_inputs
        layers[i % n_layers].forward_host_ptrs(hx[j].data_ptr(), hl[j].data_ptr(), 1, hy[j].data_ptr())
    e2e_s = time.perf_counter() - t0
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * STEP_BYTES * e2e_steps / e2e_s / 1e9

    peak, peak_kind = peak_hbm()
    result = None
    if rank == 0:
        cpu = cpu_baseline(args) if (world == 1 and not args.no_cpu) else None
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms_step, 6),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded; x, logits ~ N(0,1), int8 weights uniform in [-127,127], scales ~ U(1e-4,1e-2))",
            "config": {"workload": "moe_decode_layer_1_token", "tokens_per_step": 1,
                       "hidden": H, "experts": E, "top_k": TOPK, "expert_width": F,
                       "shared_width": FS, "mode": "weights_only (fp32 activations)",
                       "l2": f"rotating pool of {n_layers} layers x 255.5 MB (> 126 MB L2)",
                       "parallelism": f"dp{world} (independent token streams)",
                       "bytes_per_step": STEP_BYTES},
            "e2e": {"value": round(e2e, 3), "unit": "GB/s", "steps": e2e_steps,
                    "us_per_step": round(e2e_s / e2e_steps * 1e6, 3),
                    "h2d_bytes_per_step": (H + E) * 4, "d2h_bytes_per_step": H * 4},
            "roofline": {"bound": "hbm", "kernel": "moe_decode_kernel (one cooperative launch per step)",
                         "achieved": round(STEP_BYTES / (ms_step * 1e-3) / 1e9, 2),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(STEP_BYTES / (ms_step * 1e-3) / 1e9 / peak, 4),
                         "traffic": args.traffic if args.traffic is not None else DECODE_TRAFFIC},
            "gpu_launches": _launches(per_replay, reps),
            "clocks": clocks.summary(),
        }
        if cpu:
            result["cpu_baseline"] = cpu
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        del graph
        dist.destroy_process_group()
    return result


GEMV_BYTES = MAT_BYTES(F, H) + H * 4 + F * 4  # one [896x1280] GEMV: 1,298,944 B
GEMV_PER_LAUNCH = 64  # matrices per multi-GEMV launch (82.6 MB of weights)


def run_gemv(args):
    """Config 0 (secondary workload): single [896x1280] GEMV, FP32 or int8
    activations, measured as a batched stream over a pool of distinct matrices
    (64 per launch) so the weights come from HBM."""
    import torch

    import uocr_q8
    dev = "cuda:0"
    torch.cuda.set_device(0)
    ctx = uocr_q8.GpuContext(0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    pool = 256  # 256 x 1.29 MB = 330 MB > L2
    mats = []
    for _ in range(pool):
        w = torch.randint(-127, 128, (F, H), dtype=torch.int8, device=dev, generator=g)
        s = (torch.rand((F, H // 32), device=dev, generator=g) * (1e-2 - 1e-4) + 1e-4).contiguous()
        mats.append(uocr_q8.Int8Matrix.from_device(F, H, w, s, ctx))
    x = torch.randn(H, device=dev, generator=g)
    ys = [torch.empty(F, device=dev) for _ in range(pool)]
    mode = 1 if args.gemv_int8 else 0
    with torch.cuda.stream(stream):
        for i in range(0, pool, GEMV_PER_LAUNCH):
            uocr_q8.linear_multi_device(ctx, mats[i:i + GEMV_PER_LAUNCH], x,
                                        ys[i:i + GEMV_PER_LAUNCH], mode)
    ctx.sync()
    graph = kept_graph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(0, pool, GEMV_PER_LAUNCH):
            uocr_q8.linear_multi_device(ctx, mats[i:i + GEMV_PER_LAUNCH], x,
                                        ys[i:i + GEMV_PER_LAUNCH], mode)
    per_replay = graph_launches(graph)
    reps = max(1, args.steps // pool)
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(reps):
                graph.replay()
            stop.record(stream)
        stop.synchronize()
    ms = start.elapsed_time(stop)
    steps = reps * pool
    # single-call latency: one GEMV per launch
    m0 = mats[0]
    with torch.cuda.stream(stream):
        for _ in range(20):
            m0.linear_device(x.view(1, H), ys[0].view(1, F), dynamic=bool(mode))
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(200):
            mats[i % pool].linear_device(x.view(1, H), ys[0].view(1, F), dynamic=bool(mode))
        t1.record(stream)
    t1.synchronize()
    single_us = t0.elapsed_time(t1) * 1e3 / 200
    peak, peak_kind = peak_hbm()
    gbs = GEMV_BYTES * steps / (ms * 1e-3) / 1e9
    return {"metric": "q8-block32 expert GEMV GB/s (896x1280 GEMV, batched stream)",
            "value": round(gbs, 2), "unit": "GB/s", "n_gpus": 1, "steps": steps,
            "warmup": max(args.warmup, 3), "ms_per_step": round(ms / steps, 6),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8-act" if mode else "fp32", "data": "synthetic (seeded)",
            "config": {"workload": "gemv_896x1280", "pool": pool,
                       "matrices_per_launch": GEMV_PER_LAUNCH, "bytes_per_step": GEMV_BYTES},
            "single_call_us": round(single_us, 3),
            "roofline": {"bound": "hbm", "kernel": "gemv_tma_kernel", "achieved": round(gbs, 2),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(gbs / peak, 4),
                         "traffic": args.traffic if args.traffic is not None else GEMV_TRAFFIC},
            "gpu_launches": _launches(per_replay, reps), "clocks": clocks.summary(),
            "cpu_baseline": None if args.no_cpu else gemv_cpu_baseline(mode, 3.0)}


def make_cpu_layer(seed):
    import oracle
    rng = np.random.default_rng(seed)

    def m(r, c):
        return oracle.Matrix(rng.integers(-127, 128, size=(r, c), dtype=np.int8),
                             rng.uniform(1e-4, 1e-2, size=(r, (c + 31) // 32)).astype(np.float32))

    def ffn(w):
        return oracle.Ffn(m(w, H), m(w, H), m(H, w))

    return ffn(FS), [ffn(F) for _ in range(E)], rng


def cpu_baseline(args, seconds=None):
    """Reference scalar path (oracle port) on all host threads, bounded sample."""
    import oracle
    oracle.set_threads(0)
    shared, routed, rng = make_cpu_layer(7)
    budget = seconds if seconds is not None else args.cpu_seconds
    x = rng.standard_normal((1, H)).astype(np.float32)
    lg = rng.standard_normal((1, E)).astype(np.float32)
    oracle.experts(shared, routed, lg, x, TOPK, 0)  # warm
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget:
        x = rng.standard_normal((1, H)).astype(np.float32)
        lg = rng.standard_normal((1, E)).astype(np.float32)
        oracle.experts(shared, routed, lg, x, TOPK, 0)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(STEP_BYTES * n / dt / 1e9, 3), "unit": "GB/s",
            "cores": oracle.get_threads(), "kind": "port",
            "sample": f"{n} tokens (one MoE decode layer each) in {dt:.1f} s",
            "ms_per_step": round(dt / n * 1e3, 3)}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    import oracle
    oracle.set_threads(0)
    shared, routed, rng = make_cpu_layer(7)
    xs = rng.standard_normal((16, 1, H)).astype(np.float32)
    lgs = rng.standard_normal((16, 1, E)).astype(np.float32)
    for i in range(max(args.warmup, 3)):
        oracle.experts(shared, routed, lgs[i % 16], xs[i % 16], TOPK, 0)
    steps = args.steps if args.ref_steps is None else args.ref_steps
    t0 = time.perf_counter()
    for i in range(steps):
        oracle.experts(shared, routed, lgs[i % 16], xs[i % 16], TOPK, 0)
    dt = time.perf_counter() - t0
    v = STEP_BYTES * steps / dt / 1e9
    return {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s",
            "n_gpus": world, "steps": steps, "warmup": max(args.warmup, 3),
            "ms_per_step": round(dt / steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded; x, logits ~ N(0,1), int8 weights uniform in [-127,127], scales ~ U(1e-4,1e-2))",
            "config": {"workload": "moe_decode_layer_1_token", "tokens_per_step": 1,
                       "hidden": H, "experts": E, "top_k": TOPK, "expert_width": F,
                       "shared_width": FS, "mode": "weights_only (fp32 activations)",
                       "parallelism": "rank 0 only (host CPU)", "bytes_per_step": STEP_BYTES},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": oracle.get_threads(),
                             "kind": "port",
                             "sample": f"{steps} tokens, one MoE decode layer each (scalar "
                                       "restatement of the reference's Rust path; the Rust "
                                       "crate cannot be built here)"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def gemv_cpu_baseline(mode, seconds):
    """The reference's scalar linear / linear_dynamic_int8 (oracle port, rows
    split over all host threads) on one [896x1280] matrix, bounded."""
    import oracle
    rng = np.random.default_rng(0)
    m = oracle.Matrix(rng.integers(-127, 128, size=(F, H), dtype=np.int8),
                      rng.uniform(1e-4, 1e-2, size=(F, H // 32)).astype(np.float32))
    x = rng.standard_normal((1, H)).astype(np.float32)
    fn = oracle.linear_dynamic_int8 if mode else oracle.linear
    oracle.set_threads(0)
    fn(m, x)
    n, t0 = 0, time.perf_counter()
    while n == 0 or time.perf_counter() - t0 < seconds:
        fn(m, x)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(GEMV_BYTES * n / dt / 1e9, 3), "unit": "GB/s",
            "cores": oracle.get_threads(), "kind": "port",
            "sample": f"{n} GEMVs of one [896x1280] matrix in {dt:.1f} s"}


def prefill_cpu_baseline(mode, seconds):
    """The reference's serial grouped experts (oracle port, all host threads)
    on a sample of 128 tokens with Zipf(1.1) routing; TOP/s of that sample."""
    import oracle
    shared, routed, rng = make_cpu_layer(11)
    T = 128
    x = rng.standard_normal((T, H)).astype(np.float32)
    bias = np.empty(E, np.float32)
    bias[rng.permutation(E)] = -1.1 * np.log(np.arange(1, E + 1, dtype=np.float64))
    lg = (rng.standard_normal((T, E)) + bias).astype(np.float32)
    oracle.set_threads(0)
    ops = T * TOPK * 3 * 2 * F * H + T * 3 * 2 * FS * H
    n, t0 = 0, time.perf_counter()
    while n == 0 or time.perf_counter() - t0 < seconds:
        oracle.experts(shared, routed, lg, x, TOPK, mode)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(ops * n / dt / 1e12, 5), "unit": "TOP/s", "cores": oracle.get_threads(),
            "kind": "port", "sample": f"{n} prefills of 128 tokens through one MoE layer in {dt:.1f} s"}


def int8suite_cpu_baseline(seconds):
    """The reference's scalar linear_dynamic_int8 (oracle port, all host
    threads), row by row, for M = 16 rows of an [896x1280] matrix."""
    import oracle
    rng = np.random.default_rng(3)
    m = oracle.Matrix(rng.integers(-127, 128, size=(F, H), dtype=np.int8),
                      rng.uniform(1e-4, 1e-2, size=(F, H // 32)).astype(np.float32))
    x = (rng.standard_normal((16, H)) * rng.uniform(0.1, 10, (16, 1))).astype(np.float32)
    oracle.set_threads(0)
    n, t0 = 0, time.perf_counter()
    while n == 0 or time.perf_counter() - t0 < seconds:
        oracle.linear_dynamic_int8(m, x)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(2.0 * 16 * F * H * n / dt / 1e12, 5), "unit": "TOP/s",
            "cores": oracle.get_threads(), "kind": "port",
            "sample": f"{n} calls of 16 rows x [896x1280] in {dt:.1f} s"}


PREFILL_TOKENS = 1024
# grouped prefill algorithmic work: 6144 (token, expert) pairs x 3 projections of [896x1280]
# plus 1024 tokens through the shared expert's 3 projections of [1792x1280]
PREFILL_OPS = PREFILL_TOKENS * TOPK * 3 * 2 * F * H + PREFILL_TOKENS * 3 * 2 * FS * H
PREFILL_WEIGHT_BYTES = E * 3 * MAT_BYTES(F, H) + 3 * MAT_BYTES(FS, H)  # 255,467,520


def peak_tensor():
    try:
        with open(PEAKS_PATH) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def zipf_logits(gen, tokens, experts, s=1.1):
    """Router logits with a Zipf(s) popularity bias over a random expert order
    plus N(0,1) noise (the stand-in for a real prefill's routing)."""
    import torch
    order = torch.randperm(experts, generator=gen, device=gen.device)
    bias = torch.empty(experts, device=gen.device)
    bias[order] = -s * torch.log(torch.arange(1, experts + 1, device=gen.device, dtype=torch.float32))
    return (torch.randn((tokens, experts), device=gen.device, generator=gen) + bias).contiguous()


def run_prefill(args):
    """Config 2: grouped prefill through one MoE layer, 1024 tokens, top-6 of
    64 experts with a Zipf(1.1) router bias, one mode per run (--prefill-mode
    0 = weights-only fp32 activations, 2 = int8 activations for every row)."""
    import torch

    import uocr_q8
    dev = "cuda:0"
    torch.cuda.set_device(0)
    ctx = uocr_q8.GpuContext(0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    layer = build_layers(ctx, 1, dev, 4321)[0]
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    T = PREFILL_TOKENS
    x = torch.randn((T, H), device=dev, generator=gen)
    lg = zipf_logits(gen, T, E)
    y = torch.empty((T, H), device=dev)
    mode = args.prefill_mode
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            layer.forward_device(x, lg, mode, y)
    ctx.sync()
    steps = max(1, args.steps)
    # launches of one forward, counted from a captured (never replayed) copy
    try:
        counted = kept_graph()
        with torch.cuda.graph(counted, stream=stream):
            layer.forward_device(x, lg, mode, y)
        per_forward = graph_launches(counted)
        del counted
    except Exception as exc:
        print(f"prefill: launch count unavailable ({exc})", file=sys.stderr)
        per_forward = None
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(steps):
                layer.forward_device(x, lg, mode, y)
            stop.record(stream)
        stop.synchronize()
    ms = start.elapsed_time(stop) / steps
    ctx.sync()
    # end to end: pinned host x/logits in, y out, one synchronous call per step
    hx = torch.empty((T, H), pin_memory=True)
    hl = torch.empty((T, E), pin_memory=True)
    hy = torch.empty((T, H), pin_memory=True)
    hx.copy_(x.cpu())
    hl.copy_(lg.cpu())
    layer.forward_host_ptrs(hx.data_ptr(), hl.data_ptr(), T, hy.data_ptr(), mode)
    e2e_n = max(1, min(steps, 10))
    t0 = time.perf_counter()
    for _ in range(e2e_n):
        layer.forward_host_ptrs(hx.data_ptr(), hl.data_ptr(), T, hy.data_ptr(), mode)
    e2e_s = (time.perf_counter() - t0) / e2e_n
    tops = PREFILL_OPS / (ms * 1e-3) / 1e12
    peak_t, kind_t = peak_tensor()
    hbm, kind_h = peak_hbm()
    attainable = min(peak_t, PREFILL_OPS / PREFILL_WEIGHT_BYTES * hbm / 1e3)  # TFLOP/s
    return {"metric": "q8-block32 grouped prefill TOP/s (MoE layer, 1024 tokens)",
            "value": round(tops, 3), "unit": "TOP/s", "n_gpus": 1, "steps": steps,
            "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8-act" if mode else "fp32",
            "data": "synthetic (seeded; x ~ N(0,1), Zipf(1.1)-biased router logits)",
            "config": {"workload": "grouped_prefill_1024_tokens", "tokens": T, "experts": E,
                       "top_k": TOPK, "hidden": H, "expert_width": F, "shared_width": FS,
                       "mode": "weights_only (fp32 activations)" if mode == 0 else
                               "dynamic int8 activations, every row",
                       "ops_per_step": PREFILL_OPS, "weight_bytes": PREFILL_WEIGHT_BYTES,
                       "l2": "one layer = 255.5 MB of weights (> 126 MB L2)"},
            "e2e": {"value": round(PREFILL_OPS / e2e_s / 1e12, 3), "unit": "TOP/s",
                    "steps": e2e_n, "ms_per_step": round(e2e_s * 1e3, 3),
                    "h2d_bytes_per_step": T * (H + E) * 4, "d2h_bytes_per_step": T * H * 4},
            "roofline": {"bound": "tensor",
                         "kernel": "whole step: grouped + shared " +
                                   ("q8_tc_gemm_f32_kernel (3 bf16 pieces)" if mode == 0 else
                                    "q8_tc_gemm_i8_kernel"),
                         "achieved": round(tops, 3), "peak": round(attainable, 1),
                         "peak_kind": f"min(bf16 dense {kind_t}, AI x HBM {kind_h})",
                         "unit": "TFLOP/s", "frac": round(tops / attainable, 5), "traffic": None},
            "gpu_launches": _launches(per_forward, steps), "clocks": clocks.summary(),
            "cpu_baseline": None if args.no_cpu else prefill_cpu_baseline(mode, 6.0)}


def run_int8suite(args):
    """Config 3: linear_dynamic_int8 (row-wise, bit-exact) for M in
    {1,16,128,512} x N in {896,1280,3840}, K = 1280; a pool of distinct
    matrices per shape keeps the weights coming from HBM."""
    import torch

    import uocr_q8
    dev = "cuda:0"
    torch.cuda.set_device(0)
    ctx = uocr_q8.GpuContext(0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    K = H
    cases = []
    launches = 0  # this library's kernels in the timed replays
    total_ops = 0.0
    total_bytes = 0.0
    total_s = 0.0
    with ClockSampler(0) as clocks:
        for N in (896, 1280, 3840):
            pool = max(2, (400 << 20) // MAT_BYTES(N, K))
            mats = []
            for _ in range(pool):
                w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
                sc = (torch.rand((N, K // 32), device=dev, generator=g) * (1e-2 - 1e-4) + 1e-4)
                mats.append(uocr_q8.Int8Matrix.from_device(N, K, w, sc.contiguous(), ctx))
            for M in (1, 16, 128, 512):
                x = (torch.randn((M, K), device=dev, generator=g) *
                     (torch.rand((M, 1), device=dev, generator=g) * 9.9 + 0.1)).contiguous()
                y = torch.empty((M, N), device=dev)
                # one call per matrix of the pool, captured once and replayed:
                # device time without the host's per-call cost
                with torch.cuda.stream(stream):
                    for i in range(pool):
                        mats[i].linear_device(x, y, dynamic=True)
                ctx.sync()
                graph = kept_graph()
                with torch.cuda.graph(graph, stream=stream):
                    for i in range(pool):
                        mats[i].linear_device(x, y, dynamic=True)
                replays = max(1, 2048 // pool)
                per = graph_launches(graph)
                launches = None if launches is None or per is None else launches + per * replays
                for _ in range(3):
                    graph.replay()
                torch.cuda.synchronize()
                t0 = torch.cuda.Event(enable_timing=True)
                t1 = torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(stream):
                    t0.record(stream)
                    for _ in range(replays):
                        graph.replay()
                    t1.record(stream)
                t1.synchronize()
                reps = replays * pool
                us = t0.elapsed_time(t1) * 1e3 / reps
                del graph
                ops = 2.0 * M * N * K
                byts = MAT_BYTES(N, K) + M * K * 4 + M * N * 4
                cases.append({"M": M, "N": N, "K": K, "us": round(us, 3),
                              "TOP/s": round(ops / (us * 1e-6) / 1e12, 3),
                              "GB/s": round(byts / (us * 1e-6) / 1e9, 1)})
                total_ops += ops
                total_bytes += byts
                total_s += us * 1e-6
            del mats
            ctx.sync()
    ctx.sync()
    agg = total_ops / total_s / 1e12
    return {"metric": "q8-block32 linear_dynamic_int8 micro-suite TOP/s",
            "value": round(agg, 3), "unit": "TOP/s", "n_gpus": 1, "steps": len(cases),
            "warmup": 3, "ms_per_step": round(total_s * 1e3 / len(cases), 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8-act",
            "data": "synthetic (seeded; rows ~ N(0,1) * U(0.1,10))",
            "config": {"workload": "int8_micro_suite", "K": K,
                       "aggregate": "total ops / total time over the 12 cases",
                       "timing": "CUDA graph of one call per pool matrix, replayed; "
                                 "pool > 400 MB so weights come from HBM"},
            "cases": cases, "clocks": clocks.summary(), "gpu_launches": launches,
            "roofline": {"bound": "hbm (M = 1, 16) / tensor (M >= 128)",
                         "kernel": "all cases: gemv_tma_kernel (M = 1), small_rows_kernel "
                                   "(M = 16), q8_tc_gemm_i8_kernel (M >= 128)",
                         "achieved": round(total_bytes / total_s / 1e9, 2),
                         "peak": peak_hbm()[0], "peak_kind": peak_hbm()[1], "unit": "GB/s",
                         "frac": round(total_bytes / total_s / 1e9 / peak_hbm()[0], 4),
                         "traffic": None},
            "cpu_baseline": None if args.no_cpu else int8suite_cpu_baseline(3.0)}


EP_TOKENS = 64  # a decode batch of 64 independent sequences
EP_EXPERT_BYTES = 3 * MAT_BYTES(F, H)
EP_SHARED_BYTES = 3 * MAT_BYTES(FS, H)


def ep_init(world, rank, local):
    """Process group of the EP workload: torchrun's, or one NCCL rank."""
    import datetime
    import socket

    import torch.distributed as dist
    if dist.is_initialized():
        return
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        return
    with socket.socket() as s_:
        s_.bind(("127.0.0.1", 0))
        port = s_.getsockname()[1]
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=120))


def run_ep(args):
    """Config 4's MoE layer at decode with expert parallelism: a global batch
    of 64 tokens split evenly over the ranks (strong scaling); each rank holds
    the shared expert and a contiguous block of the 64 routed experts; rows
    travel by NCCL all_to_all.  One step = one forward of the layer for the
    whole batch (route, dispatch, experts, return, combine).  Weights depend
    only on the expert id, so every N runs the same layer."""
    import math

    import torch
    import torch.distributed as dist

    import uocr_q8
    from uocr_q8.expert_parallel import ExpertParallelMoe, LibraryBackend, expert_bounds
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    ep_init(world, rank, local)
    ctx = uocr_q8.GpuContext(local)
    stream = torch.cuda.Stream(device=dev)
    bounds = expert_bounds(E, world)
    mine = range(bounds[rank], bounds[rank + 1])
    per_rank_bytes = len(mine) * EP_EXPERT_BYTES + EP_SHARED_BYTES
    n_layers = max(2, math.ceil(3 * 126e6 / per_rank_bytes))  # > L2 between reuses

    def mat(seed, r, c):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        w = torch.randint(-127, 128, (r, c), dtype=torch.int8, device=dev, generator=g)
        sc = torch.rand((r, (c + 31) // 32), device=dev, generator=g) * (1e-2 - 1e-4) + 1e-4
        return uocr_q8.Int8Matrix.from_device(r, c, w, sc.float().contiguous(), ctx)

    eps = []
    with torch.cuda.stream(stream):
        for li in range(n_layers):
            base = 100000 * (li + 1)
            shared = [mat(base + i, *rc) for i, rc in enumerate(((FS, H), (FS, H), (H, FS)))]
            experts = [[mat(base + 10 * (e + 1) + i, *rc)
                        for i, rc in enumerate(((F, H), (F, H), (H, F)))] for e in mine]
            layer = uocr_q8.MoeLayer(ctx, shared, experts, top_k=1)
            # fixed-capacity exchange: no counts on the host, so steps are captured in a graph
            eps.append(ExpertParallelMoe(LibraryBackend(ctx, layer, E, TOPK), E, TOPK, H,
                                         capacity=(EP_TOKENS // world) * TOPK))
    torch.cuda.synchronize()
    T = EP_TOKENS // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(555 + rank)
    n_in = 8
    xs = torch.randn((n_in, T, H), device=dev, generator=gen)
    lg = torch.randn((n_in, T, E), device=dev, generator=gen)
    mode = args.ep_mode

    def step(i, x, l):
        return eps[i % n_layers].forward(x, l, mode)[0]

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3) + n_layers):  # also sizes every layer's workspace
            step(i, xs[i % n_in], lg[i % n_in])
    torch.cuda.synchronize()
    # one graph of n_layers consecutive steps (distinct layers and tokens)
    graph = kept_graph()
    graphed = True
    try:
        with torch.cuda.graph(graph, stream=stream):
            for i in range(n_layers):
                step(i, xs[i % n_in], lg[i % n_in])
        per_replay = graph_launches(graph)
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
    except Exception as exc:  # capture not available: time eager steps
        graphed = False
        print(f"ep_decode: graph capture failed ({exc}); timing eager steps", file=sys.stderr)
    reps = max(1, args.steps // n_layers)
    steps = reps * n_layers
    dist.barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for r in range(reps):
                if graphed:
                    graph.replay()
                else:
                    for i in range(n_layers):
                        step(i, xs[i % n_in], lg[i % n_in])
            stop.record(stream)
        stop.synchronize()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop)
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    ms_step = ms / steps
    value = EP_TOKENS * steps / (ms * 1e-3)

    # end to end: pinned host x/logits in, y out, every step
    hx = torch.empty((n_in, T, H), pin_memory=True)
    hl = torch.empty((n_in, T, E), pin_memory=True)
    hy = torch.empty((n_in, T, H), pin_memory=True)
    hx.copy_(xs.cpu())
    hl.copy_(lg.cpu())
    e2e_steps = max(1, min(steps, args.e2e_steps))
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for i in range(e2e_steps):
            j = i % n_in
            x = hx[j].to(dev, non_blocking=True)
            l = hl[j].to(dev, non_blocking=True)
            hy[j].copy_(step(i, x, l), non_blocking=True)
        stream.synchronize()
    e2e_s = time.perf_counter() - t0
    t = torch.tensor([e2e_s], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_s = float(t.item())
    e2e = EP_TOKENS * e2e_steps / e2e_s
    ctx.sync()

    peak, peak_kind = peak_hbm()
    # bytes a rank must read per step: its experts' weights (at a batch of 64
    # nearly every expert is selected) and the shared expert's
    achieved = per_rank_bytes / (ms_step * 1e-3) / 1e9
    result = None
    if rank == 0:
        cpu = ep_cpu_baseline(args) if (world == 1 and not args.no_cpu) else None
        result = {
            "metric": "MoE layer decode tok/s (batch 64, expert-parallel over NCCL all_to_all)",
            "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": max(args.warmup, 3), "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp32" if mode == 0 else "int8-act",
            "data": "synthetic (seeded; int8 weights uniform in [-127,127], scales ~ U(1e-4,1e-2))",
            "config": {"workload": "moe_layer_ep_decode_nccl", "global_batch": EP_TOKENS,
                       "tokens_per_rank": T, "hidden": H, "experts": E, "top_k": TOPK,
                       "experts_per_rank": len(mine), "expert_width": F, "shared_width": FS,
                       "mode": mode, "parallelism": f"ep{world} (NCCL all_to_all, fixed capacity)",
                       "cuda_graph": graphed,
                       "l2": f"rotating pool of {n_layers} layers x "
                             f"{per_rank_bytes / 1e6:.1f} MB per rank (> 126 MB L2)"},
            "e2e": {"value": round(e2e, 1), "unit": "tok/s", "steps": e2e_steps,
                    "h2d_bytes_per_step": T * (H + E) * 4, "d2h_bytes_per_step": T * H * 4},
            "roofline": {"bound": "hbm", "kernel": "whole EP step (per-rank weight bytes)",
                         "achieved": round(achieved, 2), "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None},
            # route, dispatch (plan + rows), expert rows (grouping, split or quantize,
            # 3 warp-level + 3 tensor-core projections, SwiGLU, un-permute), shared
            # expert (split or quantize, 3 projections, SwiGLU), combine
            "gpu_launches": _launches(per_replay, reps) if graphed else None,
            "clocks": clocks.summary(),
        }
        if cpu:
            result["cpu_baseline"] = cpu
    dist.barrier()
    del graph  # a graph holding NCCL calls goes before the process group
    dist.destroy_process_group()
    return result


def ep_cpu_baseline(args):
    """The reference's scalar path (oracle port, all host threads) on a
    bounded sample: batches of 64 tokens through one MoE layer."""
    import oracle
    oracle.set_threads(0)
    shared, routed, rng = make_cpu_layer(7)
    x = rng.standard_normal((EP_TOKENS, H)).astype(np.float32)
    lg = rng.standard_normal((EP_TOKENS, E)).astype(np.float32)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < args.cpu_seconds:
        oracle.experts(shared, routed, lg, x, TOPK, args.ep_mode)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(EP_TOKENS * n / dt, 2), "unit": "tok/s", "cores": oracle.get_threads(),
            "kind": "port", "sample": f"{n} batches of 64 tokens through one MoE layer in {dt:.1f} s"}


ATTN_BATCH, ATTN_HEADS, ATTN_DIM, ATTN_PREFIX, ATTN_WINDOW = 64, 10, 128, 2048, 128
ATTN_TOKENS = ATTN_PREFIX + ATTN_WINDOW
# keys + values read per layer step: every token of every sequence, 4 B each
ATTN_BYTES = ATTN_BATCH * ATTN_TOKENS * ATTN_HEADS * ATTN_DIM * 4 * 2


def run_attn(args):
    """Config 4's attention (secondary workload): one decode step of
    ops::attention_decode for 64 sequences (10 heads x 128) over a KV cache
    of a 2048-token prefix plus a full 128-token ring, through
    uocr_kv_attention; value = KV bytes read / device time."""
    import torch

    import uocr_q8
    from uocr_q8.attention import KvCache
    torch.cuda.set_device(0)
    dev = "cuda:0"
    ctx = uocr_q8.GpuContext(0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    W = ATTN_HEADS * ATTN_DIM
    n_layers = 2  # 2 x 1.43 GB caches rotated (> L2)
    caches = []
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    with torch.cuda.stream(stream):
        for _ in range(n_layers):
            kv = KvCache(ctx, ATTN_BATCH, ATTN_HEADS, ATTN_DIM, ATTN_WINDOW, ATTN_PREFIX)
            for b in range(ATTN_BATCH):
                k = torch.randn((ATTN_PREFIX, W), device=dev, generator=g)
                kv.prefill(b, k, k.mul(0.5))
            for _ in range(ATTN_WINDOW):  # fill the ring
                r = torch.randn((ATTN_BATCH, W), device=dev, generator=g)
                kv.push(r, r)
            caches.append(kv)
        q = torch.randn((ATTN_BATCH, W), device=dev, generator=g) * 0.05
        out = torch.empty_like(q)
    ctx.sync()
    steps = max(4, min(args.steps, 400))
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            caches[i % n_layers].attention(q, out)
    ctx.sync()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for i in range(steps):
                caches[i % n_layers].attention(q, out)
            stop.record(stream)
        stop.synchronize()
    ctx.sync()
    ms = start.elapsed_time(stop) / steps
    gbs = ATTN_BYTES / (ms * 1e-3) / 1e9
    peak, peak_kind = peak_hbm()
    res = {"metric": "decode attention KV GB/s (batch 64, 10 heads x 128, prefix 2048 + ring 128)",
           "value": round(gbs, 2), "unit": "GB/s", "n_gpus": 1, "steps": steps,
           "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded)",
           "config": {"workload": "attention_decode_batch64", "batch": ATTN_BATCH,
                      "heads": ATTN_HEADS, "head_dim": ATTN_DIM, "prefix": ATTN_PREFIX,
                      "window": ATTN_WINDOW, "bytes_per_step": ATTN_BYTES,
                      "l2": "2 caches x 1.43 GB rotated (> 126 MB L2)"},
           "roofline": {"bound": "hbm", "kernel": "attn_decode_tma_kernel", "achieved": round(gbs, 2),
                        "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                        "frac": round(gbs / peak, 4), "traffic": args.traffic},
           "gpu_launches": steps, "clocks": clocks.summary()}
    if not args.no_cpu:
        res["cpu_baseline"] = attn_cpu_baseline(min(args.cpu_seconds, 8.0))
    for kv in caches:
        kv.free()
    return res


DEC_BATCH, DEC_PREFIX = 64, 2048


def decode_step_bytes(cfg, tokens_per_seq, lm_head="q8"):
    """Algorithmic HBM bytes of one batched decode step: every layer's KV
    (keys + values of every present token of every sequence), every weight
    the step reads (attention projections, the dense FFN, the shared expert,
    the routed experts the batch selects — all of them at batch 64 — and
    lm_head), the router and the embedding rows."""
    H = cfg.hidden
    kv = cfg.layers * DEC_BATCH * tokens_per_seq * H * 4 * 2
    q8 = lambda r, c: r * c + r * ((c + 31) // 32) * 4
    attn = cfg.layers * 4 * q8(H, H)
    dense = cfg.first_dense * (2 * q8(cfg.dense_width, H) + q8(H, cfg.dense_width))
    moe_layers = cfg.layers - cfg.first_dense
    moe = moe_layers * ((cfg.experts * (2 * q8(cfg.expert_width, H) + q8(H, cfg.expert_width)))
                        + 2 * q8(cfg.shared_width, H) + q8(H, cfg.shared_width)
                        + cfg.experts * H * 2)
    head = q8(cfg.vocab, H) if lm_head == "q8" else cfg.vocab * H * 2
    return kv + attn + dense + moe + head + DEC_BATCH * H * 2


def attn_cpu_baseline(seconds):
    """The oracle's ops::attention_decode (scalar port of the reference) for
    one sequence over 2176 tokens of 10 heads x 128, timed on the host for a
    bounded number of seconds; GB/s of keys + values read."""
    import oracle
    rng = np.random.default_rng(5)
    W = ATTN_HEADS * ATTN_DIM
    k = rng.standard_normal((ATTN_TOKENS, W)).astype(np.float32)
    v = (k * 0.5).astype(np.float32)
    q = (rng.standard_normal(W) * 0.05).astype(np.float32)
    oracle.attention_decode(q, k, v, ATTN_HEADS)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        oracle.attention_decode(q, k, v, ATTN_HEADS)
        n += 1
    dt = time.perf_counter() - t0
    per_seq = ATTN_TOKENS * W * 4 * 2
    return {"value": round(per_seq * n / dt / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{n} single-sequence attention_decode calls (2176 tokens) in {dt:.1f} s"}


def decode_cpu_baseline(seconds, prefix=DEC_PREFIX, mode=0, head=False):
    """One sequence's decode step through the oracle (the reference's scalar
    operations): attention block (norm, q/k/v/o, rope, cache push, attention
    over prefix + 128 tokens), BF16 router and MoE layer (64 experts, top 6,
    shared 1792), timed for a bounded number of seconds over MoE layers, plus
    one dense layer (and, with head, the q8 lm_head) timed once; tokens/s of
    a 12-layer step (1 dense + 11 MoE layers) for one sequence.  mode 1:
    DynamicActivations (every one-row projection with int8 activations)."""
    import oracle
    rng = np.random.default_rng(6)
    lin = oracle.linear_dynamic_int8 if mode else oracle.linear
    H, heads, dim = 1280, ATTN_HEADS, ATTN_DIM

    def m(r, c):
        return oracle.Matrix(rng.integers(-127, 128, size=(r, c), dtype=np.int8),
                             rng.uniform(1e-4, 1e-2, size=(r, (c + 31) // 32)).astype(np.float32))

    qkvo = [m(H, H) for _ in range(4)]
    norm = np.ones(H, np.float32)
    cache = oracle.LayerCache(heads, dim, 128)
    kp = rng.standard_normal((prefix, H)).astype(np.float32)
    cache.prefill(kp, kp * 0.5, prefix)
    for _ in range(127):
        r = rng.standard_normal(H).astype(np.float32)
        cache.push(r, r)
    shared = oracle.Ffn(m(FS, H), m(FS, H), m(H, FS))
    experts = [oracle.Ffn(m(F, H), m(F, H), m(H, F)) for _ in range(E)]
    router = (rng.standard_normal((E, H)).astype(np.float32) * 0.03).view(np.uint32) >> 16
    router = router.astype(np.uint16)

    def attention_block(x):
        n = oracle.rms_norm(x, norm)
        q, k, v = (lin(mm, n)[0] for mm in qkvo[:3])
        pos = cache.position()
        q, k = oracle.rope(q, dim, pos), oracle.rope(k, dim, pos)
        cache.push(k, v)
        a = oracle.attention_decode(q, cache.keys, cache.values, heads)
        return lin(qkvo[3], a[None])[0] + x[0]

    def moe_layer(x):
        r = attention_block(x)
        n = oracle.rms_norm(r[None], norm)
        lg = oracle.linear_bf16(router, n)
        y, _, _ = oracle.experts(shared, experts, lg, n, TOPK, mode)
        return (r + y[0])[None]

    x = rng.standard_normal((1, H)).astype(np.float32)
    moe_layer(x)
    n_layers, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        x = moe_layer(x)
        n_layers += 1
    moe_s = (time.perf_counter() - t0) / n_layers
    dense = oracle.Ffn(m(6848, H), m(6848, H), m(H, 6848))
    t1 = time.perf_counter()
    r = attention_block(x)
    oracle.feed_forward(dense, oracle.rms_norm(r[None], norm), mode)
    dense_s = time.perf_counter() - t1
    head_s = 0.0
    if head:
        lm = m(129280, H)
        t2 = time.perf_counter()
        lin(lm, oracle.rms_norm(x, norm))
        head_s = time.perf_counter() - t2
    step_s = 11 * moe_s + dense_s + head_s
    what = f"and the q8 lm_head ({head_s * 1e3:.1f} ms)" if head else "(lm_head not included)"
    return {"value": round(1.0 / step_s, 3), "unit": "tok/s", "cores": oracle.get_threads(),
            "kind": "port",
            "sample": f"{n_layers} MoE layers ({moe_s * 1e3:.1f} ms each) and one dense layer "
                      f"({dense_s * 1e3:.1f} ms) of one sequence over a {prefix}-token prefix, "
                      f"mode {mode}; a 12-layer step = 11 MoE + 1 dense {what}"}


def run_decode(args):
    """Config 4 on one GPU: a batched decode step of the 12-layer decoder
    (64 sequences, 2048-token prefixes, 128-token ring) with random-init q8
    weights, replayed from a CUDA graph; value = tokens/s."""
    import torch

    import uocr_q8
    from uocr_q8.decoder import DecodeState, Decoder, DecoderConfig, decode_step
    torch.cuda.set_device(0)
    dev = "cuda:0"
    ctx = uocr_q8.GpuContext(0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    cfg = DecoderConfig()
    mode = args.decode_mode
    with torch.cuda.stream(stream):
        dec = Decoder.random(ctx, cfg, seed=11, lm_head=args.lm_head)
        state = DecodeState(dec, DEC_BATCH, DEC_PREFIX)
        g = torch.Generator(device=dev)
        g.manual_seed(12)
        for cache in state.caches:
            for b in range(DEC_BATCH):
                k = torch.randn((DEC_PREFIX, cfg.hidden), device=dev, generator=g)
                cache.prefill(b, k, k.mul(0.5))
        tokens = torch.randint(0, cfg.vocab, (DEC_BATCH,), device=dev, generator=g)
        logits = torch.empty((DEC_BATCH, cfg.vocab), device=dev)
        for _ in range(max(args.warmup, 3)):  # eager: sizes every workspace
            decode_step(dec, state, tokens, mode, logits)
    ctx.sync()
    graph = kept_graph()
    with torch.cuda.graph(graph, stream=stream):
        decode_step(dec, state, tokens, mode, logits)
        tokens.copy_(torch.argmax(logits, dim=1))
    per_replay = graph_launches(graph)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    steps = max(4, min(args.steps, 200))
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(steps):
                graph.replay()
            stop.record(stream)
        stop.synchronize()
    ms = start.elapsed_time(stop) / steps
    tok_s = DEC_BATCH / (ms * 1e-3)
    # ---- end to end: token ids in from pinned host memory, next ids out
    e2e_steps = max(4, min(steps, 50))
    h_in = torch.randint(0, cfg.vocab, (DEC_BATCH,), dtype=torch.int64).pin_memory()
    h_out = torch.empty((DEC_BATCH,), dtype=torch.int64).pin_memory()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for _ in range(e2e_steps):
            tokens.copy_(h_in, non_blocking=True)
            graph.replay()
            h_out.copy_(tokens, non_blocking=True)
            stream.synchronize()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    tokens_now = state.caches[0].state(0)[0]
    step_bytes = decode_step_bytes(cfg, tokens_now, args.lm_head)
    gbs = step_bytes / (ms * 1e-3) / 1e9
    peak, peak_kind = peak_hbm()
    res = {"metric": "decode tok/s (12-layer MoE decoder, batch 64, KV 2048)",
           "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": 1, "steps": steps,
           "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None,
           "dtype": "int8-act" if mode else "fp32", "data": "synthetic (seeded; random-init weights)",
           "config": {"workload": "decode_step_12_layers", "batch": DEC_BATCH, "prefix": DEC_PREFIX,
                      "window": cfg.window, "layers": cfg.layers, "hidden": cfg.hidden,
                      "experts": cfg.experts, "top_k": cfg.top_k, "vocab": cfg.vocab,
                      "lm_head": args.lm_head, "mode": mode, "cuda_graph": True,
                      "tokens_per_sequence": tokens_now, "bytes_per_step": step_bytes,
                      "l2": "17 GB of KV per step (> 126 MB L2)"},
           "e2e": {"value": round(DEC_BATCH / e2e_s, 1), "unit": "tok/s", "steps": e2e_steps,
                   "ms_per_step": round(e2e_s * 1e3, 4), "h2d_bytes_per_step": DEC_BATCH * 8,
                   "d2h_bytes_per_step": DEC_BATCH * 8},
           "roofline": {"bound": "hbm", "kernel": "whole step (attention, MoE, projections)",
                        "achieved": round(gbs, 2), "peak": peak, "peak_kind": peak_kind,
                        "unit": "GB/s", "frac": round(gbs / peak, 4), "traffic": None},
           "gpu_launches": _launches(per_replay, steps), "clocks": clocks.summary()}
    if args.lm_head == "bf16":
        # the BF16 lm_head alone (uocr_linear_bf16_tc, 129,280 x 1280 at batch
        # 64), weights from HBM (331 MB, more than L2), events on its stream
        from uocr_q8.decoder import linear_bf16_tc_device
        hx = torch.randn((DEC_BATCH, cfg.hidden), device=dev)
        hy = torch.empty((DEC_BATCH, cfg.vocab), device=dev)
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for _ in range(3):
                linear_bf16_tc_device(ctx, dec.lm_head, hx, hy)
            h0.record(stream)
            for _ in range(20):
                linear_bf16_tc_device(ctx, dec.lm_head, hx, hy)
            h1.record(stream)
        h1.synchronize()
        ctx.sync()
        us = h0.elapsed_time(h1) * 1e3 / 20
        hb = cfg.vocab * cfg.hidden * 2 + DEC_BATCH * cfg.hidden * 4 + DEC_BATCH * cfg.vocab * 4
        res["lm_head"] = {"kernel": "bf16_head_kernel (+ the activation split)", "us": round(us, 2),
                          "bytes": hb, "GB/s": round(hb / (us * 1e-6) / 1e9, 1),
                          "frac": round(hb / (us * 1e-6) / 1e9 / peak, 4), "peak_kind": peak_kind}
    state.free()
    if not args.no_cpu:
        res["cpu_baseline"] = decode_cpu_baseline(min(args.cpu_seconds, 10.0))
    return res



def decode_step_bytes_ep(cfg, tokens_per_seq, world, lm_head="q8"):
    """decode_step_bytes for one GPU of an expert-parallel step: this GPU's
    sequences' KV and projections, the shared expert and 1/world of every MoE
    layer's routed experts."""
    q8 = lambda r, c: r * c + r * ((c + 31) // 32) * 4
    routed = (cfg.layers - cfg.first_dense) * cfg.experts * (
        2 * q8(cfg.expert_width, cfg.hidden) + q8(cfg.hidden, cfg.expert_width))
    return decode_step_bytes(cfg, tokens_per_seq, lm_head) - routed + routed // world


def run_decode_ep(args):
    """Config 4 on N GPUs: the 12-layer decode step with the sequences split
    over the GPUs (each GPU: 64 sequences with 2048-token prefixes, their
    attention, projections, KV cache and lm_head) and every MoE layer's routed
    experts split over the GPUs (each holds 64/N of them; rows cross NVLink
    through the library's peer-memory exchange, uocr_ep_*).  Weak scaling:
    value = all GPUs' tokens / the slowest GPU's step time.  Rank 0 checks the
    first step against the plain one-GPU step (all experts) on a copy of its
    state."""
    import torch

    import uocr_q8
    from uocr_q8.decoder import DecodeState, Decoder, DecoderConfig, decode_step
    from uocr_q8.expert_parallel import decoder_peer_experts
    world, rank, local = dist_setup(args.gpus)
    if world > 1:
        import torch.distributed as dist
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    ctx = uocr_q8.GpuContext(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    cfg = DecoderConfig()
    mode = args.decode_mode
    with torch.cuda.stream(stream):
        dec = Decoder.random(ctx, cfg, seed=11, lm_head=args.lm_head)  # the same weights on every GPU
        states = [DecodeState(dec, DEC_BATCH, DEC_PREFIX) for _ in range(2 if rank == 0 else 1)]
        g = torch.Generator(device=dev)
        g.manual_seed(12 + rank)
        for li in range(cfg.layers):
            for b in range(DEC_BATCH):
                k = torch.randn((DEC_PREFIX, cfg.hidden), device=dev, generator=g)
                for st in states:
                    st.caches[li].prefill(b, k, k.mul(0.5))
        tokens = torch.randint(0, cfg.vocab, (DEC_BATCH,), device=dev, generator=g)
        logits = torch.empty((DEC_BATCH, cfg.vocab), device=dev)
    ctx.sync()
    eps = decoder_peer_experts(dec, DEC_BATCH)
    state = states[0]
    # parity of the first step (every GPU steps through the exchange together)
    with torch.cuda.stream(stream):
        decode_step(dec, state, tokens, mode, logits, experts=eps)
    ctx.sync()
    parity = None
    if rank == 0:
        with torch.cuda.stream(stream):
            ref = decode_step(dec, states[1], tokens, mode)
        ctx.sync()
        a, b_ = logits.cpu().numpy(), ref.cpu().numpy()
        same = float(np.mean(a.view(np.uint32) == b_.view(np.uint32)))
        rel = float(np.max(np.abs(a.astype(np.float64) - b_)) / max(float(np.max(np.abs(b_))), 1e-30))
        parity = {"bit_identical": round(same, 6), "max_rel_diff": rel,
                  "ok": same == 1.0 if mode == 2 else rel <= 1e-3}
        states[1].free()
        del ref
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3) - 1):  # eager: sizes every workspace
            decode_step(dec, state, tokens, mode, logits, experts=eps)
    ctx.sync()
    if world > 1:
        dist.barrier()
    graph = kept_graph()
    with torch.cuda.graph(graph, stream=stream):
        decode_step(dec, state, tokens, mode, logits, experts=eps)
        tokens.copy_(torch.argmax(logits, dim=1))
    per_replay = graph_launches(graph)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    steps = max(4, min(args.steps, 200))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(steps):
                graph.replay()
            stop.record(stream)
        stop.synchronize()
    ms = start.elapsed_time(stop) / steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # ---- end to end: token ids in from pinned host memory, next ids out
    e2e_steps = max(4, min(steps, 50))
    h_in = torch.randint(0, cfg.vocab, (DEC_BATCH,), dtype=torch.int64).pin_memory()
    h_out = torch.empty((DEC_BATCH,), dtype=torch.int64).pin_memory()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for _ in range(e2e_steps):
            tokens.copy_(h_in, non_blocking=True)
            graph.replay()
            h_out.copy_(tokens, non_blocking=True)
            stream.synchronize()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    tokens_now = state.caches[0].state(0)[0]
    step_bytes = decode_step_bytes_ep(cfg, tokens_now, world, args.lm_head)
    gbs = step_bytes / (ms * 1e-3) / 1e9
    peak, peak_kind = peak_hbm()
    res = {"metric": "decode tok/s (12-layer MoE decoder, 64 sequences per GPU, KV 2048, "
                     "experts split over the GPUs)",
           "value": round(world * DEC_BATCH / (ms * 1e-3), 1), "unit": "tok/s", "n_gpus": world,
           "steps": steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "int8-act" if mode else "fp32", "data": "synthetic (seeded; random-init weights)",
           "config": {"workload": "decode_step_12_layers_ep", "batch_per_gpu": DEC_BATCH,
                      "prefix": DEC_PREFIX, "window": cfg.window, "layers": cfg.layers,
                      "hidden": cfg.hidden, "experts": cfg.experts, "top_k": cfg.top_k,
                      "vocab": cfg.vocab, "lm_head": args.lm_head, "mode": mode,
                      "parallelism": f"sequences split, experts split (ep{world}), peer memory",
                      "cuda_graph": True, "tokens_per_sequence": tokens_now,
                      "bytes_per_step_per_gpu": step_bytes,
                      "l2": "17 GB of KV per step and GPU (> 126 MB L2)"},
           "ep_parity": parity,
           "e2e": {"value": round(world * DEC_BATCH / e2e_s, 1), "unit": "tok/s",
                   "steps": e2e_steps, "ms_per_step": round(e2e_s * 1e3, 4),
                   "h2d_bytes_per_step": DEC_BATCH * 8, "d2h_bytes_per_step": DEC_BATCH * 8},
           "roofline": {"bound": "hbm", "kernel": "whole step per GPU (attention, MoE, projections)",
                        "achieved": round(gbs, 2), "peak": peak, "peak_kind": peak_kind,
                        "unit": "GB/s", "frac": round(gbs / peak, 4), "traffic": None},
           "gpu_launches": _launches(per_replay, steps), "clocks": clocks.summary()}
    del graph  # before the exchange and the process group go
    for e in eps:
        if e is not None:
            e.free()
    state.free()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res if rank == 0 else None


# ---------------------------------------------------------------------------
# The reference's fixed-work decoder benchmark (src/model/benchmark.rs:5-64):
# a 1517-token prefill, then 512 teacher-forced decode steps of one sequence
# whose logits are all consumed by a checksum, DynamicActivations, q8 lm_head.
FW_PREFIX, FW_STEPS, FW_RECORDED = 1517, 512, 250
FW_METRIC = "fixed-work decode tok/s (1517-token prefill, 512 teacher-forced steps, batch 1)"


def fixed_work_step_bytes(cfg, tokens):
    """Algorithmic HBM bytes of one batch-1 decode step: every weight the
    step reads (attention projections, dense FFN, shared expert, six routed
    experts per MoE layer, routers, q8 lm_head) and every layer's KV."""
    H = cfg.hidden
    q8 = lambda r, c: r * c + r * ((c + 31) // 32) * 4
    attn = cfg.layers * 4 * q8(H, H)
    dense = cfg.first_dense * (2 * q8(cfg.dense_width, H) + q8(H, cfg.dense_width))
    per_moe = (cfg.top_k * (2 * q8(cfg.expert_width, H) + q8(H, cfg.expert_width))
               + 2 * q8(cfg.shared_width, H) + q8(H, cfg.shared_width) + cfg.experts * H * 2)
    kv = cfg.layers * tokens * H * 4 * 2
    return attn + dense + (cfg.layers - cfg.first_dense) * per_moe + kv + q8(cfg.vocab, H)


def run_fixed_work(args):
    """The fixed-work decoder benchmark on one GPU with random-init weights of
    the upstream decoder's shapes (12 layers, 64 experts, q8 lm_head over
    129,280 tokens).  Synthetic stand-ins: the 1517 prefill rows (1513 image
    features + 4 prompt embeddings in the reference) are N(0, 1) rows, and the
    250 recorded token ids are seeded random ids, cycled to 512 steps.

    Each repetition: the embeddings (pinned host memory) are copied in, the
    prefill runs (eager launches; uocr_kv_attention_prefill for its causal
    attention), then 512 replays of a CUDA graph of one step (the step's token
    read from the device list, the decode step, the checksum of all 129,280
    logits), then the 8-byte checksum is read back.  The reference's first
    repetition is its warm-up; here a whole warm-up repetition precedes the
    timed ones.  value = 512 / decode seconds (median repetition)."""
    import torch

    import uocr_q8
    from uocr_q8.decoder import (DecodeState, Decoder, DecoderConfig, decode_step,
                                 logits_checksum_device, prefill)
    torch.cuda.set_device(0)
    dev = "cuda:0"
    ctx = uocr_q8.GpuContext(0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    cfg = DecoderConfig()
    mode = uocr_q8.QuantizationMode.DYNAMIC_ACTIVATIONS
    rng = np.random.default_rng(23)
    emb_h = torch.from_numpy(
        rng.standard_normal((FW_PREFIX, cfg.hidden)).astype(np.float32)).pin_memory()
    recorded = rng.integers(0, cfg.vocab, FW_RECORDED)
    tok_h = torch.from_numpy(np.resize(recorded, FW_STEPS).astype(np.int64)).pin_memory()
    acc_h = torch.zeros(1, dtype=torch.int64).pin_memory()
    with torch.cuda.stream(stream):
        dec = Decoder.random(ctx, cfg, seed=21, lm_head="q8")
        state = DecodeState(dec, 1, FW_PREFIX)
        emb_d = torch.empty((FW_PREFIX, cfg.hidden), device=dev)
        tok_d = torch.empty(FW_STEPS, dtype=torch.int64, device=dev)
        ctr = torch.zeros(1, dtype=torch.int64, device=dev)
        acc = torch.zeros(1, dtype=torch.int64, device=dev)
        logits = torch.empty((1, cfg.vocab), device=dev)

    def step():
        decode_step(dec, state, tok_d.index_select(0, ctr), mode, logits)
        logits_checksum_device(ctx, logits, acc)
        ctr.add_(1)

    def begin():
        state.reset(0)
        emb_d.copy_(emb_h, non_blocking=True)
        tok_d.copy_(tok_h, non_blocking=True)
        ctr.zero_()
        acc.zero_()
        return prefill(dec, state, emb_d, mode)

    with torch.cuda.stream(stream):  # warm-up: sizes every workspace
        begin()
        for i in range(3):
            if i == 2:  # one eager step in an NVTX range, for a profiler's launch list
                torch.cuda.nvtx.range_push("fixed_work_step")
            step()
            if i == 2:
                torch.cuda.nvtx.range_pop()
    ctx.sync()
    torch.cuda.synchronize()
    graph = kept_graph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    per_replay = graph_launches(graph)
    with torch.cuda.stream(stream):  # warm-up repetition through the graph
        begin()
        for _ in range(FW_STEPS):
            graph.replay()
    ctx.sync()
    torch.cuda.synchronize()
    reps = max(3, min(args.steps, 5))
    prefill_s, decode_s, sums = [], [], []
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    with ClockSampler(0) as clocks:
        for _ in range(reps):
            with torch.cuda.stream(stream):
                ev[0].record(stream)
                begin()
                ev[1].record(stream)
                for _ in range(FW_STEPS):
                    graph.replay()
                acc_h.copy_(acc, non_blocking=True)
                ev[2].record(stream)
            ev[2].synchronize()
            prefill_s.append(ev[0].elapsed_time(ev[1]) * 1e-3)
            decode_s.append(ev[1].elapsed_time(ev[2]) * 1e-3)
            sums.append(int(acc_h.numpy().view(np.uint64)[0]))
    ctx.sync()
    med = sorted(range(reps), key=lambda i: decode_s[i])[reps // 2]
    dsec, psec = decode_s[med], prefill_s[med]
    # KV present at step g: the prefix plus min(g + 1, window) ring tokens
    total_bytes = sum(fixed_work_step_bytes(cfg, FW_PREFIX + min(g + 1, cfg.window))
                      for g in range(FW_STEPS))
    step_bytes = total_bytes // FW_STEPS
    gbs = total_bytes / dsec / 1e9
    peak, peak_kind = peak_hbm()
    res = {"metric": FW_METRIC, "value": round(FW_STEPS / dsec, 1), "unit": "tok/s", "n_gpus": 1,
           "steps": reps, "warmup": 1, "ms_per_step": round(dsec / FW_STEPS * 1e3, 4),
           "higher_is_better": True, "scaling": "none (one sequence)", "vs_baseline": None,
           "dtype": "int8-act", "data": "synthetic (seeded; random-init weights)",
           "config": {"workload": "fixed_work_decoder", "prefix_tokens": FW_PREFIX,
                      "decode_steps": FW_STEPS, "layers": cfg.layers, "hidden": cfg.hidden,
                      "experts": cfg.experts, "top_k": cfg.top_k, "vocab": cfg.vocab,
                      "lm_head": "q8", "mode": "DynamicActivations", "cuda_graph": "decode step",
                      "l2": f"{step_bytes / 1e6:.0f} MB read per step (> 126 MB L2)"},
           "prefill_seconds": round(psec, 5), "decode_with_checksum_seconds": round(dsec, 5),
           "prefill_tok_s": round(FW_PREFIX / psec, 1),
           "repetitions": [{"prefill_s": round(p, 5), "decode_s": round(d, 5)}
                           for p, d in zip(prefill_s, decode_s)],
           "logits_checksum": sums[med], "checksums_equal": len(set(sums)) == 1,
           "e2e": {"value": round(FW_STEPS / dsec, 1), "unit": "tok/s",
                   "h2d_bytes_per_step": FW_PREFIX * cfg.hidden * 4 + FW_STEPS * 8,
                   "d2h_bytes_per_step": 8,
                   "note": "a step is a whole repetition: embeddings and token ids in, "
                           "checksum out"},
           "roofline": {"bound": "hbm", "kernel": "whole decode step (attention, MoE, projections, "
                                                "lm_head)",
                        "achieved": round(gbs, 2), "peak": peak, "peak_kind": peak_kind,
                        "unit": "GB/s", "frac": round(gbs / peak, 4), "traffic": None},
           # the timed repetitions' decode replays (the eager prefills' launches are
           # not counted)
           "gpu_launches": _launches(per_replay, FW_STEPS * reps), "clocks": clocks.summary(),
           "reference_published": {"decode_with_checksum_seconds": 4.031535, "tok_s": 127.0,
                                   "hardware": "M4 Pro, 8 threads"}}
    del graph
    state.free()
    if not args.no_cpu:
        res["cpu_baseline"] = decode_cpu_baseline(min(args.cpu_seconds, 8.0), prefix=FW_PREFIX,
                                                  mode=1, head=True)
    return res


# ---------------------------------------------------------------------------
# Default workload: the 12-layer decoder's MoE layer at decode with its routed
# experts split over the GPUs (expert parallelism), rows exchanged through
# NVLink peer memory by the library's own kernels (uocr_ep_*).
EPP_TOKENS = 64          # decode batch per rank (weak scaling: fixed per GPU)
EPP_METRIC = "decode tok/s (MoE decoder layer, expert-parallel, 64 tokens per GPU)"
EPP_MIN_TIMED_S = 0.6    # timed region at least this long (clock samples)


def cpu_model():
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for line in out.splitlines():
            if line.startswith("Model name:"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return None


def epp_weights(dev, ctx, layer_index, expert_ids):
    """Deterministic weights of one layer: every matrix seeded by (layer,
    expert, projection), so that any rank builds the same expert."""
    import torch

    import uocr_q8

    def mat(seed, r, c):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        w = torch.randint(-127, 128, (r, c), dtype=torch.int8, device=dev, generator=g)
        sc = torch.rand((r, (c + 31) // 32), device=dev, generator=g) * (1e-2 - 1e-4) + 1e-4
        return uocr_q8.Int8Matrix.from_device(r, c, w, sc.float().contiguous(), ctx)

    base = 100000 * (layer_index + 1)
    shared = [mat(base + i, *rc) for i, rc in enumerate(((FS, H), (FS, H), (H, FS)))]
    experts = [[mat(base + 10 * (e + 1) + i, *rc) for i, rc in enumerate(((F, H), (F, H), (H, F)))]
               for e in expert_ids]
    return shared, experts


def epp_cpu_baseline(seconds, mode=0):
    """The reference's scalar path (oracle port) on a bounded sample: batches
    of 64 tokens through one MoE layer, on all host threads and on one."""
    import oracle
    shared, routed, rng = make_cpu_layer(7)
    x = rng.standard_normal((EPP_TOKENS, H)).astype(np.float32)
    lg = rng.standard_normal((EPP_TOKENS, E)).astype(np.float32)
    out = {}
    for threads, budget in ((0, seconds), (1, seconds / 2)):
        oracle.set_threads(threads)
        n, t0 = 0, time.perf_counter()
        while n == 0 or time.perf_counter() - t0 < budget:
            oracle.experts(shared, routed, lg, x, TOPK, mode)
            n += 1
        dt = time.perf_counter() - t0
        out[threads] = (EPP_TOKENS * n / dt, n, dt, oracle.get_threads())
    oracle.set_threads(0)
    v, n, dt, cores = out[0]
    v1, n1, dt1, _ = out[1]
    return {"value": round(v, 2), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n} batches of 64 tokens through one MoE layer in {dt:.1f} s "
                      "(scalar restatement of the reference's Rust path; the crate cannot be "
                      "built here)",
            "single_thread": {"value": round(v1, 2), "unit": "tok/s", "cores": 1,
                              "sample": f"{n1} batches in {dt1:.1f} s"},
            "cpu_model": cpu_model(), "nproc": os.cpu_count()}


def run_ep_peer(args):
    """The MoE layer of the 12-layer decoder (64 routed experts of width 896,
    top-6, shared expert of width 1792, hidden 1280) at decode: every rank
    brings a batch of 64 tokens (weak scaling) and holds a contiguous block of
    the routed experts plus the shared expert; one layer forward = route,
    dispatch of the (token, expert) rows into the owners' memory over NVLink,
    the owners' grouped SwiGLU experts, return of the outputs, ordered
    combine.  A bench step replays a CUDA graph of R consecutive layer
    forwards (distinct layers rotated so that every layer's weights come from
    HBM), R chosen so that the K timed steps last at least 0.6 s."""
    import datetime
    import math

    import torch
    import torch.distributed as dist

    import uocr_q8
    from uocr_q8.expert_parallel import expert_bounds, peer_expert_parallel
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(dev))
    ctx = uocr_q8.GpuContext(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    mode = args.ep_mode
    bounds = expert_bounds(E, world)
    mine = list(range(bounds[rank], bounds[rank + 1]))
    per_rank_weight_bytes = len(mine) * EP_EXPERT_BYTES + EP_SHARED_BYTES
    n_layers = max(2, math.ceil(3 * 126e6 / per_rank_weight_bytes))  # > L2 between reuses
    T = EPP_TOKENS
    layers, eps = [], []
    with torch.cuda.stream(stream):
        for li in range(n_layers):
            shared, experts = epp_weights(dev, ctx, li, mine)
            layer = uocr_q8.MoeLayer(ctx, shared, experts, top_k=1)
            layers.append(layer)
            if world > 1:
                ep = peer_expert_parallel(ctx, layer, E, TOPK, T)
            else:
                ep = uocr_q8.PeerExpertParallel(ctx, layer, E, TOPK, bounds, 0, T)
                uocr_q8.PeerExpertParallel.connect_local([ep])
            ep.set_wait_limit(5.0)
            eps.append(ep)
    torch.cuda.synchronize()
    gen = torch.Generator(device=dev)
    gen.manual_seed(555 + rank)
    n_in = 8
    xs = torch.randn((n_in, T, H), device=dev, generator=gen)
    lg = torch.randn((n_in, T, E), device=dev, generator=gen)
    ys = torch.empty((n_in, T, H), device=dev)

    def step(i):
        eps[i % n_layers].forward_device(xs[i % n_in], lg[i % n_in], mode, ys[i % n_in])

    if world > 1:
        dist.barrier()
    n_warm = max(args.warmup, 3) + n_layers
    with torch.cuda.stream(stream):
        for i in range(n_warm):
            if i == n_warm - 1:  # one eager forward in an NVTX range, for a profiler's launch list
                torch.cuda.nvtx.range_push("ep_layer_forward")
            step(i)
            if i == n_warm - 1:
                torch.cuda.nvtx.range_pop()
    ctx.sync()

    # parity of one step of every rank against the single-GPU layer (all 64
    # experts) on rank 0's tokens: FP32 activations within the FP32 layer
    # tolerance, int8 activations bit for bit
    parity = {}
    for pm in (0, 2):
        if world > 1:
            dist.barrier()
        y_ep = torch.empty((T, H), device=dev)
        with torch.cuda.stream(stream):
            eps[0].forward_device(xs[0], lg[0], pm, y_ep)
        ctx.sync()
        if rank == 0:
            with torch.cuda.stream(stream):
                shared, experts = epp_weights(dev, ctx, 0, range(E))
                full = uocr_q8.MoeLayer(ctx, shared, experts, TOPK)
                y_ref = full.forward_device(xs[0], lg[0], pm)
            ctx.sync()
            a, b = y_ep.cpu().numpy(), y_ref.cpu().numpy()
            same = float(np.mean(a.view(np.uint32) == b.view(np.uint32)))
            rel = float(np.max(np.abs(a.astype(np.float64) - b)) / max(np.max(np.abs(b)), 1e-30))
            parity[f"mode{pm}"] = {"bit_identical": round(same, 6), "max_rel_diff": rel,
                                   "ok": bool(same == 1.0 if pm else rel <= 1e-4)}
            full.free()
            del shared, experts, full
    if world > 1:
        dist.barrier()

    # R layer forwards per bench step, from the measured time of one forward
    probe = torch.cuda.CUDAGraph()
    with torch.cuda.graph(probe, stream=stream):
        for i in range(n_layers):
            step(i)
    for _ in range(2):
        probe.replay()
    torch.cuda.synchronize()
    t0e, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0e.record(stream)
        for _ in range(4):
            probe.replay()
        t1e.record(stream)
    t1e.synchronize()
    t_layer = t0e.elapsed_time(t1e) * 1e-3 / (4 * n_layers)
    tl = torch.tensor([t_layer], device=dev)
    if world > 1:
        dist.all_reduce(tl, op=dist.ReduceOp.MAX)
    t_layer = float(tl.item())
    K = max(1, args.steps)
    R = n_layers * max(1, math.ceil(EPP_MIN_TIMED_S / (K * t_layer * n_layers)))
    R = min(R, n_layers * 4096)
    del probe
    graph = kept_graph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(R):
            step(i)
    per_replay = graph_launches(graph)
    warm = max(args.warmup, 3)
    for _ in range(warm):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(K):
                graph.replay()
            stop.record(stream)
        stop.synchronize()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop)
    ctx.sync()
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    forwards = K * R
    value = world * T * forwards / (ms * 1e-3)
    us_layer = ms * 1e3 / forwards
    del graph

    # end to end: pinned host x / logits in, y out, through uocr_ep_forward_host
    hx = torch.empty((n_in, T, H), pin_memory=True)
    hl = torch.empty((n_in, T, E), pin_memory=True)
    hy = torch.empty((n_in, T, H), pin_memory=True)
    hx.copy_(xs.cpu())
    hl.copy_(lg.cpu())
    e2e_steps = max(n_layers, min(args.e2e_steps, int(2.0 / max(t_layer, 1e-6)) // n_layers * n_layers))
    for i in range(n_layers):
        eps[i].forward_host_ptrs(hx[0].data_ptr(), hl[0].data_ptr(), T, hy[0].data_ptr(), mode)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        j = i % n_in
        eps[i % n_layers].forward_host_ptrs(hx[j].data_ptr(), hl[j].data_ptr(), T,
                                            hy[j].data_ptr(), mode)
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te.item())
    e2e = world * T * e2e_steps / e2e_s

    peak, peak_kind = peak_hbm()
    step_bytes = per_rank_weight_bytes + T * (H + E + H) * 4
    achieved = step_bytes / (us_layer * 1e-6) / 1e9
    result = None
    if rank == 0:
        result = {
            "metric": EPP_METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
            "steps": K, "warmup": warm, "ms_per_step": round(ms / K, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp32" if mode == 0 else "int8-act",
            "data": "synthetic (seeded; x ~ N(0,1), router logits ~ N(0,1), int8 weights "
                    "uniform in [-127,127], scales ~ U(1e-4,1e-2))",
            "config": {"workload": "moe_layer_ep_decode", "tokens_per_gpu": T,
                       "global_batch": world * T, "hidden": H, "experts": E, "top_k": TOPK,
                       "experts_per_gpu": len(mine), "expert_width": F, "shared_width": FS,
                       "mode": {0: "weights_only (fp32 activations)", 1: "dynamic activations",
                                2: "dynamic int8 activations, every row"}[mode],
                       "parallelism": f"ep{world} (routed experts split, rows exchanged by "
                                      "stores into peer memory over NVLink; no collective)",
                       "step": f"one CUDA-graph replay of {R} consecutive layer forwards",
                       "layer_forwards_per_step": R, "us_per_layer_forward": round(us_layer, 3),
                       "l2": f"rotating pool of {n_layers} layers x "
                             f"{per_rank_weight_bytes / 1e6:.1f} MB per GPU (> 126 MB L2)"},
            "e2e": {"value": round(e2e, 1), "unit": "tok/s", "steps": e2e_steps,
                    "us_per_step": round(e2e_s / e2e_steps * 1e6, 2),
                    "api": "uocr_ep_forward_host (one layer forward per call)",
                    "h2d_bytes_per_step": T * (H + E) * 4, "d2h_bytes_per_step": T * H * 4},
            "roofline": {"bound": "hbm",
                         "kernel": "one layer forward (all its launches: route, dispatch, "
                                   "small_rows_kernel gate/up and down, splits, return, "
                                   "combine); algorithmic bytes = this GPU's expert and "
                                   "shared weights + x, logits, y",
                         "achieved": round(achieved, 2), "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                         "bytes_per_layer_forward": step_bytes},
            "ep_parity": parity,
            # route, dispatch, wait, grouping, split, small-rows gate/up (+ tensor-core
            # gate, up, big-counts when a group can exceed 64 rows), SwiGLU split,
            # small-rows down (+ tensor-core down), un-permute, return, shared
            # expert (split, gate/up, SwiGLU split, down), combine
            "gpu_launches": _launches(per_replay, K),
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu:
            result["cpu_baseline"] = epp_cpu_baseline(args.cpu_seconds, mode)
    for ep in eps:
        ep.free()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def run_ep_emulated(args):
    """Profiling aid, one GPU: the expert-parallel layer of R ranks emulated on
    one device (R contexts' worth of buffers, one stream), every step driven
    through the three-part API in the order dispatch(all ranks),
    experts(all ranks), combine(all ranks), so that the kernels of all ranks
    run serialised and no wait depends on work queued behind it.  The time
    per step is the sum over the ranks (it is not a multi-GPU number)."""
    import torch

    import uocr_q8
    from uocr_q8.expert_parallel import expert_bounds
    W, T, mode = args.emulate_ranks, EPP_TOKENS, args.ep_mode
    torch.cuda.set_device(0)
    dev = "cuda:0"
    ctx = uocr_q8.GpuContext(0)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    bounds = expert_bounds(E, W)
    with torch.cuda.stream(stream):
        shared, experts = epp_weights(dev, ctx, 0, range(E))
        locs = [uocr_q8.MoeLayer(ctx, shared, experts[bounds[r]:bounds[r + 1]], top_k=1)
                for r in range(W)]
        eps = [uocr_q8.PeerExpertParallel(ctx, locs[r], E, TOPK, bounds, r, T) for r in range(W)]
        uocr_q8.PeerExpertParallel.connect_local(eps)
        gen = torch.Generator(device=dev)
        gen.manual_seed(77)
        xs = torch.randn((W, T, H), device=dev, generator=gen)
        lg = torch.randn((W, T, E), device=dev, generator=gen)
        ys = torch.empty((W, T, H), device=dev)

    def step():
        for r in range(W):
            eps[r].dispatch_device(xs[r], lg[r], mode, ys[r])
        for r in range(W):
            eps[r].experts_device()
        for r in range(W):
            eps[r].combine_device(ys[r])

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step()
    ctx.sync()
    steps = max(1, args.steps)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(steps):
            step()
        t1.record(stream)
    t1.synchronize()
    ctx.sync()
    us = t0.elapsed_time(t1) * 1e3 / steps
    for ep in eps:
        ep.free()
    return {"metric": f"emulated expert-parallel MoE layer, {W} ranks on one GPU (profiling aid)",
            "value": round(us, 2), "unit": "us per step (all ranks, serialised)", "n_gpus": 1,
            "steps": steps, "higher_is_better": False, "emulated_ranks": W,
            "us_per_rank_step": round(us / W, 2), "tokens_per_rank": T, "mode": mode}


def run_secondary(args):
    """Every other configuration, bounded, on GPU 0 (one GPU runs only)."""
    import copy
    out = {}

    def sub(name, fn, **over):
        a = copy.copy(args)
        for k, v in over.items():
            setattr(a, k, v)
        t0 = time.perf_counter()
        try:
            r = fn(a)
            r["wall_s"] = round(time.perf_counter() - t0, 1)
            out[name] = r
        except Exception as exc:  # a secondary never hides the headline line
            out[name] = {"error": f"{type(exc).__name__}: {exc}"}

    sub("moe_decode_layer_1_token", run_ours, steps=4096, e2e_steps=4000,
        cpu_seconds=min(args.cpu_seconds, 6.0))
    sub("gemv_stream_fp32", run_gemv, steps=256 * 4096, gemv_int8=False)
    sub("gemv_stream_int8", run_gemv, steps=256 * 4096, gemv_int8=True)
    sub("prefill_1024_fp32", run_prefill, steps=40, prefill_mode=0)
    sub("prefill_1024_int8", run_prefill, steps=40, prefill_mode=2)
    sub("int8_micro_suite", run_int8suite)
    sub("attention_decode", run_attn, steps=200, cpu_seconds=min(args.cpu_seconds, 5.0))
    sub("decode_step_12_layers", run_decode, steps=60, cpu_seconds=min(args.cpu_seconds, 6.0),
        lm_head="bf16")
    sub("fixed_work_decoder", run_fixed_work, steps=3, cpu_seconds=min(args.cpu_seconds, 6.0))
    return out


def run_reference_ep(args):
    """The reference's scalar CPU path (oracle port, all host threads) on the
    default workload: each step one batch of 64 tokens through one MoE layer;
    rank 0 alone runs it."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    import oracle
    oracle.set_threads(0)
    shared, routed, rng = make_cpu_layer(7)
    xs = rng.standard_normal((4, EPP_TOKENS, H)).astype(np.float32)
    lgs = rng.standard_normal((4, EPP_TOKENS, E)).astype(np.float32)
    for i in range(max(args.warmup, 3)):
        oracle.experts(shared, routed, lgs[i % 4], xs[i % 4], TOPK, args.ep_mode)
    steps = args.steps if args.ref_steps is None else args.ref_steps
    t0 = time.perf_counter()
    for i in range(steps):
        oracle.experts(shared, routed, lgs[i % 4], xs[i % 4], TOPK, args.ep_mode)
    dt = time.perf_counter() - t0
    v = EPP_TOKENS * steps / dt
    cores = oracle.get_threads()
    return {"impl": "reference", "metric": EPP_METRIC, "value": round(v, 2), "unit": "tok/s",
            "n_gpus": world, "steps": steps, "warmup": max(args.warmup, 3),
            "ms_per_step": round(dt / steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "fp32" if args.ep_mode == 0 else "int8-act",
            "data": "synthetic (seeded; same distributions as the GPU arm)",
            "config": {"workload": "moe_layer_ep_decode", "tokens_per_gpu": EPP_TOKENS,
                       "hidden": H, "experts": E, "top_k": TOPK, "expert_width": F,
                       "shared_width": FS, "parallelism": "rank 0 only (host CPU)",
                       "step": "one batch of 64 tokens through one MoE layer"},
            "cpu_baseline": {"value": round(v, 2), "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"{steps} batches of 64 tokens through one MoE layer "
                                       "(scalar restatement of the reference's Rust path; the "
                                       "Rust crate cannot be built here)",
                             "cpu_model": cpu_model()},
            "e2e": {"value": round(v, 2), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--graph-steps", type=int, default=256)
    ap.add_argument("--e2e-steps", type=int, default=4000)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-steps", type=int, default=None)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="default workload only (skip the one-GPU secondary configurations)")
    ap.add_argument("--traffic", type=float, default=None,
                    help="dram bytes per launch from an ncu capture (roofline.traffic); "
                         "defaults to the committed capture of the workload's kernel")
    ap.add_argument("--workload",
                    choices=["ep_peer", "moe_decode", "gemv", "prefill", "int8suite", "ep_decode",
                             "attn_decode", "decode_step", "fixed_work", "decode_step_ep"],
                    default="ep_peer")
    ap.add_argument("--gemv-int8", action="store_true")
    ap.add_argument("--prefill-mode", type=int, choices=[0, 2], default=0)
    ap.add_argument("--ep-mode", type=int, choices=[0, 1, 2], default=0)
    ap.add_argument("--decode-mode", type=int, choices=[0, 2], default=0)
    ap.add_argument("--lm-head", choices=["q8", "bf16"], default="q8")
    ap.add_argument("--emulate-ranks", type=int, default=0,
                    help="profiling aid: run the expert-parallel layer of this many ranks "
                         "emulated on GPU 0 (serialised), print its time per step")
    args = ap.parse_args()
    if args.impl == "reference":
        if args.workload == "ep_peer":
            res = run_reference_ep(args)
        else:
            if args.ref_steps is None:
                args.ref_steps = min(args.steps, 1500)
            res = run_reference(args)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if args.emulate_ranks > 1:
        print(json.dumps(run_ep_emulated(args)), flush=True)
        return
    single = {"gemv": run_gemv, "prefill": run_prefill, "decode_step": run_decode,
              "attn_decode": run_attn, "int8suite": run_int8suite, "fixed_work": run_fixed_work}
    if args.workload in single:
        print(json.dumps(single[args.workload](args)), flush=True)
        return
    if args.workload == "ep_decode":
        res = run_ep(args)
    elif args.workload == "decode_step_ep":
        res = run_decode_ep(args)
    elif args.workload == "moe_decode":
        res = run_ours(args)
    else:
        res = run_ep_peer(args)
        world = int(os.environ.get("WORLD_SIZE", "1"))
        if res is not None and world == 1 and not args.no_secondary:
            res["secondary"] = run_secondary(args)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
