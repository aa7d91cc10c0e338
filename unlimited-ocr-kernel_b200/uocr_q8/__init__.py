"""uocr_q8 — Python front end of the B200 q8-block32 library (libuocr_q8.so).

Mirrors the reference's operator surface (Rust crate `uocr`):

* ``Int8Matrix`` — ``from_parts``, ``quantize``, ``dequantize``,
  ``storage_bytes``, ``linear``, ``linear_dynamic_int8``
  (src/cpu/quantized.rs:11-237);
* ``QuantizationMode`` (src/cpu/quantized.rs:242-247);
* ``GpuContext`` — stands where ``CpuContext`` stands (src/cpu/mod.rs:18-79):
  the device, the scratch limit and the stream every call runs on;
* ``route`` (src/decoder/moe.rs:7-30) and ``MoeLayer`` — ``Decoder::experts``
  (src/decoder/mod.rs:124-220);
* ``QuantizedWeights`` — the ``uocr-q8-block32-v1`` overlay loader
  (src/cpu/quantized.rs:305-369), in ``uocr_q8.overlay``.

Errors raise ``OcrError`` whose ``kind`` is the reference's OcrError variant
name.  Host methods take and return numpy arrays (Tensor in, Tensor out);
``*_device`` methods take torch CUDA tensors and run asynchronously on the
context's stream.  Every compute call goes to the CUDA library; nothing here
computes on the CPU.
"""
from __future__ import annotations

import ctypes
import enum
from typing import Optional, Sequence

import numpy as np

from . import _lib
from ._lib import LibraryMissing

BLOCK = 32

_KINDS = {1: "Io", 2: "Json", 3: "Format", 4: "Shape", 5: "Unsupported", 6: "Resource",
          7: "Numerical", 8: "Cuda", 9: "Nccl", 10: "Timeout", 11: "Invalid"}


class OcrError(RuntimeError):
    """A failed call; ``kind`` names the reference's OcrError variant."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{_KINDS.get(code, code)}: {message}")
        self.code = code
        self.kind = _KINDS.get(code, "Unknown")
        self.message = message


def _check(code: int) -> None:
    if code:
        L = _lib.load()
        raise OcrError(code, L.uocr_last_error().decode(errors="replace"))


def lib():
    return _lib.load()


class QuantizationMode(enum.IntEnum):
    WEIGHTS_ONLY = 0
    DYNAMIC_ACTIVATIONS = 1
    DYNAMIC_ROWWISE = 2  # extension: int8 activations for every row


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _tptr(t) -> int:
    return int(t.data_ptr())


class GpuContext:
    """Device, scratch limit and stream of a sequence of calls.

    The device-tensor methods take torch tensors, so by default the context
    runs on torch's current stream of its device (torch's caching allocator
    may reuse a freed tensor's memory for work on that stream at once); pass
    ``torch_stream=False`` to keep the library's own stream, then order it
    against torch's with events or ``sync()``."""

    def __init__(self, device: int = 0, scratch_limit: int = 1 << 34, torch_stream: bool = True):
        h = ctypes.c_void_p()
        _check(lib().uocr_ctx_create(int(device), int(scratch_limit), ctypes.byref(h)))
        self._h = h
        self.device = int(device)
        self.scratch_limit = int(scratch_limit)
        if torch_stream:
            try:
                import torch
                if torch.cuda.is_available():
                    self.set_stream(torch.cuda.current_stream(self.device))
            except ImportError:
                pass

    @property
    def handle(self):
        return self._h

    def set_stream(self, stream) -> None:
        """Run on a torch.cuda.Stream (or a raw cudaStream_t int)."""
        raw = getattr(stream, "cuda_stream", stream)
        _check(lib().uocr_ctx_set_stream(self._h, ctypes.c_void_p(int(raw))))

    def sync(self) -> None:
        _check(lib().uocr_ctx_sync(self._h))

    def set_wait_limit(self, seconds: float) -> None:
        """Bounded device waits of this context's kernels give up after
        `seconds` (0: the default, about 2 s) and report Timeout."""
        _check(lib().uocr_ctx_set_wait_limit(self._h, int(seconds * 1e9)))

    def hold_decode_barrier(self, hold: bool) -> None:
        """Failure-detection test hook: the one-token decode kernel's grid
        barrier waits for an arrival that never comes until released."""
        _check(lib().uocr_ctx_hold_decode_barrier(self._h, int(bool(hold))))

    def sm_count(self) -> int:
        d, s = ctypes.c_int(), ctypes.c_int()
        _check(lib().uocr_ctx_device(self._h, ctypes.byref(d), ctypes.byref(s)))
        return s.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().uocr_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default_ctx = {}


def default_context(device: int = 0) -> GpuContext:
    if device not in _default_ctx:
        _default_ctx[device] = GpuContext(device)
    return _default_ctx[device]


class Int8Matrix:
    """Device-resident q8-block32 matrix (src/cpu/quantized.rs:11-16)."""

    def __init__(self, handle, ctx: GpuContext, keepalive=None, owned: bool = True):
        self._h = handle
        self.ctx = ctx
        self._keep = keepalive
        self._owned = owned  # False: a view owned by a QuantizedWeights overlay
        r, c = ctypes.c_size_t(), ctypes.c_size_t()
        _check(lib().uocr_q8_shape(self._h, ctypes.byref(r), ctypes.byref(c)))
        self.rows, self.cols = r.value, c.value

    # -- constructors -----------------------------------------------------
    @classmethod
    def from_parts(cls, rows: int, cols: int, weights, scales,
                   ctx: Optional[GpuContext] = None) -> "Int8Matrix":
        ctx = ctx or default_context()
        w = np.ascontiguousarray(weights, dtype=np.int8).reshape(-1)
        s = np.ascontiguousarray(scales, dtype=np.float32).reshape(-1)
        h = ctypes.c_void_p()
        _check(lib().uocr_q8_from_parts(ctx.handle, rows, cols, _ptr(w), w.size, _ptr(s), s.size,
                                        ctypes.byref(h)))
        return cls(h, ctx)

    @classmethod
    def quantize(cls, matrix, ctx: Optional[GpuContext] = None) -> "Int8Matrix":
        ctx = ctx or default_context()
        x = np.ascontiguousarray(matrix, dtype=np.float32)
        if x.ndim != 2:
            raise OcrError(4, "invalid tensor shape: quantization expects a nonempty matrix")
        h = ctypes.c_void_p()
        _check(lib().uocr_q8_quantize(ctx.handle, x.shape[0], x.shape[1], _ptr(x),
                                      ctypes.byref(h)))
        return cls(h, ctx)

    @classmethod
    def from_device(cls, rows: int, cols: int, weights_t, scales_t,
                    ctx: Optional[GpuContext] = None) -> "Int8Matrix":
        """Borrow torch CUDA tensors (int8 rows*cols, float32 rows*blocks)."""
        ctx = ctx or default_context()
        h = ctypes.c_void_p()
        _check(lib().uocr_q8_from_device(ctx.handle, rows, cols, ctypes.c_void_p(_tptr(weights_t)),
                                         ctypes.c_void_p(_tptr(scales_t)), ctypes.byref(h)))
        return cls(h, ctx, keepalive=(weights_t, scales_t))

    # -- properties -------------------------------------------------------
    @property
    def handle(self):
        return self._h

    def storage_bytes(self) -> int:
        return int(lib().uocr_q8_storage_bytes(self._h))

    def download(self):
        w = np.empty((self.rows, self.cols), np.int8)
        s = np.empty((self.rows, (self.cols + BLOCK - 1) // BLOCK), np.float32)
        _check(lib().uocr_q8_download(self.ctx.handle, self._h, _ptr(w), _ptr(s)))
        return w, s

    def device_ptrs(self):
        w, s = ctypes.c_void_p(), ctypes.c_void_p()
        _check(lib().uocr_q8_device_ptrs(self._h, ctypes.byref(w), ctypes.byref(s)))
        return w.value, s.value

    # -- reference operations (host tensors) --------------------------------
    def dequantize(self) -> np.ndarray:
        out = np.empty((self.rows, self.cols), np.float32)
        _check(lib().uocr_q8_dequantize_host(self.ctx.handle, self._h, _ptr(out), out.size))
        return out

    def _host_call(self, fn, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        shape = (ctypes.c_size_t * max(x.ndim, 1))(*x.shape)
        out_shape = tuple(x.shape[:-1]) + (self.rows,) if x.ndim else (self.rows,)
        y_len = int(np.prod(out_shape)) if x.ndim and x.shape[-1] == self.cols else 0
        y = np.empty((max(y_len, 1),), np.float32)
        _check(fn(self.ctx.handle, self._h, _ptr(x), shape, x.ndim, _ptr(y), y_len))
        return y[:y_len].reshape(out_shape)

    def linear(self, x) -> np.ndarray:
        return self._host_call(lib().uocr_q8_linear_host, x)

    def linear_dynamic_int8(self, x) -> np.ndarray:
        return self._host_call(lib().uocr_q8_linear_dynamic_int8_host, x)

    # -- device forms (torch CUDA tensors, asynchronous) ---------------------
    def linear_device(self, x_t, y_t=None, dynamic: bool = False):
        import torch
        batch = x_t.numel() // self.cols
        if y_t is None:
            y_t = torch.empty((batch, self.rows), dtype=torch.float32, device=x_t.device)
        fn = lib().uocr_q8_linear_dynamic_int8 if dynamic else lib().uocr_q8_linear
        _check(fn(self.ctx.handle, self._h, ctypes.c_void_p(_tptr(x_t)), batch,
                  ctypes.c_void_p(_tptr(y_t))))
        return y_t

    def dequantize_device(self, out_t=None):
        import torch
        if out_t is None:
            out_t = torch.empty((self.rows, self.cols), dtype=torch.float32,
                                device=f"cuda:{self.ctx.device}")
        _check(lib().uocr_q8_dequantize(self.ctx.handle, self._h, ctypes.c_void_p(_tptr(out_t))))
        return out_t

    def free(self) -> None:
        if getattr(self, "_h", None):
            if getattr(self, "_owned", True):
                lib().uocr_q8_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def quantize_rows_device(ctx: GpuContext, x_t, q_t=None, s_t=None):
    import torch
    rows, cols = x_t.shape
    nb = (cols + BLOCK - 1) // BLOCK
    q_t = q_t if q_t is not None else torch.empty((rows, cols), dtype=torch.int8, device=x_t.device)
    s_t = s_t if s_t is not None else torch.empty((rows, nb), dtype=torch.float32, device=x_t.device)
    _check(lib().uocr_q8_quantize_rows(ctx.handle, ctypes.c_void_p(_tptr(x_t)), rows, cols,
                                       ctypes.c_void_p(_tptr(q_t)), ctypes.c_void_p(_tptr(s_t))))
    return q_t, s_t


def linear_multi_device(ctx: GpuContext, mats: Sequence[Int8Matrix], x_t, ys: Sequence,
                        mode: int = QuantizationMode.WEIGHTS_ONLY) -> None:
    n = len(mats)
    mh = (ctypes.c_void_p * n)(*[m.handle.value for m in mats])
    yh = (ctypes.c_void_p * n)(*[_tptr(y) for y in ys])
    _check(lib().uocr_q8_linear_multi(ctx.handle, mh, n, int(mode), ctypes.c_void_p(_tptr(x_t)),
                                      yh))


def route_device(ctx: GpuContext, logits_t, top_k: int, normalize: bool = False,
                 scale: float = 1.0):
    """moe::route for every row of logits (torch CUDA tensor [tokens, experts])."""
    import torch
    tokens, n = logits_t.shape
    ids = torch.empty((tokens, top_k), dtype=torch.int32, device=logits_t.device)
    wts = torch.empty((tokens, top_k), dtype=torch.float32, device=logits_t.device)
    _check(lib().uocr_moe_route(ctx.handle, ctypes.c_void_p(_tptr(logits_t)), tokens, n, top_k,
                                int(bool(normalize)), float(scale), ctypes.c_void_p(_tptr(ids)),
                                ctypes.c_void_p(_tptr(wts))))
    return ids, wts


def combine_device(ctx: GpuContext, ids_t, wts_t, pair_out_t, y_t):
    """y[t] += wts[t, j] * pair_out[t * top_k + j] over t's pairs in ascending
    expert id (the combine of src/decoder/mod.rs:208-217).  Asynchronous."""
    tokens, top_k = ids_t.shape
    _check(lib().uocr_moe_combine(ctx.handle, ctypes.c_void_p(_tptr(ids_t)),
                                  ctypes.c_void_p(_tptr(wts_t)),
                                  ctypes.c_void_p(_tptr(pair_out_t)), tokens, top_k,
                                  y_t.shape[1], ctypes.c_void_p(_tptr(y_t))))
    return y_t


def dispatch_device(ctx: GpuContext, x_t, ids_t, rank_bounds: Sequence[int], capacity: int,
                    send_x_t=None, send_ids_t=None, pair_rows_t=None):
    """Fixed-capacity dispatch of (token, expert) pairs to the ranks owning
    the experts (uocr_moe_dispatch).  Returns (send_x [world * capacity,
    hidden], send_ids [world * capacity], pair_rows [tokens * top_k])."""
    import torch
    tokens, hidden = x_t.shape
    top_k = ids_t.shape[1]
    world = len(rank_bounds) - 1
    dev = x_t.device
    if send_x_t is None:
        send_x_t = torch.empty((world * capacity, hidden), dtype=torch.float32, device=dev)
    if send_ids_t is None:
        send_ids_t = torch.empty((world * capacity,), dtype=torch.int32, device=dev)
    if pair_rows_t is None:
        pair_rows_t = torch.empty((tokens * top_k,), dtype=torch.int32, device=dev)
    bounds = (ctypes.c_int32 * (world + 1))(*rank_bounds)
    _check(lib().uocr_moe_dispatch(ctx.handle, ctypes.c_void_p(_tptr(x_t)), tokens, hidden,
                                   ctypes.c_void_p(_tptr(ids_t)), top_k, bounds, world, capacity,
                                   ctypes.c_void_p(_tptr(send_x_t)),
                                   ctypes.c_void_p(_tptr(send_ids_t)),
                                   ctypes.c_void_p(_tptr(pair_rows_t))))
    return send_x_t, send_ids_t, pair_rows_t


def combine_rows_device(ctx: GpuContext, ids_t, wts_t, rows_t, pair_rows_t, y_t):
    """uocr_moe_combine_rows: y[t] += w * rows[pair_rows[t * top_k + j]] in
    ascending expert id.  Asynchronous."""
    tokens, top_k = ids_t.shape
    _check(lib().uocr_moe_combine_rows(ctx.handle, ctypes.c_void_p(_tptr(ids_t)),
                                       ctypes.c_void_p(_tptr(wts_t)),
                                       ctypes.c_void_p(_tptr(rows_t)),
                                       ctypes.c_void_p(_tptr(pair_rows_t)), tokens, top_k,
                                       y_t.shape[1], ctypes.c_void_p(_tptr(y_t))))
    return y_t


class MoeLayer:
    """Decoder::experts over device-resident q8 FFNs (src/decoder/mod.rs:124-220)."""

    def __init__(self, ctx: GpuContext, shared: Sequence[Int8Matrix],
                 experts: Sequence[Sequence[Int8Matrix]], top_k: int,
                 normalize_topk: bool = False, routed_scale: float = 1.0):
        n = len(experts)
        arr = lambda i: (ctypes.c_void_p * n)(*[e[i].handle.value for e in experts])
        h = ctypes.c_void_p()
        _check(lib().uocr_moe_create(ctx.handle, shared[0].handle, shared[1].handle,
                                     shared[2].handle, arr(0), arr(1), arr(2), n, top_k,
                                     int(bool(normalize_topk)), float(routed_scale),
                                     ctypes.byref(h)))
        self._h = h
        self.ctx = ctx
        self._keep = (list(shared), [list(e) for e in experts])
        self.top_k = top_k
        self.n_experts = n
        self.hidden = shared[0].cols

    @property
    def handle(self):
        return self._h

    def forward(self, x, logits, mode: int = QuantizationMode.WEIGHTS_ONLY):
        """Host tensors in, host tensors out: (y, ids, weights)."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.hidden)
        logits = np.ascontiguousarray(logits, dtype=np.float32).reshape(x.shape[0], self.n_experts)
        t = x.shape[0]
        y = np.empty_like(x)
        ids = np.empty((t, self.top_k), np.int32)
        wts = np.empty((t, self.top_k), np.float32)
        _check(lib().uocr_moe_forward_host(self.ctx.handle, self._h, int(mode), _ptr(x),
                                           _ptr(logits), t, _ptr(y), _ptr(ids), _ptr(wts)))
        return y, ids, wts

    def forward_device(self, x_t, logits_t, mode: int = QuantizationMode.WEIGHTS_ONLY, y_t=None,
                       ids_t=None, wts_t=None):
        import torch
        t = x_t.shape[0]
        y_t = y_t if y_t is not None else torch.empty_like(x_t)
        ip = ctypes.c_void_p(_tptr(ids_t)) if ids_t is not None else None
        wp = ctypes.c_void_p(_tptr(wts_t)) if wts_t is not None else None
        _check(lib().uocr_moe_forward(self.ctx.handle, self._h, int(mode),
                                      ctypes.c_void_p(_tptr(x_t)), ctypes.c_void_p(_tptr(logits_t)),
                                      t, ctypes.c_void_p(_tptr(y_t)), ip, wp))
        return y_t

    def forward_decode_noalloc(self, x_t, logits_t, mode: int = QuantizationMode.WEIGHTS_ONLY,
                               y_t=None):
        """One token through the allocation-free entry point (fixed library
        scratch; see include/uocr_q8.h).  Asynchronous on the context stream."""
        import torch
        y_t = y_t if y_t is not None else torch.empty_like(x_t)
        _check(lib().uocr_moe_forward_decode_noalloc(
            self.ctx.handle, self._h, int(mode), ctypes.c_void_p(_tptr(x_t)),
            ctypes.c_void_p(_tptr(logits_t)), ctypes.c_void_p(_tptr(y_t))))
        return y_t

    def expert_rows_device(self, x_t, expert_ids_t, mode: int = QuantizationMode.WEIGHTS_ONLY,
                           out_t=None):
        """out[i] = FFN_{expert_ids[i]}(x[i]) for the layer's own experts (ids
        local to the layer); rows of one expert form one group.  Asynchronous."""
        import torch
        out_t = out_t if out_t is not None else torch.empty_like(x_t)
        _check(lib().uocr_moe_expert_rows(self.ctx.handle, self._h, int(mode),
                                          ctypes.c_void_p(_tptr(x_t)),
                                          ctypes.c_void_p(_tptr(expert_ids_t)), x_t.shape[0],
                                          ctypes.c_void_p(_tptr(out_t))))
        return out_t

    def shared_rows_device(self, x_t, mode: int = QuantizationMode.WEIGHTS_ONLY, y_t=None):
        """y = the shared expert's FFN of every row of x.  Asynchronous."""
        import torch
        y_t = y_t if y_t is not None else torch.empty_like(x_t)
        _check(lib().uocr_moe_shared_rows(self.ctx.handle, self._h, int(mode),
                                          ctypes.c_void_p(_tptr(x_t)), x_t.shape[0],
                                          ctypes.c_void_p(_tptr(y_t))))
        return y_t

    def forward_host_ptrs(self, x_ptr: int, logits_ptr: int, tokens: int, y_ptr: int,
                          mode: int = QuantizationMode.WEIGHTS_ONLY) -> None:
        """Raw host-pointer form (pinned buffers), for end-to-end timing."""
        _check(lib().uocr_moe_forward_host(self.ctx.handle, self._h, int(mode),
                                           ctypes.c_void_p(x_ptr), ctypes.c_void_p(logits_ptr),
                                           tokens, ctypes.c_void_p(y_ptr), None, None))

    def free(self) -> None:
        if getattr(self, "_h", None):
            lib().uocr_moe_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


EP_HANDLE_BYTES = 128


class PeerExpertParallel:
    """This GPU's end of a MoE layer whose routed experts are split over the
    GPUs of one node, rows moving as stores into peer memory (uocr_ep_*).

    ``local_layer`` holds the shared expert and experts
    ``[rank_bounds[rank], rank_bounds[rank + 1])`` of an ``n_experts`` layer
    (ids local to it); ``max_tokens`` bounds the tokens of one step on every
    rank.  After ``connect`` (the handles of all ranks, in rank order, from
    ``handle()`` on each) or ``connect_local`` (ranks of this process), every
    step gives each rank ``Decoder::experts`` of its own tokens."""

    def __init__(self, ctx: GpuContext, local_layer: "MoeLayer", n_experts: int, top_k: int,
                 rank_bounds: Sequence[int], rank: int, max_tokens: int,
                 normalize_topk: bool = False, routed_scale: float = 1.0):
        world = len(rank_bounds) - 1
        bounds = (ctypes.c_int32 * (world + 1))(*rank_bounds)
        h = ctypes.c_void_p()
        _check(lib().uocr_ep_create(ctx.handle, local_layer.handle, n_experts, top_k,
                                    int(bool(normalize_topk)), float(routed_scale), bounds, world,
                                    rank, max_tokens, ctypes.byref(h)))
        self._h = h
        self.ctx = ctx
        self.layer = local_layer
        self.world, self.rank = world, rank
        self.n_experts, self.top_k, self.max_tokens = n_experts, top_k, max_tokens
        self.hidden = local_layer.hidden

    @property
    def handle_ptr(self):
        return self._h

    def handle(self) -> bytes:
        buf = ctypes.create_string_buffer(EP_HANDLE_BYTES)
        _check(lib().uocr_ep_handle(self._h, buf))
        return buf.raw

    def connect(self, handles: Sequence[bytes]) -> None:
        blob = b"".join(bytes(h) for h in handles)
        if len(blob) != EP_HANDLE_BYTES * self.world:
            raise OcrError(4, f"invalid tensor shape: expected {self.world} handles")
        buf = ctypes.create_string_buffer(blob, len(blob))
        _check(lib().uocr_ep_connect(self._h, buf))

    @staticmethod
    def connect_local(eps: Sequence["PeerExpertParallel"]) -> None:
        arr = (ctypes.c_void_p * len(eps))(*[e._h.value for e in eps])
        _check(lib().uocr_ep_connect_local(arr, len(eps)))

    def set_wait_limit(self, seconds: float) -> None:
        _check(lib().uocr_ep_set_wait_limit(self._h, max(1, int(seconds * 1e9))))

    def forward_device(self, x_t, logits_t, mode: int = QuantizationMode.WEIGHTS_ONLY, y_t=None,
                       ids_t=None, wts_t=None):
        """One step of this rank's tokens x [T, hidden] (T may be 0).
        Asynchronous on the context's stream."""
        import torch
        t = x_t.shape[0]
        y_t = y_t if y_t is not None else torch.empty_like(x_t)
        ip = ctypes.c_void_p(_tptr(ids_t)) if ids_t is not None else None
        wp = ctypes.c_void_p(_tptr(wts_t)) if wts_t is not None else None
        _check(lib().uocr_ep_forward(self.ctx.handle, self._h, int(mode),
                                     ctypes.c_void_p(_tptr(x_t)) if t else None,
                                     ctypes.c_void_p(_tptr(logits_t)) if t else None, t,
                                     ctypes.c_void_p(_tptr(y_t)) if t else None, ip, wp))
        return y_t

    def forward_host_ptrs(self, x_ptr: int, logits_ptr: int, tokens: int, y_ptr: int,
                          mode: int = QuantizationMode.WEIGHTS_ONLY) -> None:
        """Host buffers (raw pointers): copy in, one step, copy out, synchronise."""
        _check(lib().uocr_ep_forward_host(self.ctx.handle, self._h, int(mode),
                                          ctypes.c_void_p(x_ptr), ctypes.c_void_p(logits_ptr),
                                          tokens, ctypes.c_void_p(y_ptr)))

    def forward(self, x, logits, mode: int = QuantizationMode.WEIGHTS_ONLY) -> np.ndarray:
        """Host tensors in, host tensor out (synchronous)."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.hidden)
        logits = np.ascontiguousarray(logits, dtype=np.float32).reshape(x.shape[0], self.n_experts)
        y = np.empty_like(x)
        self.forward_host_ptrs(x.ctypes.data, logits.ctypes.data, x.shape[0], y.ctypes.data, mode)
        return y

    # the step in three parts (several ranks driven from one thread, one stream)
    def dispatch_device(self, x_t, logits_t, mode: int, y_t) -> None:
        t = x_t.shape[0]
        _check(lib().uocr_ep_dispatch(self.ctx.handle, self._h, int(mode),
                                      ctypes.c_void_p(_tptr(x_t)) if t else None,
                                      ctypes.c_void_p(_tptr(logits_t)) if t else None, t,
                                      ctypes.c_void_p(_tptr(y_t)) if t else None))

    def experts_device(self) -> None:
        _check(lib().uocr_ep_experts(self.ctx.handle, self._h))

    def combine_device(self, y_t, ids_t=None, wts_t=None) -> None:
        yp = ctypes.c_void_p(_tptr(y_t)) if y_t is not None and y_t.numel() else None
        ip = ctypes.c_void_p(_tptr(ids_t)) if ids_t is not None and ids_t.numel() else None
        wp = ctypes.c_void_p(_tptr(wts_t)) if wts_t is not None and wts_t.numel() else None
        _check(lib().uocr_ep_combine(self.ctx.handle, self._h, yp, ip, wp))

    def free(self) -> None:
        if getattr(self, "_h", None):
            lib().uocr_ep_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


__all__ = ["BLOCK", "OcrError", "QuantizationMode", "GpuContext", "Int8Matrix", "MoeLayer",
           "route_device", "quantize_rows_device", "linear_multi_device", "default_context",
           "combine_device", "dispatch_device", "combine_rows_device",
           "LibraryMissing", "QuantizedWeights", "PeerExpertParallel", "EP_HANDLE_BYTES"]


def __getattr__(name):
    # QuantizedWeights lives in uocr_q8.overlay (imported on first use)
    if name == "QuantizedWeights":
        from .overlay import QuantizedWeights
        return QuantizedWeights
    raise AttributeError(name)
