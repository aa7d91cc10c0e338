"""The decoder on one GPU: prefill of a sequence and a batched decode step.

Decoder::step (src/decoder/mod.rs:400-420) for `batch` independent sequences
at once: embedding lookup (BF16 table), then per layer Decoder::layer
(:241-367) — RMSNorm, q/k/v projections, rope at each sequence's position,
KV-cache push, decode attention, o projection, residual, RMSNorm, then the
dense FFN (Decoder::feed_forward) for layers below ``first_dense`` or the MoE
(BF16 router logits, Decoder::experts), residual — and finally
Decoder::logits (:369-380): RMSNorm of the last hidden state and lm_head.

Every operation is a call into the CUDA library (uocr_rms_norm,
uocr_q8_linear[_dynamic_int8], uocr_kv_*, uocr_feed_forward,
uocr_linear_bf16, uocr_moe_forward); torch supplies device memory, the
embedding gather and the residual adds.  The whole step is asynchronous on
the context's stream with no host synchronisation, so it can be captured in
a CUDA graph.

Activation modes: the rows are independent sequences, each of which the
reference would run with one-row inputs, so DynamicActivations becomes the
row-wise int8 mode (every projection of every row with int8 activations);
WeightsOnly keeps FP32 activations everywhere.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional

import numpy as np

from . import (GpuContext, Int8Matrix, MoeLayer, QuantizationMode, _check, _tptr, lib)
from .attention import KvCache, Rope, add_rms_norm_device, rms_norm_device


@dataclass
class DecoderConfig:
    """The decoder dimensions (src/model/config.rs:30-67; the defaults are
    the upstream checkpoint's, tests/config.rs:5)."""
    hidden: int = 1280
    heads: int = 10
    layers: int = 12
    first_dense: int = 1
    experts: int = 64
    top_k: int = 6
    expert_width: int = 896
    shared_width: int = 1792
    dense_width: int = 6848
    vocab: int = 129280
    window: int = 128
    eps: float = 1e-6
    theta: float = 10000.0
    max_positions: int = 32768
    normalize: bool = False
    routed_scale: float = 1.0

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def _p(t):
    return ctypes.c_void_p(_tptr(t))


def linear_bf16_device(ctx: GpuContext, w_t, x_t, y_t=None):
    """ops::linear_weight BF16 branch: y [rows x n] = x @ w^T, w a BF16 (or its
    int16 bit patterns) [n x k] device tensor; bit-exact sequential sums."""
    import torch
    n, k = w_t.shape
    rows = x_t.numel() // k
    y_t = y_t if y_t is not None else torch.empty((rows, n), device=x_t.device)
    _check(lib().uocr_linear_bf16(ctx.handle, _p(w_t), n, k, _p(x_t), rows, _p(y_t)))
    return y_t


def linear_bf16_tc_device(ctx: GpuContext, w_t, x_t, y_t=None):
    """ops::linear_weight BF16 branch for a large weight (the lm_head): exact
    products on the tensor cores, FP32 accumulation (FP32 tolerance)."""
    import torch
    n, k = w_t.shape
    rows = x_t.numel() // k
    y_t = y_t if y_t is not None else torch.empty((rows, n), device=x_t.device)
    _check(lib().uocr_linear_bf16_tc(ctx.handle, _p(w_t), n, k, _p(x_t), rows, _p(y_t)))
    return y_t


def feed_forward_device(ctx: GpuContext, gate: Int8Matrix, up: Int8Matrix, down: Int8Matrix,
                        x_t, mode: int, y_t=None):
    """Decoder::feed_forward over rows of x (uocr_feed_forward)."""
    import torch
    rows = x_t.numel() // gate.cols
    y_t = y_t if y_t is not None else torch.empty((rows, down.rows), device=x_t.device)
    _check(lib().uocr_feed_forward(ctx.handle, gate.handle, up.handle, down.handle, int(mode),
                                   _p(x_t), rows, _p(y_t)))
    return y_t


class DecoderLayer:
    """Weights of one decoder layer on the device.  ``qkv`` is the q, k and v
    projections stacked into one [3*hidden x hidden] matrix (one launch for
    the three; each output row is the same dot as in its own matrix).
    ``dense`` holds the dense FFN with its width zero-padded to a multiple of
    128 (zero weights and scales in the extra rows of gate/up and columns of
    down, which leaves every output unchanged); ``dense_width`` is the
    unpadded width."""

    def __init__(self, input_norm_t, qkv: Int8Matrix, o: Int8Matrix, post_norm_t, dense=None,
                 dense_width: int = 0, router_t=None, moe: Optional[MoeLayer] = None):
        self.input_norm, self.qkv, self.o = input_norm_t, qkv, o
        self.post_norm = post_norm_t
        self.dense = dense      # (gate, up, down) Int8Matrix
        self.dense_width = dense_width
        self.router = router_t  # BF16 [experts x hidden]
        self.moe = moe


class Decoder:
    """Device-resident decoder weights (q8 projections, BF16 embedding and
    router, q8 or BF16 lm_head)."""

    def __init__(self, ctx: GpuContext, cfg: DecoderConfig, layers: List[DecoderLayer],
                 embedding_t, final_norm_t, lm_head):
        self.ctx, self.cfg, self.layers = ctx, cfg, layers
        self.embedding = embedding_t  # torch.bfloat16 [vocab x hidden]
        self.final_norm = final_norm_t
        self.lm_head = lm_head        # Int8Matrix, or a bf16 torch tensor [vocab x hidden]

    @classmethod
    def random(cls, ctx: GpuContext, cfg: DecoderConfig, seed: int = 0, lm_head: str = "q8"):
        """Random-init weights of the decoder's architecture, generated on the
        device (q8 weights uniform in [-127, 127], scales U(1e-4, 1e-2); norms
        near 1; BF16 embedding and router N(0, 1))."""
        import torch
        dev = f"cuda:{ctx.device}"
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        H = cfg.hidden

        def mat(r, c, lo=1e-4, hi=1e-2):
            w = torch.randint(-127, 128, (r, c), dtype=torch.int8, device=dev, generator=g)
            s = torch.rand((r, (c + 31) // 32), device=dev, generator=g) * (hi - lo) + lo
            return Int8Matrix.from_device(r, c, w, s.contiguous(), ctx)

        def norm():
            return (torch.rand(H, device=dev, generator=g) * 0.5 + 0.75).contiguous()

        def padded_ffn(F):
            # rows F.. of gate/up and columns F.. of down are zero (weights and
            # scales): the padded FFN computes exactly the unpadded one
            Fp = (F + 127) // 128 * 128
            gw = torch.zeros((Fp, H), dtype=torch.int8, device=dev)
            uw = torch.zeros((Fp, H), dtype=torch.int8, device=dev)
            gs = torch.zeros((Fp, H // 32), device=dev)
            us = torch.zeros((Fp, H // 32), device=dev)
            dw = torch.zeros((H, Fp), dtype=torch.int8, device=dev)
            ds = torch.zeros((H, Fp // 32), device=dev)
            for w_, s_ in ((gw, gs), (uw, us)):
                w_[:F] = torch.randint(-127, 128, (F, H), dtype=torch.int8, device=dev, generator=g)
                s_[:F] = torch.rand((F, H // 32), device=dev, generator=g) * (1e-2 - 1e-4) + 1e-4
            dw[:, :F] = torch.randint(-127, 128, (H, F), dtype=torch.int8, device=dev, generator=g)
            ds[:, :F // 32] = torch.rand((H, F // 32), device=dev, generator=g) * (1e-2 - 1e-4) + 1e-4
            return (Int8Matrix.from_device(Fp, H, gw, gs, ctx),
                    Int8Matrix.from_device(Fp, H, uw, us, ctx),
                    Int8Matrix.from_device(H, Fp, dw, ds, ctx))

        layers = []
        for i in range(cfg.layers):
            qkv, o = mat(3 * H, H, 1e-4, 1e-3), mat(H, H, 1e-4, 1e-3)
            if i < cfg.first_dense:
                layers.append(DecoderLayer(norm(), qkv, o, norm(), dense=padded_ffn(cfg.dense_width),
                                           dense_width=cfg.dense_width))
            else:
                shared = [mat(cfg.shared_width, H), mat(cfg.shared_width, H),
                          mat(H, cfg.shared_width)]
                experts = [[mat(cfg.expert_width, H), mat(cfg.expert_width, H),
                            mat(H, cfg.expert_width)] for _ in range(cfg.experts)]
                moe = MoeLayer(ctx, shared, experts, cfg.top_k, cfg.normalize, cfg.routed_scale)
                router = (torch.randn((cfg.experts, H), device=dev, generator=g) * 0.03).to(
                    torch.bfloat16)
                layers.append(DecoderLayer(norm(), qkv, o, norm(), router_t=router, moe=moe))
        emb = torch.randn((cfg.vocab, H), device=dev, generator=g).to(torch.bfloat16)
        if lm_head == "q8":
            head = mat(cfg.vocab, H, 1e-4, 1e-3)
        else:
            head = (torch.randn((cfg.vocab, H), device=dev, generator=g) * 0.03).to(
                torch.bfloat16)
        return cls(ctx, cfg, layers, emb, norm(), head)


class DecodeState:
    """Per-layer KV caches (LayerCache for every sequence) and the rotary table."""

    def __init__(self, decoder: Decoder, batch: int, max_prefix: int):
        cfg = decoder.cfg
        self.batch = batch
        self.max_prefix = max_prefix
        self.caches = [KvCache(decoder.ctx, batch, cfg.heads, cfg.head_dim, cfg.window, max_prefix)
                       for _ in range(cfg.layers)]
        self.rope = Rope(decoder.ctx, cfg.head_dim, cfg.theta, cfg.max_positions)

    def reset(self, seq: int = 0):
        """Every layer's cache of sequence seq empty again (a new prefill)."""
        for c in self.caches:
            c.reset(seq)

    def free(self):
        for c in self.caches:
            c.free()
        self.rope.free()


def decode_step(decoder: Decoder, state: DecodeState, tokens_t, mode: int = 0, logits_t=None,
                experts=None):
    """One decode step for every sequence: tokens_t int64 [batch] -> logits
    [batch x vocab] (device, asynchronous).  ``experts``: optional, per layer
    index, an object whose ``forward_device(x, logits, mode)`` replaces the
    layer's own MoE (a ``PeerExpertParallel`` holding this GPU's share of the
    routed experts: attention and projections run on this GPU's sequences,
    the MoE layers over the GPUs of the node)."""
    import torch
    ctx, cfg = decoder.ctx, decoder.cfg
    rowwise = mode in (QuantizationMode.DYNAMIC_ACTIVATIONS, QuantizationMode.DYNAMIC_ROWWISE)
    lin_mode = QuantizationMode.DYNAMIC_ROWWISE if rowwise else QuantizationMode.WEIGHTS_ONLY
    H = cfg.hidden
    x = decoder.embedding.index_select(0, tokens_t).float()
    y = None  # the previous layer's FFN output, added to x before the next norm
    for li, (layer, cache) in enumerate(zip(decoder.layers, state.caches)):
        # attention half of Decoder::layer (src/decoder/mod.rs:266-347); each
        # residual add runs fused with the RMSNorm of its sum
        if y is None:
            n = rms_norm_device(ctx, x, layer.input_norm, cfg.eps)
        else:
            n = add_rms_norm_device(ctx, x, y, layer.input_norm, cfg.eps, sum_t=x)
        qkv = layer.qkv.linear_device(n, dynamic=rowwise)
        q = cache.rope_push_qkv(state.rope, qkv)  # rope of q, k; push of k, v
        a = cache.attention(q)
        r = layer.o.linear_device(a, dynamic=rowwise)
        n = add_rms_norm_device(ctx, r, x, layer.post_norm, cfg.eps, sum_t=r)  # r += x
        if layer.moe is not None:
            logits = linear_bf16_device(ctx, layer.router, n)
            moe = experts[li] if experts is not None and experts[li] is not None else layer.moe
            y = moe.forward_device(n, logits, lin_mode)
        else:
            y = feed_forward_device(ctx, *layer.dense, n, lin_mode)
        x = r  # x + y is formed by the next norm
    h = add_rms_norm_device(ctx, x, y, decoder.final_norm, cfg.eps, sum_t=x)
    if isinstance(decoder.lm_head, Int8Matrix):
        return decoder.lm_head.linear_device(h, logits_t, dynamic=rowwise)
    # BF16 head: the tensor-core BF16 linear straight from the bf16 weights
    return linear_bf16_tc_device(ctx, decoder.lm_head, h, logits_t)


def prefill(decoder: Decoder, state: DecodeState, embeddings_t, mode: int = 0, seq: int = 0,
            logits_t=None):
    """Decoder::prefill (src/decoder/mod.rs:382-398) of sequence `seq` of the
    state: embeddings_t [tokens x hidden] (FP32, device) through every layer
    at positions 0..tokens-1 — Decoder::layer with position 0
    (:241-367): RMSNorm, q/k/v projections, rope of every row at its
    position, LayerCache::prefill, the causal attention over the prefix, o
    projection, residual, RMSNorm, the dense FFN or the MoE over all rows,
    residual — then Decoder::logits (:369-380) of the last row.  Projections
    follow Decoder::projection: int8 activations only for one-row inputs in
    DynamicActivations (so a prefill of several rows runs its projections
    with FP32 activations, and an expert that receives one row runs it with
    int8 activations), every row in the row-wise mode.  Returns the logits
    [1 x vocab] (device, asynchronous)."""
    import torch
    ctx, cfg = decoder.ctx, decoder.cfg
    H = cfg.hidden
    x = embeddings_t.reshape(-1, H).float().clone()
    T = x.shape[0]
    if T > state.max_prefix:
        raise ValueError("prefill longer than the state's prefix capacity")
    dyn = mode == QuantizationMode.DYNAMIC_ROWWISE or (
        mode == QuantizationMode.DYNAMIC_ACTIVATIONS and T == 1)
    positions = torch.arange(T, dtype=torch.int32, device=x.device)
    y = None
    for layer, cache in zip(decoder.layers, state.caches):
        if y is None:
            n = rms_norm_device(ctx, x, layer.input_norm, cfg.eps)
        else:
            n = add_rms_norm_device(ctx, x, y, layer.input_norm, cfg.eps, sum_t=x)
        qkv = layer.qkv.linear_device(n, dynamic=dyn)
        q, k, v = (qkv[:, i * H:(i + 1) * H].contiguous() for i in range(3))
        state.rope.apply(q, k, positions)
        cache.prefill(seq, k, v)
        a = cache.attention_prefill(seq, q)
        r = layer.o.linear_device(a, dynamic=dyn)
        n = add_rms_norm_device(ctx, r, x, layer.post_norm, cfg.eps, sum_t=r)  # r += x
        if layer.moe is not None:
            logits = linear_bf16_device(ctx, layer.router, n)
            y = layer.moe.forward_device(n, logits, mode)
        else:
            y = feed_forward_device(ctx, *layer.dense, n, mode)
        x = r
    h = add_rms_norm_device(ctx, x[T - 1:], y[T - 1:], decoder.final_norm, cfg.eps)
    if isinstance(decoder.lm_head, Int8Matrix):
        return decoder.lm_head.linear_device(
            h, logits_t, dynamic=mode != QuantizationMode.WEIGHTS_ONLY)
    return linear_bf16_tc_device(ctx, decoder.lm_head, h, logits_t)


def logits_checksum_device(ctx: GpuContext, logits_t, acc_t):
    """acc_t (int64 [1], device) += the bit patterns of logits_t as u64,
    wrapping (the fixed-work benchmark's checksum, uocr_bits_checksum)."""
    _check(lib().uocr_bits_checksum(ctx.handle, _p(logits_t), logits_t.numel(), _p(acc_t)))


# ---- loading a checkpoint with its INT8 overlay -------------------------------

_CONFIG_REQUIRED = ("model_type", "hidden_size", "intermediate_size", "moe_intermediate_size",
                    "num_hidden_layers", "num_attention_heads", "num_key_value_heads",
                    "n_routed_experts", "n_shared_experts", "num_experts_per_tok",
                    "first_k_dense_replace", "use_mla", "vocab_size")


def config_from_json(text: str) -> DecoderConfig:
    """ModelConfig::from_json (src/model/config.rs:69-117): the same required
    fields, defaults and checks (Unsupported for an attention or routing
    variant the decoder does not implement, Shape for invalid dimensions)."""
    import json

    from . import OcrError
    try:
        c = json.loads(text)
    except ValueError as e:
        raise OcrError(2, f"JSON: {e}") from None
    if not isinstance(c, dict):
        raise OcrError(2, "JSON: invalid type, expected struct ModelConfig")
    for key in _CONFIG_REQUIRED:
        if key not in c:
            raise OcrError(2, f"JSON: missing field `{key}`")
    g = lambda k, d: c.get(k, d)  # noqa: E731
    if (c["model_type"] != "unlimited-ocr" or c["use_mla"] or g("attention_bias", False)
            or g("rope_scaling", None) is not None or g("topk_method", "greedy") != "greedy"
            or g("scoring_func", "softmax") != "softmax" or g("moe_layer_freq", 1) != 1):
        raise OcrError(5, "unsupported configuration: model attention or routing configuration")
    hidden, heads = c["hidden_size"], c["num_attention_heads"]
    eps, theta = g("rms_norm_eps", 1e-6), g("rope_theta", 10000.0)
    scale = g("routed_scaling_factor", 1.0)
    bad = (hidden == 0 or heads == 0 or hidden % heads or (hidden // heads) % 2
           or heads != c["num_key_value_heads"] or c["num_hidden_layers"] == 0
           or c["vocab_size"] == 0 or c["intermediate_size"] == 0
           or c["moe_intermediate_size"] == 0 or c["n_shared_experts"] == 0
           or c["num_experts_per_tok"] == 0
           or c["num_experts_per_tok"] > c["n_routed_experts"]
           or c["first_k_dense_replace"] > c["num_hidden_layers"]
           or g("sliding_window", 128) == 0 or g("max_position_embeddings", 32768) == 0
           or not (eps > 0 and eps != float("inf")) or not (theta > 0 and theta != float("inf"))
           or not (scale > 0 and scale != float("inf")))
    if bad:
        raise OcrError(4, "invalid tensor shape: invalid decoder configuration")
    return DecoderConfig(hidden=hidden, heads=heads, layers=c["num_hidden_layers"],
                         first_dense=c["first_k_dense_replace"], experts=c["n_routed_experts"],
                         top_k=c["num_experts_per_tok"],
                         expert_width=c["moe_intermediate_size"],
                         shared_width=c["moe_intermediate_size"] * c["n_shared_experts"],
                         dense_width=c["intermediate_size"], vocab=c["vocab_size"],
                         window=g("sliding_window", 128), eps=float(eps), theta=float(theta),
                         max_positions=g("max_position_embeddings", 32768),
                         normalize=bool(g("norm_topk_prob", False)), routed_scale=float(scale))


class _Checkpoint:
    """Read-only view of a safetensors file's tensors (host, memory-mapped);
    layout validation is the library's (the overlay loader checks the source
    with the reference's rules before this reads it)."""

    def __init__(self, path):
        import json
        import struct
        with open(path, "rb") as f:
            n = struct.unpack("<Q", f.read(8))[0]
            header = json.loads(f.read(n))
        header.pop("__metadata__", None)
        self.header, self.start = header, 8 + n
        self.mm = np.memmap(path, dtype=np.uint8, mode="r")

    def raw(self, name):
        from . import OcrError
        d = self.header.get(name)
        if d is None:
            raise OcrError(3, f"invalid checkpoint: missing tensor: {name}")
        b = self.mm[self.start + d["data_offsets"][0]:self.start + d["data_offsets"][1]]
        return d["dtype"], list(d["shape"]), b

    def f32(self, name, shape):
        """WeightView::to_f32 (src/checkpoint.rs:75-107) of a tensor whose
        shape must be `shape` (Decoder::new's check, src/decoder/mod.rs:34-43)."""
        from . import OcrError
        dt, sh, b = self.raw(name)
        if sh != list(shape):
            raise OcrError(4, f"invalid tensor shape: {name}: expected {list(shape)}, got {sh}")
        if dt == "F32":
            v = b.view("<f4")
        elif dt == "BF16":
            v = (b.view("<u2").astype(np.uint32) << 16).view(np.float32)
        elif dt == "F16":
            v = b.view("<f2").astype(np.float32)
        elif dt == "I8":
            v = b.view(np.int8).astype(np.float32)
        elif dt == "I64":
            v = b.view("<i8").astype(np.float32)
        else:
            raise OcrError(5, f"unsupported configuration: dtype {dt} of {name}")
        return np.array(v.reshape(shape), dtype=np.float32)  # a writable copy


def _device_view(ptr: int, n: int, typestr: str, device: int):
    """A torch tensor over n elements of device memory owned elsewhere."""
    import torch

    class _Arr:
        __cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False),
                                    "version": 3, "strides": None}
    return torch.as_tensor(_Arr(), device=f"cuda:{device}")


def _matrix_tensors(m: Int8Matrix):
    """(weights int8 [rows, cols], scales float [rows, blocks]) device views."""
    w, s = m.device_ptrs()
    nb = (m.cols + 31) // 32
    return (_device_view(w, m.rows * m.cols, "|i1", m.ctx.device).view(m.rows, m.cols),
            _device_view(s, m.rows * nb, "<f4", m.ctx.device).view(m.rows, nb))


def load_decoder(ctx: GpuContext, directory, overlay_path,
                 mode: int = QuantizationMode.WEIGHTS_ONLY, source_path=None) -> "Decoder":
    """Model::load_with_quantization (src/model/mod.rs:81-105) for the decoder:
    config.json and the checkpoint of ``directory``, the INT8 overlay validated
    and uploaded by QuantizedWeights::load (uocr_overlay_load, every check of
    the reference), the checkpoint's shapes checked as Decoder::new does
    (src/decoder/mod.rs:32-83).  Norms, the router (BF16) and the embedding
    come from the checkpoint; every projection and lm_head from the overlay.
    On the device the q/k/v projections are stacked into one matrix and the
    dense FFN is zero-padded to a multiple of 128 rows (exactly the same
    outputs); the routed and shared experts are the overlay's own matrices."""
    import os

    import torch

    from . import OcrError
    from .overlay import QuantizedWeights
    if overlay_path is None:
        if mode == QuantizationMode.DYNAMIC_ACTIVATIONS:
            raise OcrError(3, "dynamic INT8 requires a quantized weight overlay")
        raise OcrError(5, "unsupported configuration: the device decoder runs the INT8 overlay "
                          "(BF16 projections are outside it)")
    source_path = source_path or os.path.join(directory, "model-00001-of-000001.safetensors")
    with open(os.path.join(directory, "config.json")) as f:
        cfg = config_from_json(f.read())
    ov = QuantizedWeights.load(overlay_path, source_path, ctx)
    ck = _Checkpoint(source_path)
    H, dev = cfg.hidden, f"cuda:{ctx.device}"

    def q8(name, rows, cols):
        m = ov.get(name)
        if m is None:
            raise OcrError(3, f"invalid checkpoint: missing tensor: {name}")
        if (m.rows, m.cols) != (rows, cols):
            raise OcrError(4, f"invalid tensor shape: {name}: expected {[rows, cols]}, "
                              f"got {[m.rows, m.cols]}")
        return m

    def vec(name):
        return torch.from_numpy(ck.f32(name, [H])).to(dev)

    def padded_ffn(prefix, F):
        g, u, d = (q8(f"{prefix}.{p}_proj.weight", *shape) for p, shape in
                   (("gate", (F, H)), ("up", (F, H)), ("down", (H, F))))
        Fp = (F + 127) // 128 * 128
        if Fp == F:
            return (g, u, d), []
        nbH, nbF, nbP = (H + 31) // 32, (F + 31) // 32, Fp // 32
        if F % 32:
            raise OcrError(5, "unsupported configuration: dense FFN width not a multiple of 32")
        out, keep = [], []
        for m in (g, u):
            w, s = _matrix_tensors(m)
            wp = torch.zeros((Fp, H), dtype=torch.int8, device=dev)
            sp = torch.zeros((Fp, nbH), device=dev)
            wp[:F], sp[:F] = w, s
            out.append(Int8Matrix.from_device(Fp, H, wp, sp, ctx))
        w, s = _matrix_tensors(d)
        wp = torch.zeros((H, Fp), dtype=torch.int8, device=dev)
        sp = torch.zeros((H, nbP), device=dev)
        wp[:, :F], sp[:, :nbF] = w, s
        out.append(Int8Matrix.from_device(H, Fp, wp, sp, ctx))
        return tuple(out), keep

    layers = []
    for i in range(cfg.layers):
        pre = f"model.layers.{i}"
        parts = [_matrix_tensors(q8(f"{pre}.self_attn.{p}_proj.weight", H, H)) for p in "qkv"]
        qkv = Int8Matrix.from_device(3 * H, H, torch.cat([w for w, _ in parts]).contiguous(),
                                     torch.cat([s for _, s in parts]).contiguous(), ctx)
        o = q8(f"{pre}.self_attn.o_proj.weight", H, H)
        in_norm, post_norm = vec(f"{pre}.input_layernorm.weight"), \
            vec(f"{pre}.post_attention_layernorm.weight")
        if i < cfg.first_dense:
            dense, _ = padded_ffn(f"{pre}.mlp", cfg.dense_width)
            layers.append(DecoderLayer(in_norm, qkv, o, post_norm, dense=dense,
                                       dense_width=cfg.dense_width))
            continue
        dt, sh, b = ck.raw(f"{pre}.mlp.gate.weight")
        if sh != [cfg.experts, H]:
            raise OcrError(4, f"invalid tensor shape: {pre}.mlp.gate.weight: expected "
                              f"{[cfg.experts, H]}, got {sh}")
        if dt != "BF16":
            raise OcrError(5, f"unsupported configuration: router dtype {dt} (BF16 only)")
        router = torch.from_numpy(np.array(b.view("<i2")).reshape(cfg.experts, H)).to(dev)
        ffn = lambda name, F: [q8(f"{name}.{p}_proj.weight", *shape) for p, shape in  # noqa: E731
                               (("gate", (F, H)), ("up", (F, H)), ("down", (H, F)))]
        shared = ffn(f"{pre}.mlp.shared_experts", cfg.shared_width)
        experts = [ffn(f"{pre}.mlp.experts.{e}", cfg.expert_width) for e in range(cfg.experts)]
        moe = MoeLayer(ctx, shared, experts, cfg.top_k, cfg.normalize, cfg.routed_scale)
        layers.append(DecoderLayer(in_norm, qkv, o, post_norm, router_t=router, moe=moe))
    dt, sh, b = ck.raw("model.embed_tokens.weight")
    if sh != [cfg.vocab, H]:
        raise OcrError(4, f"invalid tensor shape: model.embed_tokens.weight: expected "
                          f"{[cfg.vocab, H]}, got {sh}")
    if dt == "BF16":
        emb = torch.from_numpy(np.array(b.view("<i2")).reshape(cfg.vocab, H)).to(dev).view(
            torch.bfloat16)
    else:
        emb = torch.from_numpy(ck.f32("model.embed_tokens.weight", [cfg.vocab, H])).to(dev)
    head = q8("lm_head.weight", cfg.vocab, H)
    dec = Decoder(ctx, cfg, layers, emb, vec("model.norm.weight"), head)
    dec.mode = int(mode)
    dec.overlay = ov  # the overlay owns the matrices the layers borrow
    return dec


__all__ = ["DecoderConfig", "Decoder", "DecoderLayer", "DecodeState", "decode_step",
           "linear_bf16_device", "feed_forward_device", "config_from_json", "load_decoder"]
