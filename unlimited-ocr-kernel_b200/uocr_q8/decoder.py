"""A batched decode step of the decoder on one GPU.

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

from . import (GpuContext, Int8Matrix, MoeLayer, QuantizationMode, _check, _tptr, lib)
from .attention import KvCache, Rope, rms_norm_device


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
        self.lm_head = lm_head        # Int8Matrix, or a float32 torch tensor [vocab x hidden]

    @classmethod
    def random(cls, ctx: GpuContext, cfg: DecoderConfig, seed: int = 0, lm_head: str = "q8"):
        """Random-init weights of the decoder's architecture, generated on the
        device (q8 weights uniform in [-127, 127], scales U(1e-4, 1e-2) as in
        BASELINE config 0; norms near 1; BF16 embedding and router N(0, 1))."""
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
                torch.bfloat16).float()
        return cls(ctx, cfg, layers, emb, norm(), head)


class DecodeState:
    """Per-layer KV caches (LayerCache for every sequence) and the rotary table."""

    def __init__(self, decoder: Decoder, batch: int, max_prefix: int):
        cfg = decoder.cfg
        self.batch = batch
        self.caches = [KvCache(decoder.ctx, batch, cfg.heads, cfg.head_dim, cfg.window, max_prefix)
                       for _ in range(cfg.layers)]
        self.rope = Rope(decoder.ctx, cfg.head_dim, cfg.theta, cfg.max_positions)

    def free(self):
        for c in self.caches:
            c.free()
        self.rope.free()


def decode_step(decoder: Decoder, state: DecodeState, tokens_t, mode: int = 0, logits_t=None):
    """One decode step for every sequence: tokens_t int64 [batch] -> logits
    [batch x vocab] (device, asynchronous)."""
    import torch
    ctx, cfg = decoder.ctx, decoder.cfg
    rowwise = mode in (QuantizationMode.DYNAMIC_ACTIVATIONS, QuantizationMode.DYNAMIC_ROWWISE)
    lin_mode = QuantizationMode.DYNAMIC_ROWWISE if rowwise else QuantizationMode.WEIGHTS_ONLY
    H = cfg.hidden
    x = decoder.embedding.index_select(0, tokens_t).float()
    for layer, cache in zip(decoder.layers, state.caches):
        # attention half of Decoder::layer (src/decoder/mod.rs:266-347)
        n = rms_norm_device(ctx, x, layer.input_norm, cfg.eps)
        qkv = layer.qkv.linear_device(n, dynamic=rowwise)
        q = cache.rope_push_qkv(state.rope, qkv)  # rope of q, k; push of k, v
        a = cache.attention(q)
        r = layer.o.linear_device(a, dynamic=rowwise)
        r += x
        n = rms_norm_device(ctx, r, layer.post_norm, cfg.eps)
        if layer.moe is not None:
            logits = linear_bf16_device(ctx, layer.router, n)
            y = layer.moe.forward_device(n, logits, lin_mode)
        else:
            y = feed_forward_device(ctx, *layer.dense, n, lin_mode)
        x = r.add_(y)
    h = rms_norm_device(ctx, x, decoder.final_norm, cfg.eps)
    if isinstance(decoder.lm_head, Int8Matrix):
        return decoder.lm_head.linear_device(h, logits_t, dynamic=rowwise)
    out = torch.matmul(h, decoder.lm_head.t())  # BF16 head: a library GEMM over its f32 copy
    if logits_t is not None:
        logits_t.copy_(out)
        return logits_t
    return out


__all__ = ["DecoderConfig", "Decoder", "DecoderLayer", "DecodeState", "decode_step",
           "linear_bf16_device", "feed_forward_device"]
