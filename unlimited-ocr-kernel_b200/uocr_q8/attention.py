"""Decode-side attention ops of a decoder layer on the GPU.

Mirrors the reference's operators on device tensors (torch CUDA tensors,
asynchronous on the context's stream):

* ``rms_norm_device`` — ops::rms_norm (src/cpu/ops.rs:362-414, 419-421);
* ``Rope`` — ops::rope (src/cpu/ops.rs:423-437) with a host-built cos/sin table;
* ``attention_decode_device`` — ops::attention_decode (src/cpu/ops.rs:515-606);
* ``KvCache`` — LayerCache (src/decoder/cache.rs) for a batch of sequences,
  with ``push``, ``rope`` (at each sequence's position) and ``attention``;
* ``AttentionBlock`` — the attention half of Decoder::layer
  (src/decoder/mod.rs:241-341) at decode: norm, q/k/v projections (q8
  overlay matrices), rope, cache push, attention, o projection, residual.

Every call goes to the CUDA library (libuocr_q8.so).
"""
from __future__ import annotations

import ctypes
from typing import Optional

from . import GpuContext, Int8Matrix, QuantizationMode, _check, _tptr, lib


def _p(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(_tptr(t)) if t is not None else None


def rms_norm_device(ctx: GpuContext, x_t, weight_t, eps: float = 1e-6, out_t=None):
    import torch
    width = x_t.shape[-1]
    out_t = out_t if out_t is not None else torch.empty_like(x_t)
    _check(lib().uocr_rms_norm(ctx.handle, _p(x_t), x_t.numel() // max(width, 1), width,
                               _p(weight_t), float(eps), _p(out_t)))
    return out_t


def add_rms_norm_device(ctx: GpuContext, x_t, res_t, weight_t, eps: float = 1e-6, sum_t=None,
                        out_t=None):
    """sum = x + res (into sum_t, which may be x_t or res_t), then the RMSNorm
    of sum into out_t, in one launch (uocr_add_rms_norm).  Returns out_t."""
    import torch
    width = x_t.shape[-1]
    sum_t = sum_t if sum_t is not None else torch.empty_like(x_t)
    out_t = out_t if out_t is not None else torch.empty_like(x_t)
    _check(lib().uocr_add_rms_norm(ctx.handle, _p(x_t), _p(res_t), x_t.numel() // max(width, 1),
                                   width, _p(weight_t), float(eps), _p(sum_t), _p(out_t)))
    return out_t


def attention_decode_device(ctx: GpuContext, q_t, keys_t, values_t, heads: int, out_t=None):
    """One query [width] over token-major keys/values [tokens x width]."""
    import torch
    out_t = out_t if out_t is not None else torch.empty_like(q_t)
    _check(lib().uocr_attention_decode(ctx.handle, _p(q_t), _p(keys_t), keys_t.numel(),
                                       _p(values_t), values_t.numel(), q_t.numel(), heads,
                                       _p(out_t)))
    return out_t


def attention_prefill_device(ctx: GpuContext, q_t, keys_t, values_t, heads: int, out_t=None):
    """Causal attention of a prefill: token-major q/keys/values [tokens x
    width], row i over tokens 0..i (uocr_attention_prefill)."""
    import torch
    tokens, width = q_t.shape
    out_t = out_t if out_t is not None else torch.empty_like(q_t)
    _check(lib().uocr_attention_prefill(ctx.handle, _p(q_t), _p(keys_t), _p(values_t), tokens,
                                        width, heads, _p(out_t)))
    return out_t


class Rope:
    """cos/sin table of positions [0, max_positions) (device)."""

    def __init__(self, ctx: GpuContext, head_dim: int, theta: float = 10000.0,
                 max_positions: int = 32768):
        self.ctx = ctx
        self.head_dim = head_dim
        h = ctypes.c_void_p()
        _check(lib().uocr_rope_create(ctx.handle, head_dim, float(theta), max_positions,
                                      ctypes.byref(h)))
        self._h = h

    def apply(self, q_t, k_t, positions_t):
        """Rotate q (and k) rows [rows x width] at positions (int32, device)."""
        width = q_t.shape[-1]
        _check(lib().uocr_rope_apply(self.ctx.handle, self._h, _p(q_t), _p(k_t),
                                     q_t.numel() // width, width, _p(positions_t)))

    def free(self):
        if getattr(self, "_h", None):
            lib().uocr_rope_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class KvCache:
    """LayerCache for `batch` sequences (device)."""

    def __init__(self, ctx: GpuContext, batch: int, heads: int, head_dim: int, window: int,
                 max_prefix: int):
        self.ctx = ctx
        self.batch, self.heads, self.head_dim = batch, heads, head_dim
        self.width = heads * head_dim
        h = ctypes.c_void_p()
        _check(lib().uocr_kv_create(ctx.handle, batch, heads, head_dim, window, max_prefix,
                                    ctypes.byref(h)))
        self._h = h

    def prefill(self, seq: int, keys_t, values_t):
        tokens = keys_t.numel() // self.width
        _check(lib().uocr_kv_prefill(self.ctx.handle, self._h, seq, _p(keys_t), _p(values_t),
                                     tokens))

    def push(self, k_t, v_t):
        _check(lib().uocr_kv_push(self.ctx.handle, self._h, _p(k_t), _p(v_t)))

    def rope(self, rope: Rope, q_t, k_t):
        _check(lib().uocr_kv_rope(self.ctx.handle, self._h, rope._h, _p(q_t), _p(k_t)))

    def rope_push_qkv(self, rope: Rope, qkv_t, q_out_t=None):
        """rope + push from fused projection rows [q | k | v]; returns the
        rotated q rows (uocr_kv_rope_push_qkv)."""
        import torch
        q_out_t = q_out_t if q_out_t is not None else torch.empty(
            (self.batch, self.width), device=qkv_t.device)
        _check(lib().uocr_kv_rope_push_qkv(self.ctx.handle, self._h, rope._h, _p(qkv_t),
                                           _p(q_out_t)))
        return q_out_t

    def attention(self, q_t, out_t=None):
        import torch
        out_t = out_t if out_t is not None else torch.empty_like(q_t)
        _check(lib().uocr_kv_attention(self.ctx.handle, self._h, _p(q_t), _p(out_t)))
        return out_t

    def set_attention_form(self, form: int):
        """0 by size, 1 one CTA per (head, sequence), 2 split over tokens
        (uocr_kv_set_attention_form); the same results either way."""
        _check(lib().uocr_kv_set_attention_form(self._h, int(form)))

    def reset(self, seq: int):
        """Sequence seq empty again, to be prefilled anew (uocr_kv_reset)."""
        _check(lib().uocr_kv_reset(self.ctx.handle, self._h, seq))

    def attention_prefill(self, seq: int, q_t, out_t=None):
        """Causal attention of the prefill rows of sequence seq, right after
        their prefill (uocr_kv_attention_prefill)."""
        import torch
        out_t = out_t if out_t is not None else torch.empty_like(q_t)
        _check(lib().uocr_kv_attention_prefill(self.ctx.handle, self._h, seq, _p(q_t),
                                               q_t.numel() // self.width, _p(out_t)))
        return out_t

    def state(self, seq: int):
        """(tokens, position) of sequence seq (synchronous)."""
        t, p = ctypes.c_size_t(), ctypes.c_size_t()
        _check(lib().uocr_kv_state(self.ctx.handle, self._h, seq, ctypes.byref(t), ctypes.byref(p)))
        return t.value, p.value

    def export(self, seq: int):
        """LayerCache::keys / ::values of sequence seq: token-major [tokens,
        width] device tensors (a copy)."""
        import torch
        n = ctypes.c_size_t()
        _check(lib().uocr_kv_export(self.ctx.handle, self._h, seq, None, None, ctypes.byref(n)))
        k = torch.empty((n.value, self.width), device=f"cuda:{self.ctx.device}")
        v = torch.empty_like(k)
        _check(lib().uocr_kv_export(self.ctx.handle, self._h, seq, _p(k), _p(v), ctypes.byref(n)))
        return k, v

    def free(self):
        if getattr(self, "_h", None):
            lib().uocr_kv_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class AttentionBlock:
    """The attention half of Decoder::layer at decode for a batch of
    sequences (src/decoder/mod.rs:241-341): residual = x + o_proj(attn(rope(
    q_proj(n)), rope(k_proj(n)), v_proj(n))) with n = rms_norm(x), k/v pushed
    into the cache first.  Projections are q8 matrices under the given
    QuantizationMode (Decoder::projection, src/decoder/mod.rs:99-112)."""

    def __init__(self, ctx: GpuContext, norm_t, q: Int8Matrix, k: Int8Matrix, v: Int8Matrix,
                 o: Int8Matrix, cache: KvCache, rope: Rope, eps: float = 1e-6):
        self.ctx, self.norm, self.q, self.k, self.v, self.o = ctx, norm_t, q, k, v, o
        self.cache, self.rope_table, self.eps = cache, rope, eps

    def forward_device(self, x_t, mode: int = QuantizationMode.WEIGHTS_ONLY, out_t=None):
        """Rows of x_t are independent sequences (one token each), so both
        int8 modes quantize every row's activations, as one-row calls would."""
        import torch
        dyn = mode in (QuantizationMode.DYNAMIC_ACTIVATIONS, QuantizationMode.DYNAMIC_ROWWISE)
        n = rms_norm_device(self.ctx, x_t, self.norm, self.eps)
        q = self.q.linear_device(n, dynamic=dyn)
        k = self.k.linear_device(n, dynamic=dyn)
        v = self.v.linear_device(n, dynamic=dyn)
        self.cache.rope(self.rope_table, q, k)
        self.cache.push(k, v)
        a = self.cache.attention(q)
        out_t = out_t if out_t is not None else torch.empty_like(x_t)
        self.o.linear_device(a, out_t, dynamic=dyn)
        out_t += x_t
        return out_t


__all__ = ["rms_norm_device", "add_rms_norm_device", "attention_decode_device", "Rope", "KvCache",
           "AttentionBlock"]
