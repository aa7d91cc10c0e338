"""Loader and ctypes signatures of libuocr_q8.so (include/uocr_q8.h).

The product path is the CUDA library; there is no CPU fallback.  If the
library is missing, importing the package still works (so CPU-only tooling
can inspect it) but every call raises ``LibraryMissing``.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "libuocr_q8.so")


class LibraryMissing(RuntimeError):
    pass


P = ctypes.c_void_p
S = ctypes.c_size_t
I = ctypes.c_int
F = ctypes.c_float
PP = ctypes.POINTER(ctypes.c_void_p)

# name -> (restype, argtypes); mirrors include/uocr_q8.h one to one.
SIGNATURES = {
    "uocr_abi_version": (I, []),
    "uocr_last_error": (ctypes.c_char_p, []),
    "uocr_status_name": (ctypes.c_char_p, [I]),
    "uocr_ctx_create": (I, [I, S, PP]),
    "uocr_ctx_destroy": (I, [P]),
    "uocr_ctx_set_stream": (I, [P, P]),
    "uocr_ctx_sync": (I, [P]),
    "uocr_ctx_device": (I, [P, ctypes.POINTER(I), ctypes.POINTER(I)]),
    "uocr_ctx_set_wait_limit": (I, [P, ctypes.c_uint64]),
    "uocr_ctx_hold_decode_barrier": (I, [P, I]),
    "uocr_q8_from_parts": (I, [P, S, S, P, S, P, S, PP]),
    "uocr_q8_from_device": (I, [P, S, S, P, P, PP]),
    "uocr_q8_quantize": (I, [P, S, S, P, PP]),
    "uocr_q8_free": (I, [P]),
    "uocr_q8_shape": (I, [P, ctypes.POINTER(S), ctypes.POINTER(S)]),
    "uocr_q8_storage_bytes": (S, [P]),
    "uocr_q8_device_ptrs": (I, [P, PP, PP]),
    "uocr_q8_download": (I, [P, P, P, P]),
    "uocr_q8_dequantize": (I, [P, P, P]),
    "uocr_q8_dequantize_host": (I, [P, P, P, S]),
    "uocr_q8_linear": (I, [P, P, P, S, P]),
    "uocr_q8_linear_host": (I, [P, P, P, P, S, P, S]),
    "uocr_q8_linear_dynamic_int8": (I, [P, P, P, S, P]),
    "uocr_q8_linear_dynamic_int8_host": (I, [P, P, P, P, S, P, S]),
    "uocr_q8_quantize_rows": (I, [P, P, S, S, P, P]),
    "uocr_q8_linear_multi": (I, [P, P, S, I, P, P]),
    "uocr_moe_route": (I, [P, P, S, S, S, I, F, P, P]),
    "uocr_moe_create": (I, [P, P, P, P, P, P, P, S, S, I, F, PP]),
    "uocr_moe_free": (I, [P]),
    "uocr_moe_forward": (I, [P, P, I, P, P, S, P, P, P]),
    "uocr_moe_forward_host": (I, [P, P, I, P, P, S, P, P, P]),
    "uocr_moe_forward_decode_noalloc": (I, [P, P, I, P, P, P]),
    "uocr_moe_expert_rows": (I, [P, P, I, P, P, S, P]),
    "uocr_moe_shared_rows": (I, [P, P, I, P, S, P]),
    "uocr_moe_combine": (I, [P, P, P, P, S, S, S, P]),
    "uocr_moe_dispatch": (I, [P, P, S, S, P, S, P, S, S, P, P, P]),
    "uocr_moe_combine_rows": (I, [P, P, P, P, P, S, S, S, P]),
    "uocr_ep_create": (I, [P, P, S, S, I, F, P, S, S, S, PP]),
    "uocr_ep_free": (I, [P]),
    "uocr_ep_handle": (I, [P, P]),
    "uocr_ep_connect": (I, [P, P]),
    "uocr_ep_connect_local": (I, [P, S]),
    "uocr_ep_set_wait_limit": (I, [P, ctypes.c_uint64]),
    "uocr_ep_forward": (I, [P, P, I, P, P, S, P, P, P]),
    "uocr_ep_forward_host": (I, [P, P, I, P, P, S, P]),
    "uocr_ep_dispatch": (I, [P, P, I, P, P, S, P]),
    "uocr_ep_experts": (I, [P, P]),
    "uocr_ep_combine": (I, [P, P, P, P, P]),
    "uocr_feed_forward": (I, [P, P, P, P, I, P, S, P]),
    "uocr_linear_bf16": (I, [P, P, S, S, P, S, P]),
    "uocr_linear_bf16_tc": (I, [P, P, S, S, P, S, P]),
    "uocr_rms_norm": (I, [P, P, S, S, P, F, P]),
    "uocr_add_rms_norm": (I, [P, P, P, S, S, P, F, P, P]),
    "uocr_rope_create": (I, [P, S, F, S, PP]),
    "uocr_rope_free": (I, [P]),
    "uocr_rope_apply": (I, [P, P, P, P, S, S, P]),
    "uocr_attention_decode": (I, [P, P, P, S, P, S, S, S, P]),
    "uocr_kv_create": (I, [P, S, S, S, S, S, PP]),
    "uocr_kv_free": (I, [P]),
    "uocr_kv_prefill": (I, [P, P, S, P, P, S]),
    "uocr_kv_push": (I, [P, P, P, P]),
    "uocr_kv_rope": (I, [P, P, P, P, P]),
    "uocr_kv_attention": (I, [P, P, P, P]),
    "uocr_kv_attention_prefill": (I, [P, P, S, P, S, P]),
    "uocr_kv_reset": (I, [P, P, S]),
    "uocr_kv_set_attention_form": (I, [P, I]),
    "uocr_bits_checksum": (I, [P, P, S, P]),
    "uocr_attention_prefill": (I, [P, P, P, P, S, S, S, P]),
    "uocr_kv_rope_push_qkv": (I, [P, P, P, P, P]),
    "uocr_kv_state": (I, [P, P, S, ctypes.POINTER(S), ctypes.POINTER(S)]),
    "uocr_kv_export": (I, [P, P, S, P, P, ctypes.POINTER(S)]),
    "uocr_overlay_check": (I, [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(S),
                               ctypes.POINTER(S)]),
    "uocr_overlay_load": (I, [P, ctypes.c_char_p, ctypes.c_char_p, PP]),
    "uocr_overlay_get": (I, [P, ctypes.c_char_p, PP]),
    "uocr_overlay_count": (S, [P]),
    "uocr_overlay_name": (ctypes.c_char_p, [P, S]),
    "uocr_overlay_device_bytes": (S, [P]),
    "uocr_overlay_free": (I, [P]),
    "uocr_sha256_file": (I, [ctypes.c_char_p, ctypes.c_char_p]),
}

_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LibraryMissing(
                f"{LIB_PATH} is not built; run `make -C {PKG_DIR}` or __graft_entry__.build()")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list:
    return sorted(SIGNATURES)
