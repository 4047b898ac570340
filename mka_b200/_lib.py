"""ctypes binding of libfastmka_b200.so, the C ABI declared in include/fastmka_b200.h.

The library is built in-tree (python -m mka_b200.build). Loading fails loudly when
it is missing: there is no CPU or PyTorch fallback for any op.
"""
from __future__ import annotations

import ctypes
import os
import threading
from ctypes import c_float, c_int, c_int64, c_size_t, c_uint32, c_void_p, POINTER
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfastmka_b200.so"

_P = c_void_p
_I = c_int
_L = c_int64
_F = c_float

# name -> (restype, argtypes); mirrors include/fastmka_b200.h
_SIGNATURES = {
    "fmka_version": (ctypes.c_char_p, []),
    "fmka_get_last_error": (_I, [ctypes.c_char_p, _I]),
    "fmka_device_status": (_I, [POINTER(c_uint32), _I, _P]),
    "fmka_num_sms": (_I, []),
    "fmka_gemm_bf16": (_I, [_P, _L, _P, _L, _P, _P, _L, _I, _I, _I, _P]),
    "fmka_gemm_bf16_kblocked": (_I, [_P, _I, _L, _L, _P, _L, _P, _P, _L, _I, _I, _I, _P]),
    "fmka_gemm_bf16_swiglu": (_I, [_P, _L, _P, _L, _P, _P, _L, _I, _I, _I, _P]),
    "fmka_qr_proj": (_I, [_P, _L, _P, _L, _P, _I, _I, _I, _I, _I, _P, _L, _L, _L, _I,
                          _P, _P, _L, _L, _P, _I, _I, _P, _P]),
    "fmka_kv_proj": (_I, [_P, _L, _P, _L, _P, _I, _I, _I, _I, _P, _P, _L, _L, _L, _I,
                          _P, _P, _L, _L, _P]),
    "fmka_route_ema_blend_workspace_size": (c_size_t, [_I, _I, _I]),
    "fmka_route_ema_blend": (_I, [_P, _L, _L, _P, _P, _P, _I, _P, _L, _L, _I, _F, _I, _I, _I,
                                  _P, _L, _L, _P, _P, c_size_t, _P]),
    "fmka_route_ema_blend_noalloc": (_I, [_P, _L, _L, _P, _P, _P, _I, _P, _L, _L, _I, _F, _I, _I, _I,
                                          _P, _L, _L, _P, _P]),
    "fmka_route_ema_blend_noalloc_scratch_bytes": (c_size_t, []),
    "fmka_route_ema_blend_state": (_I, [_P, _L, _L, _P, _P, _P, _I, _P, _L, _L, _I, _F, _I, _I, _I,
                                        _P, _L, _L, _P, _P, _P, _P, c_size_t, _P]),
    "fmka_route_ema_blend_kv_workspace_size": (c_size_t, [_I, _I, _I]),
    "fmka_route_ema_blend_kv": (_I, [_P, _L, _L, _P, _P, _P, _L, _L, _I, _F, _I, _I, _I, _P, _P, _P, _L, _L, _L, _I, _P, _P,
                                     _L, _L, _P, _P, _P, _P, c_size_t, _P]),
    "fmka_route_blend": (_I, [_P, _L, _L, _P, _L, _L, _P, _L, _L, _I, _P, _I, _I, _I, _I, _P, _L, _L, _P]),
    "fmka_attn_fwd_prefill": (_I, [_P, _L, _L, _L, _P, _P, _L, _L, _L, _P, _L, _L, _L, _P, _L, _L,
                                   _I, _I, _I, _I, _I, _I, _I, _F, _P]),
    "fmka_attn_fwd_prefill_scatter": (_I, [_P, _L, _L, _L, _P, _P, _L, _L, _L, _P, _I, _I, _L, _L, _L,
                                           _I, _I, _I, _I, _I, _I, _I, _F, _P]),
    "fmka_gemm_bf16_kblocked_scatter": (_I, [_P, _I, _L, _L, _P, _L, _P, _P, _I, _L, _L, _I, _I, _I, _P]),
    "fmka_peer_alloc": (_I, [c_size_t, POINTER(_P)]),
    "fmka_peer_free": (_I, [_P]),
    "fmka_peer_export": (_I, [_P, _P]),
    "fmka_peer_import": (_I, [_P, POINTER(_P)]),
    "fmka_peer_close": (_I, [_P]),
    "fmka_peer_barrier": (_I, [_P, _I, _I, c_uint32, _P]),
    "fmka_rmsnorm_bf16": (_I, [_P, _L, _P, _F, _P, _L, _I, _I, _P]),
    "fmka_silu_mul_bf16": (_I, [_P, _P, _P, _L, _P]),
    "fmka_gemm_bf16_f32out": (_I, [_P, _L, _P, _L, _P, _L, _I, _I, _I, _P]),
    "fmka_l3_block_mean_bf16": (_I, [_P, _L, _L, _I, _I, _I, _I, _P, _L, _P]),
    "fmka_l3_topr_f32": (_I, [_P, _L, _I, _I, _I, _F, _P, _P, _P]),
    "fmka_l3_recall_gather_bf16": (_I, [_P, _P, _I, _P, _L, _I, _I, _I, _I, _I, _P, _L, _L, _P]),
    "fmka_attn_decode_num_splits": (_I, [_I, _I, _I]),
    "fmka_attn_decode_workspace_size": (c_size_t, [_I, _I, _I, _I, _I]),
    "fmka_attn_decode_splitkv": (_I, [_P, _L, _L, _P, _P, _L, _L, _L, _P, _L, _L, _P, _L,
                                      _I, _I, _I, _I, _I, _F, _I, _P, c_size_t, _P]),
}

_lib = None
_lock = threading.Lock()


class FastMKAError(RuntimeError):
    """Raised when a C-ABI entry point returns a nonzero status."""


def load() -> ctypes.CDLL:
    """Loads the library once and declares every exported entry point."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise FastMKAError(
                f"{LIB_PATH.name} is not built; run `python -m mka_b200.build` "
                "(the FastMKA B200 ops have no fallback)")
        lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_LOCAL)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def last_error() -> tuple[int, str]:
    lib = load()
    buf = ctypes.create_string_buffer(512)
    code = lib.fmka_get_last_error(buf, 512)
    return code, buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != 0:
        code, msg = last_error()
        raise FastMKAError(f"{what} failed (status {rc}): {msg}")


def call(name: str, *args) -> None:
    """Calls a status-returning entry point and raises FastMKAError on failure."""
    rc = getattr(load(), name)(*args)
    check(rc, name)
