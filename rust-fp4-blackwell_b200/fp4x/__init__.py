"""Python mirror of the fp4x C ABI (include/fp4x.h).

The product is ``libfp4x.so``: hand-written sm_100a CUDA kernels behind an
``extern "C"`` boundary.  This module only loads that library with ctypes and
passes torch CUDA tensors to it as raw device pointers, on the current torch
stream.  There is no CPU fallback: if the library cannot be built or loaded, or
no CUDA device is present, every operator raises.

Operator names follow the reference's kernel API (examples/llama_run/src/main.rs:
fp4_gemv, rmsnorm, rope, copy_into, attn_decode, swiglu, residual, argmax).
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

from . import _build

__all__ = ["lib", "Fp4xError", "build"]

_lib = None


class Fp4xError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"fp4x status {status}: {msg}")
        self.status = status


def build(force: bool = False) -> Path:
    return _build.build(force=force)


_vp = C.c_void_p
_u32 = C.c_uint32
_u64 = C.c_uint64
_f32 = C.c_float
_sz = C.c_size_t

# name -> (restype, argtypes); pointers are passed as c_void_p
SIGNATURES = {
    "fp4x_last_error": (C.c_char_p, []),
    "fp4x_version": (C.c_char_p, []),
    "fp4x_device_error": (C.c_int, [_vp, C.POINTER(_u32)]),
    "fp4x_set_wait_limit": (C.c_int, [_u32]),
    "fp4_quantize_mxfp4": (C.c_int, [_vp, _u32, _u32, _vp, _vp, _vp]),
    "fp4_quantize_ref": (C.c_int, [_vp, _u32, _u32, _vp, _vp, _vp]),
    "fp4_dequantize_mxfp4": (C.c_int, [_vp, _u32, _u32, _vp, _vp, _vp]),
    "fp4x_fill_normal_f32": (C.c_int, [_vp, _u64, _u64, _f32, _vp, _sz]),
    "fp4x_fill_normal_bf16": (C.c_int, [_vp, _u64, _u64, _f32, _vp, _sz]),
    "fp4x_init_mxfp4": (C.c_int, [_vp, _u64, _f32, _u32, _u32, _vp, _vp]),
    "fp4_gemv": (C.c_int, [_vp, _u32, _u32, _vp, _vp, _vp, _vp]),
    "fp4_gemv_ref": (C.c_int, [_vp, _u32, _u32, _vp, _vp, _vp, _vp]),
    "fp4_gemv_f32x": (C.c_int, [_vp, _u32, _u32, _vp, _vp, _vp, _vp]),
    "fp4_mma_workspace_size": (_sz, [_u32, _u32, _u32]),
    "fp4_mma": (C.c_int, [_vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fp4_mma_f32": (C.c_int, [_vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp]),
    "fp4_mma_nvf4_workspace_size": (_sz, [_u32, _u32, _u32]),
    "fp4_mma_nvf4": (C.c_int, [_vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, C.c_float, _vp, _vp, _sz]),
    "fp4_mma_nvf4_f32": (C.c_int, [_vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, C.c_float, _vp]),
    "fp4_quantize_nvfp4": (C.c_int, [_vp, _u32, _u32, _vp, _vp, _vp, C.c_float]),
    "fp4_mma_allones": (C.c_int, [_vp, _vp]),
    "llama_rmsnorm": (C.c_int, [_vp, _u32, _f32, _vp, _vp, _vp]),
    "llama_rope": (C.c_int, [_vp, _u32, _u32, _u32, _vp, _vp, _vp]),
    "llama_rope_tables": (C.c_int, [_vp, _u32, _u32, C.c_double, _vp, _vp]),
    "llama_copy_into": (C.c_int, [_vp, _u32, _u32, _vp, _vp]),
    "llama_kv_append_bf16": (C.c_int, [_vp, _u32, _u32, _vp, _vp]),
    "llama_swiglu": (C.c_int, [_vp, _u32, _vp, _vp, _vp]),
    "llama_residual": (C.c_int, [_vp, _u32, _vp, _vp]),
    "llama_argmax": (C.c_int, [_vp, _u32, _vp, _vp]),
    "llama_attn_decode": (C.c_int, [_vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp]),
    "llama_attn_decode_hd": (C.c_int, [_vp, _u32, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _sz]),
    "llama_attn_workspace_size": (_sz, [_u32, _u32, _u32, _u32, _u32]),
    "llama_attn_decode_bf16": (C.c_int, [_vp, _u32, _u32, _u32, _u32, _u32, _u32,
                                         _vp, _vp, _vp, _vp, _vp, _sz]),
    "llama_attn_decode_f32q_bf16kv": (C.c_int, [_vp, _u32, _u32, _u32, _u32, _u32, _u32,
                                                _vp, _vp, _vp, _vp, _vp, _sz]),
    "llama_attn_decode_bf16_noalloc": (C.c_int, [_vp, _u32, _u32, _u32, _u32, _u32, _u32, _vp, _vp, _vp, _vp]),
    "llama_attn_noalloc_max_bytes": (_sz, []),
}


def lib():
    """Load (building first if stale) libfp4x.so and declare every C-ABI symbol.
    FP4X_LIB=<path> loads another build of the same library instead (e.g. one
    compiled with extra instrumentation)."""
    global _lib
    if _lib is None:
        import os
        path = os.environ.get("FP4X_LIB") or _build.build()
        L = C.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().fp4x_last_error().decode()


def check(status: int) -> None:
    if status != 0:
        raise Fp4xError(status, last_error())


from . import ops  # noqa: E402,F401  (torch-facing wrappers)
from . import engine  # noqa: E402,F401  (decode engine)

EXTRA_SIGNATURES = engine.SIGNATURES
