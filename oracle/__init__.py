"""CPU oracle for the MXFP4 decode path (test infrastructure only).

This package loads ``liboracle.so`` (built from ``oracle.c`` by ``build()``) and
wraps it with numpy-friendly helpers.  It is the checker the CUDA path is
compared against.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg import it; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
LIB = BUILD / "liboracle.so"

_lib = None


def build(force: bool = False) -> Path:
    """Compile oracle.c with gcc -O2 -ffp-contract=off -fopenmp into _build/liboracle.so."""
    src = HERE / "oracle.c"
    if LIB.exists() and not force and LIB.stat().st_mtime >= max(
        src.stat().st_mtime, (HERE / "oracle.h").stat().st_mtime
    ):
        return LIB
    BUILD.mkdir(exist_ok=True)
    tmp = BUILD / f"liboracle.{os.getpid()}.so"
    cmd = [
        "gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-std=c11",
        "-fPIC", "-shared", "-Wall", "-o", str(tmp), str(src), "-lm",
    ]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(str(LIB))
        _declare(_lib)
    return _lib


_u8p = C.POINTER(C.c_uint8)
_u16p = C.POINTER(C.c_uint16)
_u32p = C.POINTER(C.c_uint32)
_f32p = C.POINTER(C.c_float)


class Config(C.Structure):
    _fields_ = [
        ("n_layers", C.c_uint32), ("dim", C.c_uint32), ("ffn", C.c_uint32),
        ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
        ("vocab", C.c_uint32), ("max_seq", C.c_uint32),
        ("rope_theta", C.c_float), ("eps", C.c_float), ("seed", C.c_uint64),
    ]


def _declare(L):
    sig = {
        "orc_xorshift32_fill": (None, [C.c_uint32, _u32p, C.c_size_t]),
        "orc_hash64": (C.c_uint64, [C.c_uint64, C.c_uint64]),
        "orc_normal": (C.c_float, [C.c_uint64, C.c_uint64, C.c_float]),
        "orc_fill_normal": (None, [C.c_uint64, C.c_uint64, C.c_float, _f32p, C.c_size_t]),
        "orc_fill_normal_bf16": (None, [C.c_uint64, C.c_uint64, C.c_float, _u16p, C.c_size_t]),
        "orc_fill_uniform_ids": (None, [C.c_uint64, C.c_uint32, _u32p, C.c_size_t]),
        "orc_e2m1_decode": (C.c_float, [C.c_uint32]),
        "orc_bf16_to_f32": (C.c_float, [C.c_uint16]),
        "orc_f32_to_bf16": (C.c_uint16, [C.c_float]),
        "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
        "orc_e8m0_from_amax": (C.c_uint8, [C.c_float]),
        "orc_e8m0_to_f32": (C.c_float, [C.c_uint8]),
        "orc_e2m1_nearest": (C.c_uint32, [C.c_float]),
        "orc_quant_ref": (None, [_f32p, C.c_size_t, C.c_size_t, _u32p, _f32p]),
        "orc_quant_mxfp4": (None, [_f32p, C.c_size_t, C.c_size_t, _u8p, _u8p]),
        "orc_dequant_mxfp4": (None, [_u8p, _u8p, C.c_size_t, C.c_size_t, _f32p]),
        "orc_gemv_ref": (None, [C.c_uint32, C.c_uint32, _u32p, _f32p, _f32p, _f32p, C.c_int]),
        "orc_gemv_mxfp4": (None, [C.c_uint32, C.c_uint32, _u8p, _u8p, _f32p, _f32p, C.c_int]),
        "orc_gemv_mxfp4_bf16x": (None, [C.c_uint32, C.c_uint32, _u8p, _u8p, _u16p, _f32p, C.c_int]),
        "orc_rmsnorm": (None, [C.c_uint32, C.c_float, _f32p, _f32p, _f32p]),
        "orc_rope_tables": (None, [C.c_uint32, C.c_uint32, C.c_double, _f32p, _f32p]),
        "orc_rope": (None, [C.c_uint32, C.c_uint32, C.c_uint32, _f32p, _f32p, _f32p]),
        "orc_copy_into": (None, [C.c_uint32, C.c_uint32, _f32p, _f32p]),
        "orc_attn_decode": (None, [C.c_uint32] * 4 + [_f32p, _f32p, _f32p, _f32p, C.c_int]),
        "orc_attn_decode_bf16": (None, [C.c_uint32] * 6 + [_u16p, _u16p, _u16p, _u16p, C.c_int]),
        "orc_swiglu": (None, [C.c_uint32, _f32p, _f32p, _f32p]),
        "orc_residual": (None, [C.c_uint32, _f32p, _f32p]),
        "orc_argmax": (C.c_uint32, [C.c_uint32, _f32p]),
        "orc_mma_mxf4": (None, [C.c_uint32] * 3 + [_u8p, _u8p, _u8p, _u8p, _f32p, C.c_int]),
        "orc_model_create": (C.c_void_p, [C.POINTER(Config), C.c_int]),
        "orc_model_destroy": (None, [C.c_void_p]),
        "orc_model_packed": (_u8p, [C.c_void_p, C.c_uint32]),
        "orc_model_scales": (_u8p, [C.c_void_p, C.c_uint32]),
        "orc_model_embed": (_u16p, [C.c_void_p]),
        "orc_model_set_tensor": (None, [C.c_void_p, C.c_uint32, _u8p, _u8p]),
        "orc_ue4m3_to_f32": (C.c_float, [C.c_uint8]),
        "orc_f32_to_ue4m3": (C.c_uint8, [C.c_float]),
        "orc_quant_nvfp4": (None, [_f32p, C.c_size_t, C.c_size_t, _u8p, _u8p, C.c_float]),
        "orc_mma_nvf4": (None, [C.c_uint32, C.c_uint32, C.c_uint32, _u8p, _u8p, _u8p, _u8p, C.c_float, _f32p,
                                C.c_int]),
        "orc_model_set_embed": (None, [C.c_void_p, _u16p]),
        "orc_model_set_norm": (None, [C.c_void_p, C.c_uint32, _f32p]),
        "orc_forward": (C.c_uint32, [C.c_void_p, C.c_uint32, C.c_uint32, _f32p]),
        "orc_generate": (None, [C.c_void_p, _u32p, C.c_uint32, C.c_uint32, _u32p]),
        "orc_max_threads": (C.c_int, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p(a: np.ndarray, ctype):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(C.POINTER(ctype))


# ------------------------------------------------------------------ RNG

def xorshift32(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint32)
    lib().orc_xorshift32_fill(seed, _p(out, C.c_uint32), n)
    return out


def hash64(seed: int, i: int) -> int:
    return int(lib().orc_hash64(seed, i))


def normal(seed: int, n: int, sigma: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_fill_normal(seed, offset, sigma, _p(out, C.c_float), n)
    return out


def normal_bf16(seed: int, n: int, sigma: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().orc_fill_normal_bf16(seed, offset, sigma, _p(out, C.c_uint16), n)
    return out


def uniform_ids(seed: int, vocab: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint32)
    lib().orc_fill_uniform_ids(seed, vocab, _p(out, C.c_uint32), n)
    return out


# -------------------------------------------------------------- formats

def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (vectorised twin of orc_f32_to_bf16)."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x007FFFFF) != 0)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r.reshape(a.shape)


def quant_mxfp4(w: np.ndarray):
    w = np.ascontiguousarray(w, np.float32)
    n, k = w.shape
    packed = np.empty((n, k // 2), np.uint8)
    scales = np.empty((n, k // 32), np.uint8)
    lib().orc_quant_mxfp4(_p(w, C.c_float), n, k, _p(packed, C.c_uint8), _p(scales, C.c_uint8))
    return packed, scales


def quant_ref(w: np.ndarray):
    w = np.ascontiguousarray(w, np.float32)
    n, k = w.shape
    packed = np.empty((n, k // 8), np.uint32)
    scales = np.empty((n, k // 32), np.float32)
    lib().orc_quant_ref(_p(w, C.c_float), n, k, _p(packed, C.c_uint32), _p(scales, C.c_float))
    return packed, scales


def dequant_mxfp4(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    n = packed.shape[0]
    k = packed.shape[1] * 2
    out = np.empty((n, k), np.float32)
    lib().orc_dequant_mxfp4(_p(np.ascontiguousarray(packed), C.c_uint8),
                            _p(np.ascontiguousarray(scales), C.c_uint8), n, k, _p(out, C.c_float))
    return out


# ------------------------------------------------------------------ ops

def gemv_ref(w: np.ndarray, scales: np.ndarray, x: np.ndarray, threads: int = 0) -> np.ndarray:
    n = w.shape[0]
    k = x.shape[0]
    y = np.empty(n, np.float32)
    lib().orc_gemv_ref(n, k, _p(np.ascontiguousarray(w, np.uint32), C.c_uint32),
                       _p(np.ascontiguousarray(scales, np.float32), C.c_float),
                       _p(np.ascontiguousarray(x, np.float32), C.c_float), _p(y, C.c_float), threads)
    return y


def gemv_mxfp4(packed, scales, x, threads: int = 0) -> np.ndarray:
    n = packed.shape[0]
    k = packed.shape[1] * 2
    y = np.empty(n, np.float32)
    packed = np.ascontiguousarray(packed, np.uint8)
    scales = np.ascontiguousarray(scales, np.uint8)
    if x.dtype == np.uint16:
        lib().orc_gemv_mxfp4_bf16x(n, k, _p(packed, C.c_uint8), _p(scales, C.c_uint8),
                                   _p(np.ascontiguousarray(x), C.c_uint16), _p(y, C.c_float), threads)
    else:
        lib().orc_gemv_mxfp4(n, k, _p(packed, C.c_uint8), _p(scales, C.c_uint8),
                             _p(np.ascontiguousarray(x, np.float32), C.c_float), _p(y, C.c_float), threads)
    return y


def rmsnorm(x, w, eps=1e-5):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty_like(x)
    lib().orc_rmsnorm(x.shape[0], eps, _p(x, C.c_float), _p(w, C.c_float), _p(y, C.c_float))
    return y


def rope_tables(n_pos, head_dim, theta):
    c = np.empty((n_pos, head_dim // 2), np.float32)
    s = np.empty((n_pos, head_dim // 2), np.float32)
    lib().orc_rope_tables(n_pos, head_dim, float(theta), _p(c, C.c_float), _p(s, C.c_float))
    return c, s


def rope(q, num_heads, head_dim, cos_base, cos_t, sin_t):
    q = np.array(q, np.float32, copy=True)
    lib().orc_rope(num_heads, head_dim, cos_base, _p(np.ascontiguousarray(cos_t, np.float32), C.c_float),
                   _p(np.ascontiguousarray(sin_t, np.float32), C.c_float), _p(q, C.c_float))
    return q


def attn_decode(q, kc, vc, n_heads, n_kv, head_dim, seq, threads=0):
    out = np.empty(n_heads * head_dim, np.float32)
    lib().orc_attn_decode(n_heads, n_kv, head_dim, seq,
                          _p(np.ascontiguousarray(q, np.float32), C.c_float),
                          _p(np.ascontiguousarray(kc, np.float32), C.c_float),
                          _p(np.ascontiguousarray(vc, np.float32), C.c_float), _p(out, C.c_float), threads)
    return out


def attn_decode_bf16(q, kc, vc, batch, n_heads, n_kv, head_dim, seq, max_seq, threads=0):
    out = np.empty((batch, n_heads, head_dim), np.uint16)
    lib().orc_attn_decode_bf16(batch, n_heads, n_kv, head_dim, seq, max_seq,
                               _p(np.ascontiguousarray(q, np.uint16), C.c_uint16),
                               _p(np.ascontiguousarray(kc, np.uint16), C.c_uint16),
                               _p(np.ascontiguousarray(vc, np.uint16), C.c_uint16),
                               _p(out, C.c_uint16), threads)
    return out


def swiglu(g, u):
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    out = np.empty_like(g)
    lib().orc_swiglu(g.shape[0], _p(g, C.c_float), _p(u, C.c_float), _p(out, C.c_float))
    return out


def residual(y, x):
    x = np.array(x, np.float32, copy=True)
    lib().orc_residual(x.shape[0], _p(np.ascontiguousarray(y, np.float32), C.c_float), _p(x, C.c_float))
    return x


def argmax(logits) -> int:
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_argmax(logits.shape[0], _p(logits, C.c_float)))


def mma_mxf4(a, sa, w, sw, threads=0):
    m = a.shape[0]
    n = w.shape[0]
    k = a.shape[1] * 2
    d = np.empty((m, n), np.float32)
    lib().orc_mma_mxf4(m, n, k, _p(np.ascontiguousarray(a, np.uint8), C.c_uint8),
                       _p(np.ascontiguousarray(sa, np.uint8), C.c_uint8),
                       _p(np.ascontiguousarray(w, np.uint8), C.c_uint8),
                       _p(np.ascontiguousarray(sw, np.uint8), C.c_uint8), _p(d, C.c_float), threads)
    return d


# ---------------------------------------------------------------- NVFP4

def ue4m3_to_f32(b: int) -> float:
    return float(lib().orc_ue4m3_to_f32(int(b)))


def f32_to_ue4m3(s: float) -> int:
    return int(lib().orc_f32_to_ue4m3(float(s)))


def quant_nvfp4(w: np.ndarray, g: float = 1.0):
    """f32 [n][k] -> (packed [n][k/2], UE4M3 scales [n][k/16]) with per-tensor scale g."""
    w = np.ascontiguousarray(w, np.float32)
    n, k = w.shape
    packed = np.empty((n, k // 2), np.uint8)
    scales = np.empty((n, k // 16), np.uint8)
    lib().orc_quant_nvfp4(_p(w, C.c_float), n, k, _p(packed, C.c_uint8), _p(scales, C.c_uint8), g)
    return packed, scales


def mma_nvf4(a, sa, w, sw, alpha: float = 1.0, threads: int = 0):
    m, n, k = a.shape[0], w.shape[0], a.shape[1] * 2
    d = np.empty((m, n), np.float32)
    lib().orc_mma_nvf4(m, n, k, _p(np.ascontiguousarray(a, np.uint8), C.c_uint8),
                       _p(np.ascontiguousarray(sa, np.uint8), C.c_uint8), _p(np.ascontiguousarray(w, np.uint8), C.c_uint8),
                       _p(np.ascontiguousarray(sw, np.uint8), C.c_uint8), alpha, _p(d, C.c_float), threads)
    return d


# ---------------------------------------------------------------- model

class Model:
    """Random-init reference model (same tensor seeds as the device initialiser)."""

    def __init__(self, cfg: dict, threads: int = 0):
        self.cfg = dict(cfg)
        self._c = Config(**{k: cfg[k] for k, _ in Config._fields_})
        self._h = lib().orc_model_create(C.byref(self._c), threads)

    def close(self):
        if self._h:
            lib().orc_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, token: int, pos: int):
        if not (0 <= pos < self.cfg["max_seq"] and 0 <= token < self.cfg["vocab"]):
            raise ValueError(f"position {pos} / token {token} outside the model")
        logits = np.empty(self.cfg["vocab"], np.float32)
        nxt = lib().orc_forward(self._h, token, pos, _p(logits, C.c_float))
        return int(nxt), logits

    def generate(self, prompt, n_gen):
        prompt = np.ascontiguousarray(prompt, np.uint32)
        out = np.empty(n_gen, np.uint32)
        lib().orc_generate(self._h, _p(prompt, C.c_uint32), len(prompt), n_gen, _p(out, C.c_uint32))
        return out

    def tensor(self, tensor_id: int, n: int, k: int):
        p = lib().orc_model_packed(self._h, tensor_id)
        s = lib().orc_model_scales(self._h, tensor_id)
        packed = np.ctypeslib.as_array(p, shape=(n * k // 2,)).reshape(n, k // 2).copy()
        scales = np.ctypeslib.as_array(s, shape=(n * k // 32,)).reshape(n, k // 32).copy()
        return packed, scales

    def set_tensor(self, tensor_id: int, packed, scales):
        """Replace a linear (canonical MXFP4 layout) -- checkpoint-loader tests."""
        lib().orc_model_set_tensor(self._h, tensor_id, _p(np.ascontiguousarray(packed, np.uint8), C.c_uint8),
                                   _p(np.ascontiguousarray(scales, np.uint8), C.c_uint8))

    def set_embed(self, embed_bf16):
        lib().orc_model_set_embed(self._h, _p(np.ascontiguousarray(embed_bf16, np.uint16), C.c_uint16))

    def set_norm(self, which: int, w):
        """which: 0..L-1 attention norm, L..2L-1 FFN norm, 2L final norm."""
        lib().orc_model_set_norm(self._h, which, _p(np.ascontiguousarray(w, np.float32), C.c_float))

    def embed(self):
        p = lib().orc_model_embed(self._h)
        n = self.cfg["vocab"] * self.cfg["dim"]
        return np.ctypeslib.as_array(p, shape=(n,)).reshape(self.cfg["vocab"], self.cfg["dim"]).copy()


def max_threads() -> int:
    return int(lib().orc_max_threads())
