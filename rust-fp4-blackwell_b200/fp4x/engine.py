"""Python mirror of the decode-engine part of the C ABI (llama_model_*,
llama_forward, llama_decode_step, llama_generate).  Host buffers are numpy
arrays; the model lives on the current CUDA device."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import check, lib

TINYLLAMA = dict(n_layers=22, dim=2048, ffn=5632, n_heads=32, n_kv_heads=4, head_dim=64, vocab=32000,
                 max_seq=2048, rope_theta=10000.0, eps=1e-5, seed=0x5EED)
LLAMA3_8B = dict(n_layers=32, dim=4096, ffn=14336, n_heads=32, n_kv_heads=8, head_dim=128, vocab=128256,
                 max_seq=8192, rope_theta=500000.0, eps=1e-5, seed=0x5EED)


class Config(C.Structure):
    _fields_ = [
        ("n_layers", C.c_uint32), ("dim", C.c_uint32), ("ffn", C.c_uint32),
        ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
        ("vocab", C.c_uint32), ("max_seq", C.c_uint32),
        ("rope_theta", C.c_float), ("eps", C.c_float), ("seed", C.c_uint64),
        ("tp_rank", C.c_uint32), ("tp_size", C.c_uint32),
    ]


_u8p = C.POINTER(C.c_uint8)
_u16p = C.POINTER(C.c_uint16)
_u32p = C.POINTER(C.c_uint32)
_f32p = C.POINTER(C.c_float)

SIGNATURES = {
    "llama_model_create": (C.c_int, [C.POINTER(Config), C.POINTER(C.c_void_p)]),
    "llama_model_destroy": (C.c_int, [C.c_void_p]),
    "llama_model_reset": (C.c_int, [C.c_void_p, C.c_void_p]),
    "llama_forward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, _u32p, _f32p]),
    "llama_decode_step": (C.c_int, [C.c_void_p, C.c_void_p]),
    "llama_generate": (C.c_int, [C.c_void_p, C.c_void_p, _u32p, C.c_uint32, C.c_uint32, _u32p, _f32p, _f32p]),
    "llama_model_export_tensor": (C.c_int, [C.c_void_p, C.c_uint32, _u8p, _u8p, _u32p, _u32p]),
    "llama_model_embedding": (C.c_int, [C.c_void_p, _u16p]),
    "llama_model_weight_bytes": (C.c_size_t, [C.c_void_p]),
    "llama_model_kernels_per_token": (C.c_uint32, [C.c_void_p]),
    "llama_decode_steps": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32]),
    "llama_model_set_path": (C.c_int, [C.c_void_p, C.c_int]),
    "llama_model_get_path": (C.c_int, [C.c_void_p]),
    "llama_model_tp_handle": (C.c_int, [C.c_void_p, C.c_void_p]),
    "llama_model_tp_connect": (C.c_int, [C.c_void_p, C.c_void_p]),
    "llama_model_shard": (C.c_int, [C.c_void_p, _u32p, _u32p]),
    "llama_model_create_from_safetensors": (C.c_int, [C.POINTER(Config), C.c_char_p, C.POINTER(C.c_void_p)]),
    "fp4x_safetensors_info": (C.c_int, [C.c_char_p, C.c_char_p, _u32p, C.POINTER(C.c_uint64), _u32p]),
    "llama_batch_create": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(C.c_void_p)]),
    "llama_batch_destroy": (C.c_int, [C.c_void_p]),
    "llama_batch_prefill": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, _u32p, C.c_uint32]),
    "llama_batch_set_length": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32]),
    "llama_batch_decode": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32]),
    "llama_batch_tokens": (C.c_int, [C.c_void_p, C.c_uint32, _u32p, C.c_uint32, _u32p]),
    "llama_batch_logits": (C.c_int, [C.c_void_p, _f32p, _u32p]),
    "llama_batch_kv_bytes": (C.c_size_t, [C.c_void_p]),
    "llama_batch_tp_handle": (C.c_int, [C.c_void_p, C.c_void_p]),
    "llama_batch_tp_connect": (C.c_int, [C.c_void_p, C.c_void_p]),
}


def _declare():
    L = lib()
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


def _p(a, ct):
    return a.ctypes.data_as(C.POINTER(ct))


class Model:
    """A random-init Llama-shape MXFP4 model on the current CUDA device."""

    def __init__(self, cfg: dict, stream: int | None = None, safetensors: str | None = None):
        """Random-init weights from cfg["seed"], or the checkpoint at `safetensors`
        (llama_model_create_from_safetensors; Hugging Face Llama tensor names)."""
        self.L = _declare()
        self.cfg = dict(cfg)
        c = Config(**{k: self.cfg.get(k, 0) for k, _ in Config._fields_})
        if c.tp_size == 0:
            c.tp_size = 1
        self._c = c
        h = C.c_void_p()
        if safetensors is None:
            check(self.L.llama_model_create(C.byref(c), C.byref(h)))
        else:
            check(self.L.llama_model_create_from_safetensors(C.byref(c), str(safetensors).encode(), C.byref(h)))
        self._h = h
        self.stream = stream

    def close(self):
        if getattr(self, "_h", None):
            self.L.llama_model_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _st(self):
        if self.stream is not None:
            return self.stream
        import torch
        return torch.cuda.current_stream().cuda_stream

    def reset(self):
        check(self.L.llama_model_reset(self._h, self._st()))

    def shard(self):
        """(v0, vocab_local): the lm_head rows this rank holds (the whole vocab without TP)."""
        v0, nv = C.c_uint32(0), C.c_uint32(0)
        check(self.L.llama_model_shard(self._h, C.byref(v0), C.byref(nv)))
        return v0.value, nv.value

    def tp_handle(self) -> bytes:
        """64-byte IPC handle of this rank's exchange area (tensor parallel)."""
        buf = C.create_string_buffer(64)
        check(self.L.llama_model_tp_handle(self._h, buf))
        return buf.raw

    def tp_connect(self, handles):
        """Map every rank's exchange area (handles in rank order) and build the graph."""
        blob = C.create_string_buffer(b"".join(handles), 64 * len(handles))
        check(self.L.llama_model_tp_connect(self._h, blob))

    def forward(self, token: int, pos: int, want_logits: bool = True):
        """Next token and logits (this rank's vocab slice under tensor parallelism)."""
        nxt = np.zeros(1, np.uint32)
        logits = np.empty(self.shard()[1], np.float32) if want_logits else None
        check(self.L.llama_forward(self._h, self._st(), token, pos, _p(nxt, C.c_uint32),
                                   _p(logits, C.c_float) if want_logits else None))
        return int(nxt[0]), logits

    def decode_step(self):
        check(self.L.llama_decode_step(self._h, self._st()))

    def decode_steps(self, n: int):
        check(self.L.llama_decode_steps(self._h, self._st(), n))

    @property
    def path(self) -> str:
        return {0: "graph", 1: "persistent", 2: "tensor"}[self.L.llama_model_get_path(self._h)]

    def set_path(self, path: str):
        check(self.L.llama_model_set_path(self._h, {"graph": 0, "persistent": 1, "tensor": 2}[path]))

    def generate(self, prompt, n_gen: int):
        prompt = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(n_gen, np.uint32)
        pre, dec = C.c_float(0), C.c_float(0)
        check(self.L.llama_generate(self._h, self._st(), _p(prompt, C.c_uint32), len(prompt), n_gen,
                                    _p(out, C.c_uint32), C.byref(pre), C.byref(dec)))
        return out, pre.value, dec.value

    def export_tensor(self, tensor_id: int):
        n, k = C.c_uint32(0), C.c_uint32(0)
        check(self.L.llama_model_export_tensor(self._h, tensor_id, None, None, C.byref(n), C.byref(k)))
        packed = np.empty((n.value, k.value // 2), np.uint8)
        scales = np.empty((n.value, k.value // 32), np.uint8)
        check(self.L.llama_model_export_tensor(self._h, tensor_id, _p(packed, C.c_uint8), _p(scales, C.c_uint8),
                                               None, None))
        return packed, scales

    def embedding(self):
        e = np.empty((self.cfg["vocab"], self.cfg["dim"]), np.uint16)
        check(self.L.llama_model_embedding(self._h, _p(e, C.c_uint16)))
        return e

    def kernels_per_token(self) -> int:
        return int(self.L.llama_model_kernels_per_token(self._h))

    def weight_bytes(self) -> int:
        return int(self.L.llama_model_weight_bytes(self._h))


class Batch:
    """Batched engine over a Model's weights (llama_batch_*): `rows` sequences
    with their own KV caches, decoded together; prompts prefilled `rows` tokens
    per pass.  Every linear runs on the tcgen05 fp4_mma GEMM."""

    def __init__(self, model: Model, rows: int):
        self.m = model
        self.L = model.L
        self.rows = rows
        h = C.c_void_p()
        check(self.L.llama_batch_create(model._h, rows, C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self.L.llama_batch_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prefill(self, seq: int, tokens):
        t = np.ascontiguousarray(tokens, np.uint32)
        check(self.L.llama_batch_prefill(self._h, self.m._st(), seq, _p(t, C.c_uint32), len(t)))

    def set_length(self, seq: int, length: int, next_token: int = 0):
        check(self.L.llama_batch_set_length(self._h, self.m._st(), seq, length, next_token))

    def decode(self, n_steps: int):
        check(self.L.llama_batch_decode(self._h, self.m._st(), n_steps))

    def tokens(self, seq: int):
        n = C.c_uint32(0)
        check(self.L.llama_batch_tokens(self._h, seq, None, 0, C.byref(n)))
        out = np.zeros(n.value, np.uint32)
        check(self.L.llama_batch_tokens(self._h, seq, _p(out, C.c_uint32), n.value, None))
        return out

    def logits(self):
        r = C.c_uint32(0)
        check(self.L.llama_batch_logits(self._h, None, C.byref(r)))
        out = np.empty((r.value, self.m.shard()[1]), np.float32)
        check(self.L.llama_batch_logits(self._h, _p(out, C.c_float), None))
        return out

    def kv_bytes(self) -> int:
        return int(self.L.llama_batch_kv_bytes(self._h))

    def tp_handle(self) -> bytes:
        """64-byte IPC handle of this rank's batch exchange area (tensor parallel)."""
        buf = C.create_string_buffer(64)
        check(self.L.llama_batch_tp_handle(self._h, buf))
        return buf.raw

    def tp_connect(self, handles):
        """Map every rank's batch exchange area (handles in rank order)."""
        blob = C.create_string_buffer(b"".join(handles), 64 * len(handles))
        check(self.L.llama_batch_tp_connect(self._h, blob))


def safetensors_info(path: str, name: str):
    """(dtype tag, shape) of one tensor of a safetensors file (host only)."""
    L = _declare()
    dt, nd = C.c_uint32(0), C.c_uint32(0)
    shape = (C.c_uint64 * 8)()
    check(L.fp4x_safetensors_info(str(path).encode(), name.encode(), C.byref(dt), shape, C.byref(nd)))
    tag = {0: "F32", 1: "BF16", 2: "F16"}.get(C.c_int32(dt.value).value, "other")
    return tag, tuple(int(shape[i]) for i in range(nd.value))
