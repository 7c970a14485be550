"""Checkpoint helpers for llama_model_create_from_safetensors: the Hugging Face
Llama tensor names the loader reads, and a minimal safetensors writer (numpy only)
for producing checkpoints from arrays.

Format: 8-byte little-endian header length, a JSON header mapping each tensor
name to {"dtype", "shape", "data_offsets"} (offsets relative to the end of the
header), then the raw little-endian tensor bytes."""
from __future__ import annotations

import json
import struct

import numpy as np

DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16}  # BF16 carried as raw uint16 bits


def llama_shapes(cfg: dict) -> dict:
    """name -> shape of every tensor the loader reads for `cfg` (untied lm_head)."""
    d, f, hd = cfg["dim"], cfg["ffn"], cfg["head_dim"]
    qd, kvd = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    out = {"model.embed_tokens.weight": (cfg["vocab"], d), "model.norm.weight": (d,), "lm_head.weight": (cfg["vocab"], d)}
    for l in range(cfg["n_layers"]):
        p = f"model.layers.{l}."
        out.update({p + "self_attn.q_proj.weight": (qd, d), p + "self_attn.k_proj.weight": (kvd, d),
                    p + "self_attn.v_proj.weight": (kvd, d), p + "self_attn.o_proj.weight": (d, qd),
                    p + "mlp.gate_proj.weight": (f, d), p + "mlp.up_proj.weight": (f, d),
                    p + "mlp.down_proj.weight": (d, f), p + "input_layernorm.weight": (d,),
                    p + "post_attention_layernorm.weight": (d,)})
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """tensors: name -> (dtype tag "F32" | "F16" | "BF16", array).  BF16 arrays are
    uint16 bit patterns (see f32_to_bf16_bits)."""
    header, blobs, off = {}, [], 0
    for name, (tag, arr) in tensors.items():
        a = np.ascontiguousarray(arr, DTYPES[tag])
        b = a.tobytes()
        header[name] = {"dtype": tag, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)))
        fh.write(h)
        for b in blobs:
            fh.write(b)
