"""Checkpoint (safetensors) host logic: the header reader of the C ABI
(fp4x_safetensors_info) on files written by fp4x.checkpoint, its rejection of
malformed files, and the bf16 rounding helper.  No GPU needed."""
import json
import struct

import numpy as np
import pytest

import oracle
from fp4x import Fp4xError, checkpoint, engine


def _write(tmp_path, tensors, name="m.safetensors"):
    p = tmp_path / name
    checkpoint.write_safetensors(str(p), tensors, metadata={"format": "pt"})
    return p


def test_info_reads_dtypes_and_shapes(tmp_path):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((3, 64)).astype(np.float32)
    p = _write(tmp_path, {"a": ("F32", a), "b": ("BF16", checkpoint.f32_to_bf16_bits(a)),
                          "c": ("F16", a.astype(np.float16)), "model.norm.weight": ("F32", a[0])})
    assert engine.safetensors_info(p, "a") == ("F32", (3, 64))
    assert engine.safetensors_info(p, "b") == ("BF16", (3, 64))
    assert engine.safetensors_info(p, "c") == ("F16", (3, 64))
    assert engine.safetensors_info(p, "model.norm.weight") == ("F32", (64,))
    with pytest.raises(Fp4xError):
        engine.safetensors_info(p, "missing")


def test_bf16_rounding_matches_oracle():
    x = oracle.normal(3, 4096, 1.0)
    np.testing.assert_array_equal(checkpoint.f32_to_bf16_bits(x), oracle.f32_to_bf16(x))


def test_llama_shapes_cover_the_config():
    cfg = dict(n_layers=2, dim=256, ffn=512, n_heads=8, n_kv_heads=2, head_dim=64, vocab=1000)
    s = checkpoint.llama_shapes(cfg)
    assert len(s) == 3 + 9 * 2
    assert s["model.layers.1.self_attn.k_proj.weight"] == (128, 256)
    assert s["model.layers.0.mlp.down_proj.weight"] == (256, 512)


@pytest.mark.parametrize("mutate", ["truncated", "huge_header", "not_json", "past_end", "bad_shape", "no_offsets"])
def test_malformed_files_are_rejected(tmp_path, mutate):
    a = np.zeros((4, 32), np.float32)
    p = _write(tmp_path, {"a": ("F32", a)})
    raw = p.read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + n])
    body = raw[8 + n:]
    if mutate == "truncated":
        out = raw[:6]
    elif mutate == "huge_header":
        out = struct.pack("<Q", 1 << 40) + raw[8:]
    elif mutate == "not_json":
        h = b"[1, 2, 3]" + b" " * (n - 9)
        out = raw[:8] + h + body
    else:
        if mutate == "past_end":
            hdr["a"]["data_offsets"] = [0, len(body) + 64]
            hdr["a"]["shape"] = [4, 36]
        elif mutate == "bad_shape":
            hdr["a"]["shape"] = [4, 33]
        else:
            del hdr["a"]["data_offsets"]
        h = json.dumps(hdr).encode()
        h += b" " * (-len(h) % 8)
        out = struct.pack("<Q", len(h)) + h + body
    q = tmp_path / "bad.safetensors"
    q.write_bytes(out)
    with pytest.raises(Fp4xError):
        engine.safetensors_info(q, "a")
