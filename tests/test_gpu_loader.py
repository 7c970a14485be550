"""Real-weight checkpoints: a safetensors file with Hugging Face Llama names
(BF16 projections, F16 embeddings, F32 norm weights) loaded by
llama_model_create_from_safetensors.  Every linear must equal the oracle's
quantisation of the same values bit for bit (shards included), and the model's
logits must match the oracle carrying the same weights within 1e-2 with the same
greedy tokens, on every decode path and in the batched engine."""
import numpy as np
import pytest

import oracle
from test_gpu_engine import TINY, compare_logits, shape_of, tensor_ids

torch = pytest.importorskip("torch")
from fp4x import checkpoint, engine  # noqa: E402

pytestmark = pytest.mark.gpu


def _name_of(cfg, tid):
    if tid == 1:
        return "lm_head.weight"
    l, w = (tid - 16) // 8, (tid - 16) % 8
    return f"model.layers.{l}." + ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                                    "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"][w] + ".weight"


def _checkpoint(cfg, path, tied=False, seed=7):
    """Random weights (not the seeded initialiser's), written to `path`; returns the
    f32 values the loader will see per tensor name."""
    rng = np.random.default_rng(seed)
    vals, out = {}, {}
    for name, shape in checkpoint.llama_shapes(cfg).items():
        if tied and name == "lm_head.weight":
            continue
        if name.endswith("norm.weight"):
            v = (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
            out[name] = ("F32", v)
        elif name == "model.embed_tokens.weight":
            v = (0.02 * rng.standard_normal(shape)).astype(np.float16)
            out[name] = ("F16", v)
            v = v.astype(np.float32)
        else:
            bits = checkpoint.f32_to_bf16_bits((0.02 * rng.standard_normal(shape)).astype(np.float32))
            out[name] = ("BF16", bits)
            v = (bits.astype(np.uint32) << 16).view(np.float32)
        vals[name] = v
    checkpoint.write_safetensors(str(path), out)
    if tied:
        vals["lm_head.weight"] = vals["model.embed_tokens.weight"]
    return vals


def _oracle_with(cfg, vals):
    ref = oracle.Model(cfg)
    for tid in tensor_ids(cfg):
        ref.set_tensor(tid, *oracle.quant_mxfp4(vals[_name_of(cfg, tid)]))
    ref.set_embed(oracle.f32_to_bf16(vals["model.embed_tokens.weight"]))
    L = cfg["n_layers"]
    for l in range(L):
        ref.set_norm(l, vals[f"model.layers.{l}.input_layernorm.weight"])
        ref.set_norm(L + l, vals[f"model.layers.{l}.post_attention_layernorm.weight"])
    ref.set_norm(2 * L, vals["model.norm.weight"])
    return ref


@pytest.mark.parametrize("tied", [False, True], ids=["untied", "tied"])
def test_loaded_weights_bit_exact(tmp_path, tied):
    cfg = TINY
    vals = _checkpoint(cfg, tmp_path / "m.safetensors", tied=tied)
    with engine.Model(cfg, safetensors=tmp_path / "m.safetensors") as m:
        for tid in tensor_ids(cfg):
            rp, rs = oracle.quant_mxfp4(vals[_name_of(cfg, tid)])
            gp, gs = m.export_tensor(tid)
            assert gp.shape == rp.shape == (shape_of(cfg, tid)[0], shape_of(cfg, tid)[1] // 2)
            np.testing.assert_array_equal(gs, rs, err_msg=f"scales of {_name_of(cfg, tid)}")
            np.testing.assert_array_equal(gp, rp, err_msg=f"nibbles of {_name_of(cfg, tid)}")
        np.testing.assert_array_equal(m.embedding(), oracle.f32_to_bf16(vals["model.embed_tokens.weight"]))


@pytest.mark.parametrize("path", ["graph", "persistent", "tensor"])
def test_loaded_model_matches_oracle(tmp_path, path):
    cfg = TINY
    vals = _checkpoint(cfg, tmp_path / "m.safetensors")
    ref = _oracle_with(cfg, vals)
    toks = oracle.uniform_ids(9, cfg["vocab"], 12)
    with engine.Model(cfg, safetensors=tmp_path / "m.safetensors") as m:
        m.set_path(path)
        for pos, t in enumerate(toks):
            gn, gl = m.forward(int(t), pos)
            rn, rl = ref.forward(int(t), pos)
            compare_logits(gl, rl)
        m.reset()
        prompt = oracle.uniform_ids(20, cfg["vocab"], 5)
        ref2 = _oracle_with(cfg, vals)
        want = ref2.generate(prompt, 12)
        got, _, _ = m.generate(prompt, 12)
        ref2.close()
    ref.close()
    np.testing.assert_array_equal(got, want)


def test_loaded_model_batched_engine(tmp_path):
    cfg = TINY
    vals = _checkpoint(cfg, tmp_path / "m.safetensors", seed=11)
    ref = _oracle_with(cfg, vals)
    prompt = oracle.uniform_ids(21, cfg["vocab"], 7)
    with engine.Model(cfg, safetensors=tmp_path / "m.safetensors") as m, engine.Batch(m, 4) as b:
        b.prefill(0, prompt)
        got = b.logits()[0]
    for pos, t in enumerate(prompt):
        _, rl = ref.forward(int(t), pos)
    ref.close()
    compare_logits(got, rl)


def test_loader_rejects_wrong_shapes(tmp_path):
    cfg = TINY
    _checkpoint(cfg, tmp_path / "m.safetensors")
    from fp4x import Fp4xError
    with pytest.raises(Fp4xError):
        engine.Model(dict(cfg, ffn=1024), safetensors=tmp_path / "m.safetensors")
    with pytest.raises(Fp4xError):
        engine.Model(cfg, safetensors=tmp_path / "missing.safetensors")
