"""Pin the C oracle (oracle/oracle.c) against the reference's known answers.

tests/golden/reference_kats.npz is produced by tests/golden/make_golden.py, an
independent float32 restatement of the reference's CPU loops; the oracle must
match it bit for bit (the published max errors in the reference are for GPU vs
CPU, not CPU vs CPU).  CPU only."""
from pathlib import Path

import numpy as np
import pytest

import oracle

G = np.load(Path(__file__).resolve().parent / "golden" / "reference_kats.npz")


def test_xorshift32_streams():
    # Marsaglia (2003), "Xorshift RNGs": state 2463534242 -> first output 723471715.
    assert int(oracle.xorshift32(2463534242, 1)[0]) == 723471715
    for name, seed in [("gemv", 0x12345678), ("rmsnorm", 0x9E3779B9), ("rope", 0x13579BDF),
                       ("attn", 0xABCD1234), ("decode", 0xDEADBEEF), ("marsaglia", 2463534242)]:
        np.testing.assert_array_equal(oracle.xorshift32(seed, 8), G[f"xs_{name}"])


def test_e2m1_table_bit_exact():
    # trackb/FP4_M16N8K64_LAYOUT.md:25-26: magnitudes {0,.5,1,1.5,2,3,4,6}, bit3 = sign (0x8 = -0.0)
    L = oracle.lib()
    got = np.array([L.orc_e2m1_decode(c) for c in range(16)], np.float32)
    np.testing.assert_array_equal(got.view(np.uint32), G["e2m1_table"].view(np.uint32))
    assert np.signbit(got[8]) and got[8] == 0.0


def test_quant_ref_ties_and_signs():
    packed, scales = oracle.quant_ref(G["quant_in"])
    np.testing.assert_array_equal(scales.ravel(), G["quant_scales"])
    codes = np.array([(packed.ravel()[i // 8] >> (4 * (i % 8))) & 0xF for i in range(96)], np.uint8)
    np.testing.assert_array_equal(codes.reshape(3, 32), G["quant_codes"])


def test_quant_mxfp4_e8m0_rule():
    L = oracle.lib()
    # 2^(floor(log2 amax) - 2) via exponent bits
    for amax, e in [(6.0, 127), (4.0, 127), (7.99, 127), (8.0, 128), (1.0, 125), (0.03, 119),
                    (2.0 ** -126, 0), (2.0 ** -125, 0), (2.0 ** -124, 1), (0.0, 127)]:
        assert L.orc_e8m0_from_amax(amax) == e, amax
    # subnormal amax: floor(log2) from the mantissa
    assert L.orc_e8m0_from_amax(np.float32(2.0 ** -130)) == 0
    # values in (6, 8) * scale clamp to 6; ties to the smaller level
    w = np.array([[7.5, 3.5 * 2, 1.75 * 2, 0.25 * 2, -0.75 * 2] + [0.0] * 27], np.float32)
    p, s = oracle.quant_mxfp4(w)
    assert s[0, 0] == 127  # amax 7.5: floor(log2) = 2 -> scale 2^0
    codes = [(p[0, i // 2] >> (4 * (i % 2))) & 0xF for i in range(5)]
    # 7.5, 7.0 -> 6 (clamp); 3.5 -> 3 (tie to smaller); 0.5 -> 0.5; -1.5 -> -1.5
    assert codes == [7, 7, 5, 1, 11]


def test_mma_kats():
    def pack(mat):  # rows of 64 logical values -> packed nibbles
        codes = np.zeros(mat.shape, np.uint8)
        for i in range(mat.shape[0]):
            for k in range(mat.shape[1]):
                v = mat[i, k]
                c = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0].index(abs(float(v)))
                codes[i, k] = c | (8 if v < 0 else 0)
        return (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)

    # all ones, scale 1.0 (ue8m0 0x7F): every D = 64 (examples/fp4_mma/src/main.rs:24-31,75)
    a = np.full((16, 32), 0x22, np.uint8)
    w = np.full((8, 32), 0x22, np.uint8)
    s1 = np.full((16, 2), 127, np.uint8)
    d = oracle.mma_mxf4(a, s1, w, np.full((8, 2), 127, np.uint8))
    np.testing.assert_array_equal(d, G["kat_allones_D"])
    # patterned A/B (trackb/fp4_mapping_test.cu:38-40); W = B^T
    A, B = G["kat_pattern_A"], G["kat_pattern_B"]
    d = oracle.mma_mxf4(pack(A), s1, pack(B.T.copy()), np.full((8, 2), 127, np.uint8))
    np.testing.assert_array_equal(d, G["kat_pattern_D"])
    # power-of-two scales (trackb/fp4_scale_test.cu:34-37,112), ue8m0 = 127 + log2 s
    sa = (127 + np.log2(G["kat_scale_SFA"])).astype(np.uint8)
    sb = (127 + np.log2(G["kat_scale_SFB"].T)).astype(np.uint8)
    d = oracle.mma_mxf4(pack(A), sa, pack(B.T.copy()), sb)
    np.testing.assert_array_equal(d, G["kat_scale_D"])


def test_gemv_ref_bit_exact():
    y = oracle.gemv_ref(G["gemv_words"], G["gemv_scales"], G["gemv_x"], threads=1)
    np.testing.assert_array_equal(y.view(np.uint32), G["gemv_y"].view(np.uint32))
    y4 = oracle.gemv_ref(G["gemv_words"], G["gemv_scales"], G["gemv_x"], threads=4)
    np.testing.assert_array_equal(y4, y)  # threading keeps the per-row order


def test_rmsnorm_bit_exact():
    y = oracle.rmsnorm(G["rms_x"], G["rms_w"], 1e-5)
    np.testing.assert_array_equal(y.view(np.uint32), G["rms_y"].view(np.uint32))


def test_rope_bit_exact():
    c, s = oracle.rope_tables(38, 64, 500000.0)
    np.testing.assert_array_equal(c[37], G["rope_cos"])
    np.testing.assert_array_equal(s[37], G["rope_sin"])
    out = oracle.rope(G["rope_q"], 32, 64, 37 * 32, c, s)
    np.testing.assert_array_equal(out.view(np.uint32), G["rope_out"].view(np.uint32))


def test_attention_matches_restatement():
    out = oracle.attn_decode(G["attn_q"], G["attn_k"], G["attn_v"], 32, 8, 64, 64)
    # exp() comes from libm on both sides; allow one ulp-level wobble
    np.testing.assert_allclose(out, G["attn_out"], rtol=2e-6, atol=1e-7)


def test_mxfp4_roundtrip_and_dequant():
    w = oracle.normal(5, 16 * 64, 0.02).reshape(16, 64)
    p, s = oracle.quant_mxfp4(w)
    d = oracle.dequant_mxfp4(p, s)
    scale = np.repeat(np.ldexp(1.0, s.astype(np.int32) - 127), 32, axis=1)
    codes = d / scale
    assert set(np.unique(np.abs(codes))).issubset({0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0})
    # nearest level: at most half the widest spacing (2 between 4 and 6), except the
    # clamp of [6, 8)*scale to 6*scale, which is below 2*scale
    assert np.all(np.abs(d - w) < scale * 2.0)


def test_generator_properties():
    z = oracle.normal(123, 200_000)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1.0) < 0.01
    assert np.all(np.abs(z) <= 6.0)
    # bf16 narrowing is round-to-nearest-even of the f32 draw
    zb = oracle.normal_bf16(123, 1000)
    np.testing.assert_array_equal(zb, oracle.f32_to_bf16(z[:1000]))
    ids = oracle.uniform_ids(9, 32000, 1000)
    assert ids.max() < 32000 and len(np.unique(ids)) > 900


def test_oracle_model_tiny_forward():
    cfg = dict(n_layers=2, dim=64, ffn=128, n_heads=4, n_kv_heads=2, head_dim=16, vocab=100, max_seq=16,
               rope_theta=10000.0, eps=1e-5, seed=7)
    m = oracle.Model(cfg)
    nxt, logits = m.forward(3, 0)
    assert np.all(np.isfinite(logits)) and 0 <= nxt < 100
    assert nxt == int(np.argmax(logits))
    m.close()
    m2 = oracle.Model(cfg)
    ids = m2.generate(np.array([3, 5, 7], np.uint32), 4)
    assert ids.shape == (4,) and ids.max() < 100
