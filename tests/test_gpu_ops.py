"""Parity of each CUDA operator with the CPU oracle on identical seeded inputs.

Every call goes through the C ABI (libfp4x.so via ctypes).  Bars:
  * integer / byte work (quantise, dequantise, E2M1 decode, initialiser): bit-exact;
  * GEMV and attention (fp32 accumulation, different order than the oracle):
    |gpu - ref| <= 1e-3 * max(|ref|, rms(ref)) per element (rel_rms), and the
    reference's own gates (rel_floor <= 1e-2 GEMV, 1e-4 RMSNorm/RoPE/attention);
  * RMSNorm / RoPE / SwiGLU / residual: the reference's 1e-4 floor-form gate.
"""
from pathlib import Path

import numpy as np
import pytest

import oracle
from conftest import rel_floor, rel_rms

torch = pytest.importorskip("torch")
import fp4x  # noqa: E402
from fp4x import ops  # noqa: E402

pytestmark = pytest.mark.gpu
G = np.load(Path(__file__).resolve().parent / "golden" / "reference_kats.npz")
GEMV_TOL = 1e-3


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def assert_no_device_error():
    import ctypes
    b = ctypes.c_uint32(0)
    st = fp4x.lib().fp4x_device_error(torch.cuda.current_stream().cuda_stream, ctypes.byref(b))
    assert st == 0 and b.value == 0, fp4x.last_error()


# ---------------------------------------------------------------- formats

def test_dequant_all_bytes_bit_exact():
    # every byte value (both nibble orders) x a spread of E8M0 scales
    packed = np.tile(np.arange(256, dtype=np.uint8), 16).reshape(-1, 16)  # 256 rows x 32 codes
    scales = (np.arange(256) % 254 + 1).astype(np.uint8).reshape(-1, 1)
    got = host(ops.dequantize_mxfp4(dev(packed), dev(scales)))
    want = oracle.dequant_mxfp4(packed, scales)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("shape", [(64, 64), (5632, 2048), (3, 4096)])
def test_quantize_mxfp4_bit_exact(shape):
    n, k = shape
    w = oracle.normal(11, n * k, 0.02).reshape(n, k)
    w[0, :32] = 0.0                    # all-zero block
    w[0, 32:64] = -1e-30               # tiny negatives -> -0 codes
    if k >= 128:
        w[0, 64:96] = np.float32(7.5) * np.linspace(-1, 1, 32, dtype=np.float32)
    p, s = ops.quantize_mxfp4(dev(w))
    wp, ws = oracle.quant_mxfp4(w)
    np.testing.assert_array_equal(host(s), ws)
    np.testing.assert_array_equal(host(p), wp)


def test_quantize_ref_bit_exact():
    blocks = G["quant_in"]
    p, s = ops.quantize_ref(dev(blocks))
    np.testing.assert_array_equal(host(s).ravel(), G["quant_scales"])
    words = host(p).view(np.uint32).ravel()
    codes = np.array([(words[i // 8] >> (4 * (i % 8))) & 0xF for i in range(96)], np.uint8)
    np.testing.assert_array_equal(codes.reshape(3, 32), G["quant_codes"])
    w = oracle.normal(3, 256 * 512, 0.5).reshape(256, 512)
    p, s = ops.quantize_ref(dev(w))
    rp, rs = oracle.quant_ref(w)
    np.testing.assert_array_equal(host(p).view(np.uint32), rp)
    np.testing.assert_array_equal(host(s), rs)


def test_generators_bit_exact():
    np.testing.assert_array_equal(host(ops.fill_normal(100_003, seed=77, sigma=0.02)),
                                  oracle.normal(77, 100_003, 0.02))
    got = host(ops.fill_normal(4097, seed=5, sigma=1.0, dtype=torch.bfloat16).view(torch.int16))
    np.testing.assert_array_equal(got.view(np.uint16), oracle.normal_bf16(5, 4097, 1.0))
    p, s = ops.init_mxfp4(256, 2048, seed=99, sigma=0.02)
    wp, ws = oracle.quant_mxfp4(oracle.normal(99, 256 * 2048, 0.02).reshape(256, 2048))
    np.testing.assert_array_equal(host(p), wp)
    np.testing.assert_array_equal(host(s), ws)


# ---------------------------------------------------------------- GEMV

def test_gemv_config0():
    """W 5632x2048 N(0,0.02) -> MXFP4 (E8M0 rule), x bf16 N(0,1), y f32."""
    n, k = 5632, 2048
    wp, ws = oracle.quant_mxfp4(oracle.normal(1, n * k, 0.02).reshape(n, k))
    xb = oracle.normal_bf16(2, k, 1.0)
    y = host(ops.gemv(dev(wp), dev(ws), dev(xb, torch.bfloat16)))
    ref = oracle.gemv_mxfp4(wp, ws, xb)
    assert rel_rms(y, ref).max() <= GEMV_TOL, rel_rms(y, ref).max()
    assert_no_device_error()


def test_gemv_reference_kat_4096():
    """examples/fp4_gemv/src/main.rs:95-173 exactly: reference storage (u32 words,
    f32 scales, f32 x), xorshift32 seed 0x12345678, gate rel_floor <= 1e-2."""
    N = K = 4096
    r = oracle.xorshift32(0x12345678, N * K + N * K // 32 + K)
    codes = (r[: N * K] & 0xF).astype(np.uint32)
    words = np.zeros(N * K // 8, np.uint32)
    for p in range(8):
        words |= codes[p::8] << (4 * p)
    scales = (np.float32(0.5) + (r[N * K: N * K + N * K // 32] % 8).astype(np.float32) * np.float32(0.25))
    x = ((r[N * K + N * K // 32:] % 17).astype(np.float32) - np.float32(8.0)) * np.float32(0.1)
    words = words.reshape(N, K // 8)
    scales = scales.reshape(N, K // 32).astype(np.float32)
    y = host(ops.gemv_ref(dev(words.view(np.int32)), dev(scales), dev(x)))
    ref = oracle.gemv_ref(words, scales, x)
    assert (rel_floor(y, ref) > 1e-2).sum() == 0
    assert rel_rms(y, ref).max() <= GEMV_TOL


def test_gemv_golden_fixture():
    y = host(ops.gemv_ref(dev(G["gemv_words"].view(np.int32)), dev(G["gemv_scales"]), dev(G["gemv_x"])))
    assert rel_rms(y, G["gemv_y"]).max() <= GEMV_TOL


def test_gemv_exact_inputs_bit_exact():
    """Inputs whose every partial sum is exact in fp32 (small-integer x, scales
    2^0) must give the oracle's result bit for bit, whatever the summation order:
    this pins the nibble/row/column layout with zero tolerance."""
    n, k = 48, 1024
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 16, size=(n, k), dtype=np.uint8)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    scales = rng.integers(124, 130, size=(n, k // 32), dtype=np.uint8)
    x = rng.integers(-8, 9, size=k).astype(np.float32)
    xb = oracle.f32_to_bf16(x)
    y = host(ops.gemv(dev(packed), dev(scales), dev(xb, torch.bfloat16)))
    ref = oracle.gemv_mxfp4(packed, scales, xb)
    np.testing.assert_array_equal(y, ref)
    y32 = host(ops.gemv(dev(packed), dev(scales), dev(x)))
    np.testing.assert_array_equal(y32, ref)


@pytest.mark.parametrize("n,k", [(1, 32), (17, 96), (2560, 2048), (2048, 5632), (32000, 2048), (100, 16384)])
def test_gemv_shapes_f32x(n, k):
    wp, ws = oracle.quant_mxfp4(oracle.normal(n + k, n * k, 0.02).reshape(n, k))
    x = oracle.normal(7, k, 1.0)
    y = host(ops.gemv(dev(wp), dev(ws), dev(x)))
    ref = oracle.gemv_mxfp4(wp, ws, x)
    assert rel_rms(y, ref).max() <= GEMV_TOL, rel_rms(y, ref).max()


def test_gemv_rejects_bad_shapes():
    w = torch.zeros((16, 24), dtype=torch.uint8, device="cuda")
    s = torch.zeros((16, 1), dtype=torch.uint8, device="cuda")
    with pytest.raises(fp4x.Fp4xError):
        ops.gemv(w, s, torch.zeros(48, dtype=torch.float32, device="cuda"))


# ---------------------------------------------------------------- small operators

def test_rmsnorm_reference_kat():
    y = host(ops.rmsnorm(dev(G["rms_x"]), dev(G["rms_w"]), 1e-5))
    assert rel_floor(y, G["rms_y"]).max() <= 1e-4


def test_rope_reference_kat():
    c, s = ops.rope_tables(38, 64, 500000.0)
    oc, os_ = oracle.rope_tables(38, 64, 500000.0)
    np.testing.assert_array_equal(host(c), oc)
    np.testing.assert_array_equal(host(s), os_)
    q = dev(G["rope_q"].copy())
    ops.rope_(q, 32, 64, 37 * 32, c, s)
    # same operations in the same order, no contraction: bit-exact
    np.testing.assert_array_equal(host(q), G["rope_out"])


def test_swiglu_residual_copy():
    g = oracle.normal(1, 5632, 2.0)
    u = oracle.normal(2, 5632, 1.0)
    got = host(ops.swiglu(dev(g), dev(u)))
    assert rel_floor(got, oracle.swiglu(g, u)).max() <= 1e-4
    x = oracle.normal(3, 2048)
    y = oracle.normal(4, 2048)
    xd = dev(x.copy())
    ops.residual_(xd, dev(y))
    np.testing.assert_array_equal(host(xd), oracle.residual(y, x))
    dst = torch.zeros(4096, device="cuda")
    ops.copy_into_(dst, dev(y[:256]), 512)
    np.testing.assert_array_equal(host(dst)[512:768], y[:256])
    kv = torch.zeros(4096, dtype=torch.bfloat16, device="cuda")
    ops.kv_append_bf16_(kv, dev(y[:256]), 256)
    np.testing.assert_array_equal(host(kv.view(torch.int16)).view(np.uint16)[256:512], oracle.f32_to_bf16(y[:256]))


def test_argmax_ties_lowest_index():
    v = oracle.normal(5, 32000)
    v[100] = 50.0
    v[31000] = 50.0
    v[20000] = 50.0
    assert int(host(ops.argmax(dev(v)))[0]) == 100 == oracle.argmax(v)
    w = np.full(128256, -3.0, np.float32)
    assert int(host(ops.argmax(dev(w)))[0]) == 0 == oracle.argmax(w)


# ---------------------------------------------------------------- attention

def test_attention_reference_kat():
    """llama_attn_decode/src/main.rs:132-210: 32q/8kv, hd 64, seq 512, seed 0xabcd1234, gate 1e-4."""
    NH, NKV, HD, SEQ = 32, 8, 64, 512
    r = oracle.xorshift32(0xABCD1234, NH * HD + 2 * SEQ * NKV * HD)
    vals = ((r % 2001).astype(np.float32) - np.float32(1000.0)) / np.float32(700.0)
    q, kc, vc = vals[: NH * HD], vals[NH * HD: NH * HD + SEQ * NKV * HD], vals[NH * HD + SEQ * NKV * HD:]
    ref = oracle.attn_decode(q, kc, vc, NH, NKV, HD, SEQ)
    got = host(ops.attn_decode(dev(q), dev(kc), dev(vc), NH, NKV, SEQ))
    assert rel_floor(got, ref).max() <= 1e-4, rel_floor(got, ref).max()
    got2 = host(ops.attn_decode_hd(dev(q), dev(kc), dev(vc), NH, NKV, HD, SEQ, split=True))
    assert rel_floor(got2, ref).max() <= 1e-4


def test_attention_golden_fixture():
    got = host(ops.attn_decode(dev(G["attn_q"]), dev(G["attn_k"]), dev(G["attn_v"]), 32, 8, 64))
    assert rel_floor(got, G["attn_out"]).max() <= 1e-4


@pytest.mark.parametrize("B,NH,NKV,HD,ctx", [(1, 32, 4, 64, 512), (8, 32, 4, 64, 2048), (2, 32, 8, 128, 1000),
                                              (1, 32, 8, 128, 8192), (3, 32, 4, 64, 1), (1, 8, 8, 128, 77)])
def test_attention_bf16_config2(B, NH, NKV, HD, ctx):
    max_seq = ctx + 5
    q = oracle.normal_bf16(1, B * NH * HD).reshape(B, NH, HD)
    kc = oracle.normal_bf16(2, B * max_seq * NKV * HD).reshape(B, max_seq, NKV, HD)
    vc = oracle.normal_bf16(3, B * max_seq * NKV * HD).reshape(B, max_seq, NKV, HD)
    ref = oracle.attn_decode_bf16(q, kc, vc, B, NH, NKV, HD, ctx, max_seq)
    got = host(ops.attn_decode_bf16(dev(q, torch.bfloat16), dev(kc, torch.bfloat16), dev(vc, torch.bfloat16),
                                    ctx).view(torch.int16)).view(np.uint16)
    g32, r32 = oracle.bf16_to_f32(got).astype(np.float64), oracle.bf16_to_f32(ref).astype(np.float64)
    # bf16 output: both sides round an fp32 result, so one bf16 ulp of the
    # reference value is allowed on top of the 1e-3 relative bar
    ulp = np.ldexp(1.0, np.floor(np.log2(np.maximum(np.abs(r32), 1e-30))).astype(int) - 7)
    bound = 1e-3 * np.maximum(np.abs(r32), np.sqrt(np.mean(r32 ** 2))) + ulp
    assert np.all(np.abs(g32 - r32) <= bound), (np.abs(g32 - r32) / bound).max()
    assert_no_device_error()
