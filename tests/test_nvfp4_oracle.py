"""NVFP4 restatement in the oracle (CPU): the UE4M3 code table, round-to-nearest
even with saturation, the quantiser's bound on the reconstruction error, and the
NVFP4 product on exact inputs."""
import numpy as np
import pytest

import oracle


def test_ue4m3_table_round_trips():
    for b in range(0x7F):  # 0x7F is NaN
        v = oracle.ue4m3_to_f32(b)
        assert oracle.f32_to_ue4m3(v) == b, (b, v)
    assert oracle.ue4m3_to_f32(0x38) == 1.0 and oracle.ue4m3_to_f32(0x7E) == 448.0
    assert oracle.ue4m3_to_f32(0x01) == 2.0 ** -9 and oracle.ue4m3_to_f32(0x08) == 2.0 ** -6


@pytest.mark.parametrize("s,code", [(1.0625, 0x38), (1.1875, 0x3A), (1000.0, 0x7E), (0.0, 0), (-3.0, 0),
                                    (2.0 ** -10, 0), (3 * 2.0 ** -10, 0x02), (464.0, 0x7E)])
def test_ue4m3_rounding_ties_to_even_and_saturates(s, code):
    assert oracle.f32_to_ue4m3(s) == code


@pytest.mark.parametrize("g", [1.0, 1.0 / 448.0, 3.0])
def test_quantiser_error_bound(g):
    w = oracle.normal(5, 64 * 256, 1.0).reshape(64, 256) * 0.5
    w[3, :16] = 0.0  # an all-zero block
    p, s = oracle.quant_nvfp4(w, g)
    assert p.shape == (64, 128) and s.shape == (64, 16)
    assert np.all(s[3, 0] == 0) and np.all(p[3, :8] == 0)
    # dequantise: e2m1 * UE4M3 * g; error per value <= half an E2M1 step of the block scale
    lut = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0.0, -.5, -1, -1.5, -2, -3, -4, -6], np.float32)
    codes = np.stack([p & 0xF, p >> 4], axis=-1).reshape(64, 256)
    sc = np.vectorize(oracle.ue4m3_to_f32)(s).astype(np.float32).repeat(16, axis=1) * np.float32(g)
    deq = lut[codes] * sc
    blk_max = np.abs(w).reshape(64, 16, 16).max(axis=2).repeat(16, axis=1)
    # E2M1 rounding: at most half a step (1.0 in [4, 6]) of a scale that rounds up by <= 1/16
    assert np.all(np.abs(deq - w) <= 0.18 * blk_max + 1e-30), np.max(np.abs(deq - w) / blk_max)


def test_mma_nvf4_exact_inputs():
    rng = np.random.default_rng(1)
    m, n, k = 5, 7, 128
    a = rng.integers(0, 256, (m, k // 2), dtype=np.uint8)
    w = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    sa = np.full((m, k // 16), 0x38, np.uint8)  # 1.0
    sw = np.full((n, k // 16), 0x40, np.uint8)  # 2.0
    d = oracle.mma_nvf4(a, sa, w, sw, 0.5)
    lut = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0.0, -.5, -1, -1.5, -2, -3, -4, -6], np.float64)
    av = lut[np.stack([a & 0xF, a >> 4], -1).reshape(m, k)]
    wv = lut[np.stack([w & 0xF, w >> 4], -1).reshape(n, k)]
    np.testing.assert_array_equal(d, (av @ wv.T * 2.0 * 0.5).astype(np.float32))
