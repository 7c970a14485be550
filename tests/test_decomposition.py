"""The 8-term MXFP4 activation decomposition used by the tensor-core decode path
(rust-fp4-blackwell_b200/csrc/persist_tc.cu, decompose_word8), restated in numpy:
per 32-block, first scale 2^e1 with e1 the smallest exponent such that the block
maximum <= 6 * 2^e1, then e1 - 2, then 3 less per term; each term rounds the
residual to the nearest E2M1 value (ties to even, saturating at 6).  Checks the
stated bound |x - sum of terms| <= 2^(e1 - 21) and that no term saturates, on
normal, uniform, heavy-tailed and wide-dynamic-range blocks."""
import numpy as np

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def rne_e2m1(y):
    a = np.minimum(np.abs(y), 6.0)
    d = np.abs(a[..., None] - E2M1)
    best = d == d.min(-1, keepdims=True)
    codes = np.arange(8)
    even = np.where(best & (codes % 2 == 0), codes, 99).min(-1)
    pick = np.where(even == 99, np.where(best, codes, 99).min(-1), even)
    return np.sign(y) * E2M1[pick], np.abs(y) > 6.0


def decompose(x):
    amax = np.abs(x).max(-1, keepdims=True).astype(np.float32)
    bits = amax.view(np.uint32)
    e = ((bits >> 23) & 0xFF).astype(np.int64) - 127
    e1 = np.where((bits & 0x7FFFFF) <= 0x400000, e - 2, e - 1)
    r = x.astype(np.float64)
    total = np.zeros_like(r)
    saturated = False
    for t in range(8):
        et = np.clip(e1 if t == 0 else e1 + 1 - 3 * t, -126, 125)
        s = np.exp2(et.astype(np.float64))
        q, sat = rne_e2m1(r / s)
        saturated |= bool(sat.any())
        total += q * s
        r -= q * s
    return total, e1, saturated


def test_decomposition_bound():
    rng = np.random.default_rng(7)
    cases = [rng.standard_normal((4000, 32)), rng.uniform(-1, 1, (4000, 32)), rng.standard_cauchy((4000, 32)),
             rng.standard_normal((4000, 32)) * np.exp(rng.uniform(-20, 20, (4000, 1)))]
    for x in cases:
        x = x.astype(np.float32)
        y, e1, saturated = decompose(x)
        assert not saturated
        err = np.abs(y - x.astype(np.float64)).max(-1)
        assert np.all(err <= np.exp2(e1[:, 0] - 21.0))
        assert np.max(err / np.abs(x).max(-1)) < 2e-7


def test_decomposition_zero_block():
    y, _, saturated = decompose(np.zeros((1, 32), np.float32))
    assert not saturated and np.all(y == 0)
