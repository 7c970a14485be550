"""NVFP4 (kind::mxf4nvf4, UE4M3 scales per 16 values) on B200: the device quantiser
equals the oracle's bit for bit, the all-ones known answer, and the GEMM against
the oracle's NVFP4 product (fp32 exact on exact inputs, 1e-5 of the rms otherwise;
bf16 output within one bf16 rounding)."""
import numpy as np
import pytest

import oracle
from conftest import rel_rms

torch = pytest.importorskip("torch")
from fp4x import ops  # noqa: E402

pytestmark = pytest.mark.gpu


def dev(a, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.view(dt) if dt is not None else t


@pytest.mark.parametrize("g", [1.0, 1.0 / 448.0, 3.0])
def test_quantiser_bit_exact(g):
    w = oracle.normal(17, 96 * 512, 1.0).reshape(96, 512)
    w[0, :16] = 0.0
    w[1, :16] *= 1e4  # saturating scales
    w[2, :16] *= 1e-6  # subnormal scales
    gp, gs = ops.quantize_nvfp4(dev(w), g)
    rp, rs = oracle.quant_nvfp4(w, g)
    np.testing.assert_array_equal(gs.cpu().numpy(), rs)
    np.testing.assert_array_equal(gp.cpu().numpy(), rp)


def test_allones_known_answer():
    m, n, k = 16, 128, 64
    a = torch.full((m, k // 2), 0x22, dtype=torch.uint8, device="cuda")
    w = torch.full((n, k // 2), 0x22, dtype=torch.uint8, device="cuda")
    sa = torch.full((m, k // 16), 0x38, dtype=torch.uint8, device="cuda")  # UE4M3 1.0
    sw = torch.full((n, k // 16), 0x38, dtype=torch.uint8, device="cuda")
    d = ops.mma_nvf4(a, sa, w, sw, 1.0, torch.float32)
    assert bool((d == 64.0).all()), d
    d = ops.mma_nvf4(a, sa, w, sw, 0.25, torch.float32)
    assert bool((d == 16.0).all())


def test_exact_inputs_bit_exact():
    """Random codes with power-of-two and non-power-of-two UE4M3 scales whose
    products and partial sums are exact in fp32: any summation order gives the
    oracle's bits (pins the nibble, scale and 16-block layouts)."""
    rng = np.random.default_rng(3)
    m, n, k = 24, 256, 512
    a = rng.integers(0, 256, (m, k // 2), dtype=np.uint8)
    w = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    sa = rng.choice(np.array([0x30, 0x38, 0x3C, 0x40, 0x44], np.uint8), (m, k // 16))
    sw = rng.choice(np.array([0x34, 0x38, 0x3A, 0x40], np.uint8), (n, k // 16))
    got = ops.mma_nvf4(dev(a), dev(sa), dev(w), dev(sw), 1.0, torch.float32).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.mma_nvf4(a, sa, w, sw, 1.0))


@pytest.mark.parametrize("m,n,k", [(16, 2560, 2048), (64, 2048, 5632), (256, 1024, 2048), (512, 384, 1024)])
def test_gemm_vs_oracle(m, n, k):
    ga, gw = 1.0 / 64.0, 1.0 / 4096.0
    a, sa = oracle.quant_nvfp4(oracle.normal(m + 1, m * k, 1.0).reshape(m, k), ga)
    w, sw = oracle.quant_nvfp4(oracle.normal(n + 2, n * k, 0.02).reshape(n, k), gw)
    ref = oracle.mma_nvf4(a, sa, w, sw, ga * gw)
    got = ops.mma_nvf4(dev(a), dev(sa), dev(w), dev(sw), ga * gw, torch.float32).cpu().numpy()
    assert rel_rms(got, ref).max() <= 1e-5
    gb = ops.mma_nvf4(dev(a), dev(sa), dev(w), dev(sw), ga * gw).float().cpu().numpy()
    assert np.max(np.abs(gb - ref) / np.maximum(np.abs(ref), 1e-30)) <= 2.0 ** -8 + 1e-6 or rel_rms(gb, ref).max() <= 4e-3
