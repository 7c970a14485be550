"""The allocation-free attention entry point (llama_attn_decode_bf16_noalloc).

It is for callers that cannot allocate device memory -- a host whose device
memory is owned by its own pool allocator, or a serving loop where cudaMalloc /
cudaFree are not allowed -- and keeps its split-KV partials in one static device
array instead of a caller workspace.  Its output must equal the regular entry
point's (which uses a caller workspace) within the attention tolerance, on two
calls in a row (the second reuses the static array left dirty by the first), and
a shape whose partials do not fit must be rejected before any launch.

Collected last (file name) so a stop-at-first-failure run has already run every
other test; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
import fp4x  # noqa: E402
from fp4x import ops  # noqa: E402

pytestmark = pytest.mark.gpu


def _bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.bfloat16).cuda()


def _noalloc(q, kc, vc, seq):
    B, H, hd = q.shape
    max_seq, n_kv = kc.shape[1], kc.shape[2]
    out = torch.empty_like(q)
    st = fp4x.lib().llama_attn_decode_bf16_noalloc(torch.cuda.current_stream().cuda_stream, B, H, n_kv, hd, seq,
                                                   max_seq, q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                                   out.data_ptr())
    return st, out


def _case(seed, B, H, NKV, HD, seq):
    max_seq = seq + 3
    q = oracle.normal_bf16(seed, B * H * HD).reshape(B, H, HD)
    kc = oracle.normal_bf16(seed + 1, B * max_seq * NKV * HD).reshape(B, max_seq, NKV, HD)
    vc = oracle.normal_bf16(seed + 2, B * max_seq * NKV * HD).reshape(B, max_seq, NKV, HD)
    return _bf16(q), _bf16(kc), _bf16(vc)


def _close(got, want):
    g = got.float().cpu().numpy().astype(np.float64)
    w = want.float().cpu().numpy().astype(np.float64)
    # same tolerance as the other attention tests: 1e-3 relative (rms floor) + one bf16 ulp
    ulp = np.ldexp(1.0, np.floor(np.log2(np.maximum(np.abs(w), 1e-30))).astype(int) - 7)
    bound = 1e-3 * np.maximum(np.abs(w), np.sqrt(np.mean(w ** 2))) + ulp
    assert np.all(np.abs(g - w) <= bound), (np.abs(g - w) / bound).max()


def test_noalloc_matches_workspace_entry_point_twice():
    # different shapes back to back, all on the split-KV scratch: the grouped MMA
    # kernel (4 and 8 q heads per KV head) and the one-head-per-KV-head kernel
    for seed, shape in [(10, (1, 32, 8, 128, 4096)), (20, (4, 32, 4, 64, 2000)), (30, (2, 8, 8, 64, 3000))]:
        B, H, NKV, HD, seq = shape
        assert fp4x.lib().llama_attn_workspace_size(B, H, NKV, HD, seq) > 0  # the scratch path is exercised
        q, kc, vc = _case(seed, *shape)
        want = ops.attn_decode_bf16(q, kc, vc, seq, split=True)
        st, got = _noalloc(q, kc, vc, seq)
        assert st == 0, fp4x.last_error()
        torch.cuda.synchronize()
        _close(got, want)


def test_noalloc_rejects_oversized_request():
    cap = fp4x.lib().llama_attn_noalloc_max_bytes()
    assert cap == 4 << 20
    H, NKV, HD, seq = 32, 4, 128, 4096
    # the smallest batch whose split-KV partials no longer fit the static array
    B = next(b for b in range(1, 4096) if fp4x.lib().llama_attn_workspace_size(b, H, NKV, HD, seq) > cap)
    q = torch.zeros((B, H, HD), dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros((1, 1, 1, HD), dtype=torch.bfloat16, device="cuda")  # never touched: rejected first
    st = fp4x.lib().llama_attn_decode_bf16_noalloc(torch.cuda.current_stream().cuda_stream, B, H, NKV, HD, seq,
                                                   seq, q.data_ptr(), kc.data_ptr(), kc.data_ptr(), q.data_ptr())
    assert st == 1 and b"static maximum" in fp4x.lib().fp4x_last_error()
    b = ctypes.c_uint32(0)
    assert fp4x.lib().fp4x_device_error(torch.cuda.current_stream().cuda_stream, ctypes.byref(b)) == 0
