"""torch-facing wrappers over the C ABI: each call hands device pointers of CUDA
tensors and the current torch stream to libfp4x.so.  Tensors must be CUDA and
contiguous; nothing here computes on the host."""
from __future__ import annotations

import torch

from . import check, lib


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor):
    if not t.is_cuda:
        raise ValueError("fp4x operators take CUDA tensors (no CPU fallback)")
    if not t.is_contiguous():
        raise ValueError("fp4x operators take contiguous tensors")
    return t.data_ptr()


def quantize_mxfp4(w: torch.Tensor):
    n, k = w.shape
    packed = torch.empty((n, k // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((n, k // 32), dtype=torch.uint8, device=w.device)
    check(lib().fp4_quantize_mxfp4(_stream(), n, k, _ptr(w), _ptr(packed), _ptr(scales)))
    return packed, scales


def quantize_nvfp4(w: torch.Tensor, global_scale: float = 1.0):
    """f32 [n][k] -> NVFP4 (packed [n][k/2], UE4M3 scales [n][k/16])."""
    n, k = w.shape
    packed = torch.empty((n, k // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((n, k // 16), dtype=torch.uint8, device=w.device)
    check(lib().fp4_quantize_nvfp4(_stream(), n, k, _ptr(w), _ptr(packed), _ptr(scales), global_scale))
    return packed, scales


def quantize_ref(w: torch.Tensor):
    n, k = w.shape
    packed = torch.empty((n, k // 8), dtype=torch.int32, device=w.device)
    scales = torch.empty((n, k // 32), dtype=torch.float32, device=w.device)
    check(lib().fp4_quantize_ref(_stream(), n, k, _ptr(w), _ptr(packed), _ptr(scales)))
    return packed, scales


def dequantize_mxfp4(packed: torch.Tensor, scales: torch.Tensor):
    n = packed.shape[0]
    k = packed.shape[1] * 2
    out = torch.empty((n, k), dtype=torch.float32, device=packed.device)
    check(lib().fp4_dequantize_mxfp4(_stream(), n, k, _ptr(packed), _ptr(scales), _ptr(out)))
    return out


def fill_normal(n: int, seed: int, sigma: float = 1.0, offset: int = 0, dtype=torch.float32, device="cuda"):
    out = torch.empty(n, dtype=dtype, device=device)
    if dtype == torch.float32:
        check(lib().fp4x_fill_normal_f32(_stream(), seed, offset, sigma, _ptr(out), n))
    elif dtype == torch.bfloat16:
        check(lib().fp4x_fill_normal_bf16(_stream(), seed, offset, sigma, _ptr(out), n))
    else:
        raise ValueError(dtype)
    return out


def init_mxfp4(n: int, k: int, seed: int, sigma: float = 0.02, device="cuda"):
    packed = torch.empty((n, k // 2), dtype=torch.uint8, device=device)
    scales = torch.empty((n, k // 32), dtype=torch.uint8, device=device)
    check(lib().fp4x_init_mxfp4(_stream(), seed, sigma, n, k, _ptr(packed), _ptr(scales)))
    return packed, scales


def gemv(packed: torch.Tensor, scales: torch.Tensor, x: torch.Tensor, out: torch.Tensor | None = None):
    """y = W x on native MXFP4 storage; x bf16 (fp4_gemv) or f32 (fp4_gemv_f32x)."""
    n = packed.shape[0]
    k = packed.shape[1] * 2
    y = out if out is not None else torch.empty(n, dtype=torch.float32, device=packed.device)
    if x.dtype == torch.bfloat16:
        check(lib().fp4_gemv(_stream(), n, k, _ptr(packed), _ptr(scales), _ptr(x), _ptr(y)))
    elif x.dtype == torch.float32:
        check(lib().fp4_gemv_f32x(_stream(), n, k, _ptr(packed), _ptr(scales), _ptr(x), _ptr(y)))
    else:
        raise ValueError(x.dtype)
    return y


def gemv_ref(words: torch.Tensor, scales: torch.Tensor, x: torch.Tensor):
    """The reference's storage: u32 words (as int32), f32 scales, f32 x."""
    n = words.shape[0]
    k = x.shape[0]
    y = torch.empty(n, dtype=torch.float32, device=words.device)
    check(lib().fp4_gemv_ref(_stream(), n, k, _ptr(words), _ptr(scales), _ptr(x), _ptr(y)))
    return y


def mma(a: torch.Tensor, sa: torch.Tensor, w: torch.Tensor, sw: torch.Tensor, out_dtype=torch.bfloat16):
    """d[m][n] = A W^T for MXFP4 A [m][k/2] (+ E8M0 scales [m][k/32]) and W [n][k/2]
    (+ [n][k/32]) on tcgen05.mma.kind::mxf4; bf16 (fp4_mma) or fp32 (fp4_mma_f32) out."""
    m, n, k = a.shape[0], w.shape[0], a.shape[1] * 2
    if w.shape[1] * 2 != k or sa.shape != (m, k // 32) or sw.shape != (n, k // 32):
        raise ValueError("fp4 mma: operand shapes disagree")
    d = torch.empty((m, n), dtype=out_dtype, device=a.device)
    if out_dtype == torch.float32:
        check(lib().fp4_mma_f32(_stream(), m, n, k, _ptr(a), _ptr(sa), _ptr(w), _ptr(sw), _ptr(d)))
        return d
    if out_dtype != torch.bfloat16:
        raise ValueError(out_dtype)
    ws_bytes = lib().fp4_mma_workspace_size(m, n, k)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=a.device)
    check(lib().fp4_mma(_stream(), m, n, k, _ptr(a), _ptr(sa), _ptr(w), _ptr(sw), _ptr(d), _ptr(ws), ws_bytes))
    return d


def mma_nvf4(a, sa, w, sw, alpha: float = 1.0, out_dtype=torch.bfloat16):
    """NVFP4 GEMM: d[m][n] = alpha * A W^T, UE4M3 scales per 16 values."""
    m, n, k = a.shape[0], w.shape[0], a.shape[1] * 2
    if w.shape[1] * 2 != k or sa.shape != (m, k // 16) or sw.shape != (n, k // 16):
        raise ValueError("nvf4 mma: operand shapes disagree")
    d = torch.empty((m, n), dtype=out_dtype, device=a.device)
    if out_dtype == torch.float32:
        check(lib().fp4_mma_nvf4_f32(_stream(), m, n, k, _ptr(a), _ptr(sa), _ptr(w), _ptr(sw), alpha, _ptr(d)))
        return d
    ws_bytes = lib().fp4_mma_nvf4_workspace_size(m, n, k)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=a.device)
    check(lib().fp4_mma_nvf4(_stream(), m, n, k, _ptr(a), _ptr(sa), _ptr(w), _ptr(sw), alpha, _ptr(d), _ptr(ws),
                             ws_bytes))
    return d


def mma_allones(device="cuda"):
    """The reference's all-ones known-answer test on tcgen05: [16][8], every value 64.0."""
    out = torch.full((16, 8), -1.0, dtype=torch.float32, device=device)
    check(lib().fp4_mma_allones(_stream(), _ptr(out)))
    return out


def rmsnorm(x, w, eps=1e-5):
    y = torch.empty_like(x)
    check(lib().llama_rmsnorm(_stream(), x.numel(), eps, _ptr(x), _ptr(w), _ptr(y)))
    return y


def rope_tables(n_pos: int, head_dim: int, theta: float, device="cuda"):
    c = torch.empty((n_pos, head_dim // 2), dtype=torch.float32, device=device)
    s = torch.empty_like(c)
    check(lib().llama_rope_tables(_stream(), n_pos, head_dim, float(theta), _ptr(c), _ptr(s)))
    return c, s


def rope_(q, num_heads, head_dim, cos_base, cos_t, sin_t):
    check(lib().llama_rope(_stream(), num_heads, head_dim, cos_base, _ptr(cos_t), _ptr(sin_t), _ptr(q)))
    return q


def copy_into_(dst, src, off):
    check(lib().llama_copy_into(_stream(), src.numel(), off, _ptr(src), _ptr(dst)))
    return dst


def kv_append_bf16_(dst, src, off):
    check(lib().llama_kv_append_bf16(_stream(), src.numel(), off, _ptr(src), _ptr(dst)))
    return dst


def swiglu(g, u):
    out = torch.empty_like(g)
    check(lib().llama_swiglu(_stream(), g.numel(), _ptr(g), _ptr(u), _ptr(out)))
    return out


def residual_(x, y):
    check(lib().llama_residual(_stream(), x.numel(), _ptr(y), _ptr(x)))
    return x


def argmax(logits):
    out = torch.empty(1, dtype=torch.int32, device=logits.device)
    check(lib().llama_argmax(_stream(), logits.numel(), _ptr(logits), _ptr(out)))
    return out


def attn_decode(q, kc, vc, n_heads, n_kv, seq):
    """Reference signature: f32, head_dim 64, cache [seq][n_kv][64]."""
    out = torch.empty(n_heads * 64, dtype=torch.float32, device=q.device)
    check(lib().llama_attn_decode(_stream(), n_heads, n_kv, seq, _ptr(q), _ptr(kc), _ptr(vc), _ptr(out)))
    return out


def attn_workspace(batch, n_heads, n_kv, head_dim, seq, device="cuda"):
    nbytes = lib().llama_attn_workspace_size(batch, n_heads, n_kv, head_dim, seq)
    return torch.empty(max(nbytes, 16), dtype=torch.uint8, device=device), nbytes


def attn_decode_hd(q, kc, vc, n_heads, n_kv, head_dim, seq, split=True):
    out = torch.empty(n_heads * head_dim, dtype=torch.float32, device=q.device)
    ws, nbytes = attn_workspace(1, n_heads, n_kv, head_dim, seq, q.device) if split else (None, 0)
    check(lib().llama_attn_decode_hd(_stream(), n_heads, n_kv, head_dim, seq, _ptr(q), _ptr(kc), _ptr(vc),
                                     _ptr(out), _ptr(ws) if ws is not None else None, nbytes))
    return out


def attn_decode_bf16(q, kc, vc, seq, split=True):
    """q [B][H][hd] bf16; kc/vc [B][max_seq][n_kv][hd] bf16 -> out [B][H][hd] bf16."""
    B, H, hd = q.shape
    max_seq, n_kv = kc.shape[1], kc.shape[2]
    out = torch.empty_like(q)
    ws, nbytes = attn_workspace(B, H, n_kv, hd, seq, q.device) if split else (None, 0)
    check(lib().llama_attn_decode_bf16(_stream(), B, H, n_kv, hd, seq, max_seq, _ptr(q), _ptr(kc), _ptr(vc),
                                       _ptr(out), _ptr(ws) if ws is not None else None, nbytes))
    return out
