// elementwise.cu -- the small per-token operators of the decode step, standalone.
//
// These are the C-ABI twins of the reference's rmsnorm / rope / copy_into /
// swiglu / residual / argmax kernels (examples/llama_run/src/main.rs:79-315).
// The decode engine fuses them into the GEMV prologues/epilogues; the
// standalone forms exist so each operator is a drop-in and parity-testable.
#include "common.cuh"

#include <cmath>
#include <vector>

namespace fp4x {
namespace ew {

constexpr int kBlock = 256;

__device__ __forceinline__ float block_sum(float v, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
    for (int i = 0; i < nw; ++i) s += red[i];  // fixed order
    __syncthreads();
    return s;
}

// llama_run/src/main.rs:79-116: one CTA, sum of squares, then y = x * rms * w.
__global__ void __launch_bounds__(1024) rmsnorm_kernel(uint32_t dim, float eps, const float *__restrict__ x,
                                                       const float *__restrict__ w, float *__restrict__ y) {
    __shared__ float red[32];
    float ss = 0.0f;
    for (uint32_t i = threadIdx.x; i < dim; i += blockDim.x) {
        const float v = x[i];
        ss += v * v;
    }
    const float total = block_sum(ss, red);
    const float rms = 1.0f / sqrtf(total / (float)dim + eps);
    for (uint32_t i = threadIdx.x; i < dim; i += blockDim.x) y[i] = x[i] * rms * w[i];
}

// llama_run/src/main.rs:118-138: one thread per (head, j < hd/2) pair.
__global__ void rope_kernel(uint32_t num_heads, uint32_t head_dim, uint32_t cos_base,
                            const float *__restrict__ cos_t, const float *__restrict__ sin_t, float *__restrict__ q) {
    const uint32_t half = head_dim / 2;
    const uint32_t gid = blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= num_heads * half) return;
    const uint32_t head = gid / half, j = gid % half, base = head * head_dim;
    const float c = cos_t[cos_base + j], s = sin_t[cos_base + j];
    const float x0 = q[base + j], x1 = q[base + j + half];
    q[base + j] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    q[base + j + half] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
}

__global__ void copy_into_kernel(uint32_t n, uint32_t off, const float *__restrict__ src, float *__restrict__ dst) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[(size_t)off + i] = src[i];
}

__global__ void kv_append_bf16_kernel(uint32_t n, uint32_t off, const float *__restrict__ src,
                                      uint16_t *__restrict__ dst) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[(size_t)off + i] = f32_to_bf16_bits(src[i]);
}

// llama_run/src/main.rs:244-252
__global__ void swiglu_kernel(uint32_t n, const float *__restrict__ g, const float *__restrict__ u,
                              float *__restrict__ out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float gv = g[i];
        out[i] = gv / (1.0f + expf(-gv)) * u[i];
    }
}

// llama_run/src/main.rs:254-261
__global__ void residual_kernel(uint32_t n, const float *__restrict__ y, float *__restrict__ x) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = x[i] + y[i];
}

// (value, index) ordering of llama_run/src/main.rs:287: larger value wins, ties to the lower index.
__device__ __forceinline__ void argmax_merge(float &bv, uint32_t &bi, float ov, uint32_t oi) {
    if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
    }
}

__global__ void __launch_bounds__(1024) argmax_kernel(uint32_t n, const float *__restrict__ logits,
                                                      uint32_t *__restrict__ out) {
    __shared__ float mv[32];
    __shared__ uint32_t mi[32];
    float bv = -1e30f;
    uint32_t bi = 0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = logits[i];
        if (v > bv) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        mv[warp] = bv;
        mi[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float gv = -1e30f;
        uint32_t gi = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) argmax_merge(gv, gi, mv[w], mi[w]);
        out[0] = gi;
    }
}

inline uint32_t blocks_for(uint32_t n) { return (n + kBlock - 1) / kBlock; }

}  // namespace ew
}  // namespace fp4x

using namespace fp4x;

extern "C" int llama_rmsnorm(fp4x_stream_t stream, uint32_t dim, float eps, const float *x, const float *weight,
                             float *y) {
    FP4X_REQUIRE(x && weight && y, "llama_rmsnorm: null pointer");
    FP4X_REQUIRE(dim > 0, "llama_rmsnorm: dim must be > 0");
    ew::rmsnorm_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(dim, eps, x, weight, y);
    return check_launch("llama_rmsnorm");
}

extern "C" int llama_rope(fp4x_stream_t stream, uint32_t num_heads, uint32_t head_dim, uint32_t cos_base,
                          const float *cos_t, const float *sin_t, float *q) {
    FP4X_REQUIRE(cos_t && sin_t && q, "llama_rope: null pointer");
    FP4X_REQUIRE(head_dim >= 2 && head_dim % 2 == 0, "llama_rope: head_dim must be even");
    FP4X_REQUIRE(num_heads > 0, "llama_rope: num_heads must be > 0");
    const uint32_t n = num_heads * (head_dim / 2);
    ew::rope_kernel<<<ew::blocks_for(n), ew::kBlock, 0, (cudaStream_t)stream>>>(num_heads, head_dim, cos_base,
                                                                               cos_t, sin_t, q);
    return check_launch("llama_rope");
}

extern "C" int llama_rope_tables(fp4x_stream_t stream, uint32_t n_pos, uint32_t head_dim, double theta,
                                 float *cos_t, float *sin_t) {
    FP4X_REQUIRE(cos_t && sin_t, "llama_rope_tables: null pointer");
    FP4X_REQUIRE(head_dim >= 2 && head_dim % 2 == 0 && n_pos > 0, "llama_rope_tables: bad shape");
    const uint32_t half = head_dim / 2;
    std::vector<float> c((size_t)n_pos * half), s((size_t)n_pos * half);
    // llama_run/src/main.rs:464-471 (f64 angle, cast to f32)
    for (uint32_t pos = 0; pos < n_pos; ++pos)
        for (uint32_t j = 0; j < half; ++j) {
            const double freq = 1.0 / std::pow(theta, 2.0 * (double)j / (double)head_dim);
            const double a = (double)pos * freq;
            c[(size_t)pos * half + j] = (float)std::cos(a);
            s[(size_t)pos * half + j] = (float)std::sin(a);
        }
    cudaError_t e = cudaMemcpyAsync(cos_t, c.data(), c.size() * 4, cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(sin_t, s.data(), s.size() * 4, cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);  // host vectors go out of scope
    if (e != cudaSuccess) {
        set_error("llama_rope_tables: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    return FP4X_OK;
}

extern "C" int llama_copy_into(fp4x_stream_t stream, uint32_t n, uint32_t off, const float *src, float *dst) {
    FP4X_REQUIRE(src && dst, "llama_copy_into: null pointer");
    if (n == 0) return FP4X_OK;
    ew::copy_into_kernel<<<ew::blocks_for(n), ew::kBlock, 0, (cudaStream_t)stream>>>(n, off, src, dst);
    return check_launch("llama_copy_into");
}

extern "C" int llama_kv_append_bf16(fp4x_stream_t stream, uint32_t n, uint32_t off, const float *src,
                                    uint16_t *dst) {
    FP4X_REQUIRE(src && dst, "llama_kv_append_bf16: null pointer");
    if (n == 0) return FP4X_OK;
    ew::kv_append_bf16_kernel<<<ew::blocks_for(n), ew::kBlock, 0, (cudaStream_t)stream>>>(n, off, src, dst);
    return check_launch("llama_kv_append_bf16");
}

extern "C" int llama_swiglu(fp4x_stream_t stream, uint32_t n, const float *gate, const float *up, float *out) {
    FP4X_REQUIRE(gate && up && out, "llama_swiglu: null pointer");
    if (n == 0) return FP4X_OK;
    ew::swiglu_kernel<<<ew::blocks_for(n), ew::kBlock, 0, (cudaStream_t)stream>>>(n, gate, up, out);
    return check_launch("llama_swiglu");
}

extern "C" int llama_residual(fp4x_stream_t stream, uint32_t n, const float *y, float *x) {
    FP4X_REQUIRE(y && x, "llama_residual: null pointer");
    if (n == 0) return FP4X_OK;
    ew::residual_kernel<<<ew::blocks_for(n), ew::kBlock, 0, (cudaStream_t)stream>>>(n, y, x);
    return check_launch("llama_residual");
}

extern "C" int llama_argmax(fp4x_stream_t stream, uint32_t n, const float *logits, uint32_t *out) {
    FP4X_REQUIRE(logits && out, "llama_argmax: null pointer");
    FP4X_REQUIRE(n > 0, "llama_argmax: n must be > 0");
    ew::argmax_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(n, logits, out);
    return check_launch("llama_argmax");
}
