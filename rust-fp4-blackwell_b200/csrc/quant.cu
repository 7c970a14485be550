// quant.cu -- MXFP4 quantisation, dequantisation and the seeded synthetic
// initialiser, on the device.
//
// Quantiser semantics restate quant_fp4, examples/llama_run/src/main.rs:334-376:
// per (row, 32-block) amax; nearest E2M1 level by a strict '<' scan over the
// ascending level table (ties -> smaller magnitude); v < 0 sets the sign bit even
// when the magnitude rounds to 0 (-0).  Every step is an exactly rounded f32
// operation (division, subtraction, fabs, compare), so results are bit-identical
// to the CPU loop.  The native variant takes the E8M0 scale
// 2^(floor(log2 amax) - 2) from the float's exponent bits.
#include "common.cuh"

namespace fp4x {
namespace quant {

enum { ROWMAP_IDENTITY = 0, ROWMAP_ROPE_PAIRS = 1, ROWMAP_INTERLEAVE8 = 2 };

__device__ __forceinline__ uint32_t nearest_code(float v) {
    // llama_run/src/main.rs:332,348-363
    const float levels[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    const float a = fabsf(v);
    uint32_t bc = 0;
    float bd = 3.40282347e+38f;
#pragma unroll
    for (uint32_t ci = 0; ci < 8; ++ci) {
        const float d = fabsf(__fsub_rn(a, levels[ci]));
        if (d < bd) {
            bd = d;
            bc = ci;
        }
    }
    return bc | (v < 0.0f ? 8u : 0u);
}

__device__ __forceinline__ int floor_log2_bits(float a) {
    const uint32_t u = __float_as_uint(a) & 0x7FFFFFFFu;
    const int ef = (int)(u >> 23);
    if (ef != 0) return ef - 127;
    return (31 - __clz(u & 0x7FFFFFu)) - 149;  // subnormal
}

__device__ __forceinline__ uint32_t e8m0_from_amax(float amax) {
    if (!(amax > 0.0f)) return 127u;
    int e = floor_log2_bits(amax) - 2 + 127;
    e = max(0, min(254, e));
    return (uint32_t)e;
}

// Quantise 32 values (in registers) into 16 packed bytes + the E8M0 byte.
__device__ __forceinline__ void quant_block_mxfp4(const float (&v)[32], uint4 &packed, uint8_t &sbyte) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const uint32_t e = e8m0_from_amax(amax);
    const float scale = e8m0_to_f32(e);
    uint32_t words[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 32; ++i) words[i / 8] |= nearest_code(__fdiv_rn(v[i], scale)) << ((i % 8) * 4);
    packed = make_uint4(words[0], words[1], words[2], words[3]);
    sbyte = (uint8_t)e;
}

// ---- NVFP4: E2M1 with an unsigned-E4M3 scale per 16 values and a per-tensor f32
// scale g (the reference's kind::mxf4nvf4 / .ue4m3 variant,
// trackb/FP4_M16N8K64_LAYOUT.md:7; the reference has no quantiser for it).  Rule:
// s = amax / 6 / g rounded to the nearest UE4M3 (ties to even, saturating at 448,
// zero for s <= 0), values divided by UE4M3(s) * g and rounded to E2M1 with the
// reference's tie rule.
__device__ __forceinline__ float ue4m3_to_f32(uint32_t b) {
    const uint32_t e = (b >> 3) & 15u, m = b & 7u;
    return e == 0 ? ldexpf((float)m, -9) : ldexpf((float)(8u + m), (int)e - 10);
}

__device__ __forceinline__ uint32_t f32_to_ue4m3(float s) {
    if (!(s > 0.0f)) return 0u;
    if (s >= 448.0f) return 0x7Eu;
    if (s < 0.015625f) return (uint32_t)rintf(s * 512.0f);  // subnormal step 2^-9 (8 = smallest normal)
    const int e = (int)((__float_as_uint(s) >> 23) & 0xFFu) - 127;
    const float mant = ldexpf(s, -e) - 1.0f;  // exact
    int E = e + 7, m = (int)rintf(mant * 8.0f);
    if (m == 8) E += 1, m = 0;
    if (E > 15 || (E == 15 && m == 7)) return 0x7Eu;
    return (uint32_t)((E << 3) | m);
}

// One thread per (row, 16-block).
__global__ void quant_nvfp4_kernel(uint64_t nblocks, const float *__restrict__ w, uint8_t *__restrict__ packed,
                                   uint8_t *__restrict__ scales, float g) {
    const uint64_t blk = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= nblocks) return;
    float v[16];
    const float4 *src = reinterpret_cast<const float4 *>(w + blk * 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 f = src[i];
        v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const uint32_t S = f32_to_ue4m3(__fdiv_rn(__fdiv_rn(amax, 6.0f), g));
    const float eff = __fmul_rn(ue4m3_to_f32(S), g);
    uint32_t words[2] = {0, 0};
    if (eff > 0.0f)
#pragma unroll
        for (int i = 0; i < 16; ++i) words[i / 8] |= nearest_code(__fdiv_rn(v[i], eff)) << ((i % 8) * 4);
    reinterpret_cast<uint2 *>(packed)[blk] = make_uint2(words[0], words[1]);
    scales[blk] = (uint8_t)S;
}

// One thread per (row, 32-block).
__global__ void quant_mxfp4_kernel(uint64_t nblocks, const float *__restrict__ w, uint8_t *__restrict__ packed,
                                   uint8_t *__restrict__ scales) {
    const uint64_t blk = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= nblocks) return;
    float v[32];
    const float4 *src = reinterpret_cast<const float4 *>(w + blk * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 f = src[i];
        v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
    }
    uint4 p;
    uint8_t s;
    quant_block_mxfp4(v, p, s);
    reinterpret_cast<uint4 *>(packed)[blk] = p;
    scales[blk] = s;
}

// llama_run/src/main.rs:339-365 exactly: scale = amax/6 (1.0 for a zero block).
__global__ void quant_ref_kernel(uint64_t nblocks, const float *__restrict__ w, uint32_t *__restrict__ packed,
                                 float *__restrict__ scales) {
    const uint64_t blk = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= nblocks) return;
    const float *src = w + blk * 32;
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(src[i]));
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 6.0f) : 1.0f;
    scales[blk] = scale;
    uint32_t words[4] = {0, 0, 0, 0};
    for (int i = 0; i < 32; ++i) words[i / 8] |= nearest_code(__fdiv_rn(src[i], scale)) << ((i % 8) * 4);
    for (int j = 0; j < 4; ++j) packed[blk * 4 + j] = words[j];
}

// Dequantise through the same hardware E2M1 -> f16x2 conversion the GEMV uses,
// so a bit-exact dequant test also pins the GEMV's decode.
__global__ void dequant_mxfp4_kernel(uint64_t nblocks, const uint8_t *__restrict__ packed,
                                     const uint8_t *__restrict__ scales, float *__restrict__ out) {
    const uint64_t blk = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= nblocks) return;
    const uint4 p = reinterpret_cast<const uint4 *>(packed)[blk];
    const float s = e8m0_to_f32(scales[blk]);
    const uint32_t words[4] = {p.x, p.y, p.z, p.w};
    float4 *dst = reinterpret_cast<float4 *>(out + blk * 32);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t h[4];
        decode_word_f16(words[j], h);
        float f[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const __half2 hh = *reinterpret_cast<const __half2 *>(&h[q]);
            f[2 * q] = __low2float(hh) * s;
            f[2 * q + 1] = __high2float(hh) * s;
        }
        dst[2 * j] = make_float4(f[0], f[1], f[2], f[3]);
        dst[2 * j + 1] = make_float4(f[4], f[5], f[6], f[7]);
    }
}

__global__ void fill_normal_f32_kernel(uint64_t seed, uint64_t offset, float sigma, float *__restrict__ out,
                                       uint64_t n) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = normal_draw(seed, offset + i, sigma);
}

__global__ void fill_normal_bf16_kernel(uint64_t seed, uint64_t offset, float sigma, uint16_t *__restrict__ out,
                                        uint64_t n) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = f32_to_bf16_bits(normal_draw(seed, offset + i, sigma));
}

// Generate + quantise one 32-block per thread; element index = row*k + col.
__global__ void init_mxfp4_kernel(uint64_t seed, float sigma, uint64_t nblocks, uint8_t *__restrict__ packed,
                                  uint8_t *__restrict__ scales) {
    const uint64_t blk = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= nblocks) return;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = normal_draw(seed, blk * 32 + i, sigma);
    uint4 p;
    uint8_t s;
    quant_block_mxfp4(v, p, s);
    reinterpret_cast<uint4 *>(packed)[blk] = p;
    scales[blk] = s;
}

// Destination row of source row r for the engine's fused layouts.
//   ROWMAP_IDENTITY:  r + off
//   ROWMAP_ROPE_PAIRS: rows of each head regrouped into 16-row tiles whose rows
//     0..7 are head rows j0..j0+7 and rows 8..15 are j0+hd/2..j0+hd/2+7, so a
//     rotate-half pair (j, j+hd/2) lands in one mma tile (rows g, g+8)
//   ROWMAP_INTERLEAVE8: 8-row groups interleaved with a partner tensor in
//     16-row tiles (gate rows at off 0, up rows at off 8)
__device__ __forceinline__ uint32_t map_row(uint32_t r, int mode, uint32_t off, uint32_t hd) {
    if (mode == ROWMAP_ROPE_PAIRS) {
        const uint32_t half = hd / 2, head = r / hd, j = r % hd;
        const uint32_t jj = j < half ? j : j - half;
        return off + (head * (half / 8) + jj / 8) * 16 + (j < half ? 0u : 8u) + jj % 8;
    }
    if (mode == ROWMAP_INTERLEAVE8) return (r / 8) * 16 + (r % 8) + off;
    return r + off;
}

// Rows [row0, row0 + n) and columns [col0, col0 + k) of the global [*][k_global]
// tensor `seed` (a tensor-parallel shard; row0 = col0 = 0, k_global = k for the
// whole tensor): element (R, C) draws normal(seed, R * k_global + C).
__global__ void init_mxfp4_rowmap_kernel(uint64_t seed, float sigma, uint32_t n, uint32_t k, uint8_t *__restrict__ packed,
                                         uint8_t *__restrict__ scales, int mode, uint32_t off, uint32_t hd,
                                         uint32_t row0, uint32_t k_global, uint32_t col0) {
    const uint64_t blk = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t nbr = k / 32;
    if (blk >= (uint64_t)n * nbr) return;
    const uint32_t r = (uint32_t)(blk / nbr), b = (uint32_t)(blk % nbr);
    const uint64_t e0 = (uint64_t)(row0 + r) * k_global + col0 + 32u * b;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = normal_draw(seed, e0 + i, sigma);
    uint4 p;
    uint8_t s;
    quant_block_mxfp4(v, p, s);
    const uint64_t dblk = (uint64_t)map_row(r, mode, off, hd) * nbr + b;
    reinterpret_cast<uint4 *>(packed)[dblk] = p;
    scales[dblk] = s;
}

inline unsigned grid_for(uint64_t n, unsigned block) { return (unsigned)((n + block - 1) / block); }

}  // namespace quant
}  // namespace fp4x

namespace fp4x {
namespace quant {
// Engine helper: generate tensor `seed` ([n][k], N(0, sigma)) straight into a
// fused layout (row map above).
int init_mxfp4_rowmap(cudaStream_t stream, uint64_t seed, float sigma, uint32_t n, uint32_t k, uint8_t *packed,
                      uint8_t *scales, int mode, uint32_t off, uint32_t hd, uint32_t row0, uint32_t k_global,
                      uint32_t col0) {
    const uint64_t nb = (uint64_t)n * (k / 32);
    init_mxfp4_rowmap_kernel<<<grid_for(nb, 128), 128, 0, stream>>>(seed, sigma, n, k, packed, scales, mode, off, hd,
                                                                     row0, k_global ? k_global : k, col0);
    return check_launch("init_mxfp4_rowmap");
}
}  // namespace quant
}  // namespace fp4x

using namespace fp4x;

extern "C" int fp4_quantize_nvfp4(fp4x_stream_t stream, uint32_t n, uint32_t k, const float *w, uint8_t *packed,
                                  uint8_t *scales, float global_scale) {
    FP4X_REQUIRE(w && packed && scales, "fp4_quantize_nvfp4: null pointer");
    FP4X_REQUIRE(k % 16 == 0 && k > 0 && n > 0, "fp4_quantize_nvfp4: k=%u must be a positive multiple of 16", k);
    FP4X_REQUIRE(global_scale > 0.0f && global_scale < 3.0e38f, "fp4_quantize_nvfp4: global scale must be positive");
    FP4X_REQUIRE(aligned16(w) && ((uintptr_t)packed & 7u) == 0, "fp4_quantize_nvfp4: w 16-byte, packed 8-byte aligned");
    const uint64_t nb = (uint64_t)n * (k / 16);
    quant::quant_nvfp4_kernel<<<quant::grid_for(nb, 128), 128, 0, (cudaStream_t)stream>>>(nb, w, packed, scales,
                                                                                        global_scale);
    return check_launch("fp4_quantize_nvfp4");
}

extern "C" int fp4_quantize_mxfp4(fp4x_stream_t stream, uint32_t n, uint32_t k, const float *w, uint8_t *packed,
                                  uint8_t *scales) {
    FP4X_REQUIRE(w && packed && scales, "fp4_quantize_mxfp4: null pointer");
    FP4X_REQUIRE(k % 32 == 0 && k > 0 && n > 0, "fp4_quantize_mxfp4: k=%u must be a positive multiple of 32", k);
    FP4X_REQUIRE(aligned16(w) && aligned16(packed), "fp4_quantize_mxfp4: w and packed must be 16-byte aligned");
    const uint64_t nb = (uint64_t)n * (k / 32);
    quant::quant_mxfp4_kernel<<<quant::grid_for(nb, 128), 128, 0, (cudaStream_t)stream>>>(nb, w, packed, scales);
    return check_launch("fp4_quantize_mxfp4");
}

extern "C" int fp4_quantize_ref(fp4x_stream_t stream, uint32_t n, uint32_t k, const float *w, uint32_t *packed,
                                float *scales) {
    FP4X_REQUIRE(w && packed && scales, "fp4_quantize_ref: null pointer");
    FP4X_REQUIRE(k % 32 == 0 && k > 0 && n > 0, "fp4_quantize_ref: k=%u must be a positive multiple of 32", k);
    const uint64_t nb = (uint64_t)n * (k / 32);
    quant::quant_ref_kernel<<<quant::grid_for(nb, 128), 128, 0, (cudaStream_t)stream>>>(nb, w, packed, scales);
    return check_launch("fp4_quantize_ref");
}

extern "C" int fp4_dequantize_mxfp4(fp4x_stream_t stream, uint32_t n, uint32_t k, const uint8_t *packed,
                                    const uint8_t *scales, float *out) {
    FP4X_REQUIRE(out && packed && scales, "fp4_dequantize_mxfp4: null pointer");
    FP4X_REQUIRE(k % 32 == 0 && k > 0 && n > 0, "fp4_dequantize_mxfp4: k=%u must be a positive multiple of 32", k);
    FP4X_REQUIRE(aligned16(out) && aligned16(packed), "fp4_dequantize_mxfp4: out and packed must be 16-byte aligned");
    const uint64_t nb = (uint64_t)n * (k / 32);
    quant::dequant_mxfp4_kernel<<<quant::grid_for(nb, 128), 128, 0, (cudaStream_t)stream>>>(nb, packed, scales, out);
    return check_launch("fp4_dequantize_mxfp4");
}

extern "C" int fp4x_fill_normal_f32(fp4x_stream_t stream, uint64_t seed, uint64_t offset, float sigma, float *out,
                                    size_t n) {
    FP4X_REQUIRE(out || n == 0, "fp4x_fill_normal_f32: null pointer");
    if (n == 0) return FP4X_OK;
    const unsigned grid = (unsigned)std::min<uint64_t>(quant::grid_for(n, 256), 148u * 16u);
    quant::fill_normal_f32_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(seed, offset, sigma, out, n);
    return check_launch("fp4x_fill_normal_f32");
}

extern "C" int fp4x_fill_normal_bf16(fp4x_stream_t stream, uint64_t seed, uint64_t offset, float sigma,
                                     uint16_t *out, size_t n) {
    FP4X_REQUIRE(out || n == 0, "fp4x_fill_normal_bf16: null pointer");
    if (n == 0) return FP4X_OK;
    const unsigned grid = (unsigned)std::min<uint64_t>(quant::grid_for(n, 256), 148u * 16u);
    quant::fill_normal_bf16_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(seed, offset, sigma, out, n);
    return check_launch("fp4x_fill_normal_bf16");
}

extern "C" int fp4x_init_mxfp4(fp4x_stream_t stream, uint64_t seed, float sigma, uint32_t n, uint32_t k,
                               uint8_t *packed, uint8_t *scales) {
    FP4X_REQUIRE(packed && scales, "fp4x_init_mxfp4: null pointer");
    FP4X_REQUIRE(k % 32 == 0 && k > 0 && n > 0, "fp4x_init_mxfp4: k=%u must be a positive multiple of 32", k);
    FP4X_REQUIRE(aligned16(packed), "fp4x_init_mxfp4: packed must be 16-byte aligned");
    const uint64_t nb = (uint64_t)n * (k / 32);
    quant::init_mxfp4_kernel<<<quant::grid_for(nb, 128), 128, 0, (cudaStream_t)stream>>>(seed, sigma, nb, packed,
                                                                                         scales);
    return check_launch("fp4x_init_mxfp4");
}
