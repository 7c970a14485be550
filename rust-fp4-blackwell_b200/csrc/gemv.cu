// gemv.cu -- batch-1 MXFP4 decode GEMV for sm_100a (the fp4_gemv operator).
//
// Replaces fp4_gemv, examples/llama_run/src/main.rs:34-77.  The reference runs
// one warp per row with scalar 32-bit loads and an f32 FMA per weight.  Here:
//   * a CTA owns a 16-row tile of W; its whole [16 x K/2] byte slab is copied
//     into shared memory with cp.async.bulk (one copy per row and warp slice,
//     completion counted on per-warp mbarriers), so HBM sees only 16-byte
//     aligned bulk reads of each weight byte exactly once;
//   * the activation is staged once per CTA as an f16 hi/lo pair (x*2^s = hi + lo
//     with a power-of-two prescale s), which carries ~22 bits of the activation;
//   * E2M1 nibbles are decoded in registers to f16 (cvt.rn.f16x2.e2m1x2) and
//     contracted on the tensor cores with mma.m16n8k16 (column 0 = hi, column 1
//     = lo of the activation), fp32 accumulation; each 32-block's partial sum is
//     scaled by its E8M0 scale in fp32 and accumulated in fp32;
//   * the four warps split K and are reduced in a fixed order (deterministic).
// Bound: HBM.  Algorithmic bytes per call = N*K/2 + N*K/32 + |x| + 4N.
#include "common.cuh"

#include <algorithm>

namespace fp4x {

namespace gemv {

constexpr int kRows = 16;   // rows per CTA (one mma M tile)
constexpr int kWarps = 4;   // K split across warps
constexpr int kThreads = kWarps * 32;

// Scale element loaders: E8M0 byte or the reference's f32 scale.
__device__ __forceinline__ float load_scale(const uint8_t *s) { return e8m0_to_f32(*s); }
__device__ __forceinline__ float load_scale(const float *s) { return *s; }

__device__ __forceinline__ float load_x(const uint16_t *x, uint32_t i) { return bf16_bits_to_f32(x[i]); }
__device__ __forceinline__ float load_x(const float *x, uint32_t i) { return x[i]; }

__host__ __device__ inline uint32_t padded_blocks(uint32_t nb) { return (nb % 2 == 0) ? nb + 1 : nb + 2; }

template <typename ST>
__host__ __device__ inline size_t smem_bytes(uint32_t k) {
    const uint32_t nb = k / 32;
    size_t off = 64;                                   // 4 mbarriers + pad
    off += (size_t)k * 2 * sizeof(__half);             // x hi / lo
    off += 64;                                         // reduction scratch [4][16] floats? (below)
    off += (size_t)kWarps * kRows * sizeof(float);
    off = (off + 15) & ~size_t(15);
    off += (size_t)kRows * nb * sizeof(ST);            // scales
    off = (off + 127) & ~size_t(127);
    off += (size_t)kRows * padded_blocks(nb) * 16;     // weight slab
    return off;
}

// y[row0..row0+15] for one 16-row tile.  ST = scale storage type, XT = x type.
template <typename ST, typename XT>
__global__ void __launch_bounds__(kThreads) gemv_tile_kernel(uint32_t n, uint32_t k, const uint8_t *__restrict__ w,
                                                             const ST *__restrict__ scales,
                                                             const XT *__restrict__ x, float *__restrict__ y) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t nb = k / 32;
    const uint32_t pnb = padded_blocks(nb);
    const uint32_t row_stride = pnb * 16;

    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    __half *xhi = reinterpret_cast<__half *>(smem + 64);
    __half *xlo = xhi + k;
    float *red = reinterpret_cast<float *>(smem + 64 + (size_t)k * 4 + 64);
    size_t off = 64 + (size_t)k * 4 + 64 + kWarps * kRows * sizeof(float);
    off = (off + 15) & ~size_t(15);
    ST *ssm = reinterpret_cast<ST *>(smem + off);
    off += (size_t)kRows * nb * sizeof(ST);
    off = (off + 127) & ~size_t(127);
    uint8_t *wt = smem + off;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t row0 = blockIdx.x * kRows;
    const uint32_t rows = min((uint32_t)kRows, n - row0);

    // warp w's block range along K
    const uint32_t wb0 = (nb * warp) / kWarps, wb1 = (nb * (warp + 1)) / kWarps;

    if (tid == 0) {
        for (int i = 0; i < kWarps; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            for (int i = 0; i < kWarps; ++i) {
                const uint32_t b0 = (nb * i) / kWarps, b1 = (nb * (i + 1)) / kWarps;
                mbar_arrive_expect_tx(&bars[i], rows * (b1 - b0) * 16);
            }
        }
        __syncwarp();
        const uint64_t pol = policy_evict_first();
        // lane -> (row, warp slice); 16 rows x 4 slices = 64 copies over 32 lanes
        for (int c = lane; c < kRows * kWarps; c += 32) {
            const uint32_t r = c % kRows, s = c / kRows;
            const uint32_t b0 = (nb * s) / kWarps, b1 = (nb * (s + 1)) / kWarps;
            if (r < rows && b1 > b0)
                bulk_g2s_hint(wt + r * row_stride + b0 * 16, w + (size_t)(row0 + r) * (k / 2) + b0 * 16,
                              (b1 - b0) * 16, &bars[s], pol);
        }
    }

    // activation: x*2^s = hi + lo (f16 pair), s chosen so max|x|*2^s is in [2^14, 2^15)
    float amax = 0.0f;
    for (uint32_t i = tid; i < k; i += kThreads) amax = fmaxf(amax, fabsf(load_x(x, i)));
    amax = warp_max(amax);
    if (lane == 0) red[warp] = amax;
    // scales of this tile
    for (uint32_t i = tid; i < kRows * nb; i += kThreads) {
        const uint32_t r = i / nb, b = i % nb;
        ssm[i] = (r < rows) ? scales[(size_t)(row0 + r) * nb + b] : ST(0);
    }
    __syncthreads();
    amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    int sexp = 0;
    if (amax > 0.0f && amax < 3.0e38f) {
        int e;
        frexpf(amax, &e);            // amax in [2^(e-1), 2^e)
        sexp = 15 - e;               // amax * 2^sexp in [2^14, 2^15)
        sexp = max(-126, min(126, sexp));
    }
    const float pre = ldexpf(1.0f, sexp), post = ldexpf(1.0f, -sexp);
    for (uint32_t i = tid; i < k; i += kThreads) {
        const float v = load_x(x, i) * pre;
        const __half h = __float2half_rn(v);
        xhi[i] = h;
        xlo[i] = __float2half_rn(v - __half2float(h));
    }
    __syncthreads();

    const int g = lane >> 2, t = lane & 3;
    float acc0 = 0.0f, acc1 = 0.0f;  // rows g and g+8 (meaningful on t == 0)

    if (mbar_wait_bounded(&bars[warp], 0)) {
        const __half *xsel = (g == 0) ? xhi : xlo;
        const bool xlive = g < 2;
        // ldmatrix row address of this lane: matrix j = lane/8 -> (row half, block offset)
        const int mj = lane >> 3, mi = lane & 7;
        const uint8_t *lrow = wt + (mi + 8 * (mj & 1)) * row_stride + (mj >> 1) * 16;
        const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t b = wb0;
        for (; b + 2 <= wb1; b += 2) {
            uint32_t r[4];
            ldmatrix_x4(r, lrow + b * 16);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const uint32_t bb = b + half;
                uint32_t ha[4], hb[4];
                decode_word_f16(r[2 * half + 0], ha);  // row g
                decode_word_f16(r[2 * half + 1], hb);  // row g+8
                uint4 xv = *reinterpret_cast<const uint4 *>(xsel + bb * 32 + 8 * t);
                if (!xlive) xv = make_uint4(0, 0, 0, 0);
                float d[4];
                const uint32_t a0[4] = {ha[0], hb[0], ha[1], hb[1]};
                const uint32_t a1[4] = {ha[2], hb[2], ha[3], hb[3]};
                mma_f16_16816(d, a0, xv.x, xv.y, zero4);
                mma_f16_16816(d, a1, xv.z, xv.w, d);
                acc0 += load_scale(&ssm[g * nb + bb]) * (d[0] + d[1]);
                acc1 += load_scale(&ssm[(g + 8) * nb + bb]) * (d[2] + d[3]);
            }
        }
        if (b < wb1) {
            uint32_t r[2];
            ldmatrix_x2(r, lrow + b * 16);  // lanes 0..15 supply addresses of matrices 0,1
            uint32_t ha[4], hb[4];
            decode_word_f16(r[0], ha);
            decode_word_f16(r[1], hb);
            uint4 xv = *reinterpret_cast<const uint4 *>(xsel + b * 32 + 8 * t);
            if (!xlive) xv = make_uint4(0, 0, 0, 0);
            float d[4];
            const uint32_t a0[4] = {ha[0], hb[0], ha[1], hb[1]};
            const uint32_t a1[4] = {ha[2], hb[2], ha[3], hb[3]};
            mma_f16_16816(d, a0, xv.x, xv.y, zero4);
            mma_f16_16816(d, a1, xv.z, xv.w, d);
            acc0 += load_scale(&ssm[g * nb + b]) * (d[0] + d[1]);
            acc1 += load_scale(&ssm[(g + 8) * nb + b]) * (d[2] + d[3]);
        }
    }
    __syncthreads();  // red[] reuse
    if (t == 0) {
        red[warp * kRows + g] = acc0;
        red[warp * kRows + g + 8] = acc1;
    }
    __syncthreads();
    if (tid < (int)rows) {
        float s = red[tid];
#pragma unroll
        for (int i = 1; i < kWarps; ++i) s += red[i * kRows + tid];
        y[row0 + tid] = s * post;
    }
}

template <typename ST, typename XT>
int launch(cudaStream_t stream, uint32_t n, uint32_t k, const uint8_t *w, const ST *scales, const XT *x, float *y,
           uint32_t kmax) {
    FP4X_REQUIRE(w && scales && x && y, "fp4_gemv: null pointer");
    FP4X_REQUIRE(n > 0, "fp4_gemv: n must be > 0");
    FP4X_REQUIRE(k >= 32 && k % 32 == 0 && k <= kmax, "fp4_gemv: k=%u must be a multiple of 32 in [32, %u]", k,
                 kmax);
    FP4X_REQUIRE(aligned16(w), "fp4_gemv: weights must be 16-byte aligned");
    const size_t smem = smem_bytes<ST>(k);
    auto kern = gemv_tile_kernel<ST, XT>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) {
            set_error("fp4_gemv: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            return FP4X_ECUDA;
        }
    }
    const uint32_t grid = (n + kRows - 1) / kRows;
    kern<<<grid, kThreads, smem, stream>>>(n, k, w, scales, x, y);
    return check_launch("fp4_gemv");
}

}  // namespace gemv
}  // namespace fp4x

using namespace fp4x;

extern "C" int fp4_gemv(fp4x_stream_t stream, uint32_t n, uint32_t k, const uint8_t *w, const uint8_t *scales,
                        const uint16_t *x, float *y) {
    return gemv::launch<uint8_t, uint16_t>((cudaStream_t)stream, n, k, w, scales, x, y, 16384);
}

extern "C" int fp4_gemv_f32x(fp4x_stream_t stream, uint32_t n, uint32_t k, const uint8_t *w, const uint8_t *scales,
                             const float *x, float *y) {
    return gemv::launch<uint8_t, float>((cudaStream_t)stream, n, k, w, scales, x, y, 16384);
}

extern "C" int fp4_gemv_ref(fp4x_stream_t stream, uint32_t n, uint32_t k, const uint32_t *w, const float *scales,
                            const float *x, float *y) {
    return gemv::launch<float, float>((cudaStream_t)stream, n, k, reinterpret_cast<const uint8_t *>(w), scales, x,
                                      y, 8192);
}
