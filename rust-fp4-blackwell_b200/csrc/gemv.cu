// gemv.cu -- batch-1 MXFP4 decode GEMV for sm_100a (the fp4_gemv operator) and
// its fused forms used by the decode engine.
//
// Replaces fp4_gemv, examples/llama_run/src/main.rs:34-77.  The reference runs
// one warp per row with scalar 32-bit loads and an f32 FMA per weight.  Here:
//   * a CTA owns a 16-row tile of W; its whole [16 x K/2] byte slab is copied
//     into shared memory with cp.async.bulk (one copy per row and warp slice,
//     completion counted on per-warp mbarriers, L2 evict-first), so HBM sees
//     only 16-byte aligned bulk reads of each weight byte, exactly once;
//   * the copies are issued BEFORE the kernel waits on its predecessor
//     (programmatic dependent launch): weights never depend on activations, so
//     a kernel's weight stream overlaps the tail of the previous kernel;
//   * the activation is staged once per CTA as an f16 hi/lo pair (x*2^s = hi + lo,
//     power-of-two prescale s), carrying ~22 bits of the f32 activation;
//   * E2M1 nibbles are decoded in registers to f16 with the sm_100a hardware
//     conversion (cvt.rn.f16x2.e2m1x2) and contracted on the tensor cores with
//     mma.m16n8k16 (column 0 = hi, column 1 = lo), fp32 accumulation; each 32-
//     block's sum is scaled by its E8M0 scale in fp32;
//   * the eight warps split K and are reduced in a fixed order (deterministic);
//   * prologues fuse RMSNorm (llama_run:79-116) and the embedding gather
//     (llama_run:509-510); epilogues fuse the residual add (:254-261), SwiGLU
//     (:244-252) and RoPE + bf16 KV append (:118-146).
// Bound: HBM.  Algorithmic bytes per call = N*K/2 + N*K/32 (+ |x| + |y|).
#include "common.cuh"
#include "gemv.cuh"

#include <algorithm>

namespace fp4x {
namespace gemv {

// Scale element loaders: E8M0 byte or the reference's f32 scale.
__device__ __forceinline__ float load_scale(const uint8_t *s) { return e8m0_to_f32(*s); }
__device__ __forceinline__ float load_scale(const float *s) { return *s; }

__device__ __forceinline__ float load_x(const uint16_t *x, size_t i) { return bf16_bits_to_f32(x[i]); }
__device__ __forceinline__ float load_x(const float *x, size_t i) { return x[i]; }

__host__ __device__ inline uint32_t padded_blocks(uint32_t nb) { return (nb % 2 == 0) ? nb + 1 : nb + 2; }

struct Layout {
    uint32_t xs, xpost, red, ssm, wt, total;
};

constexpr uint32_t kRedFloats = 256;

template <typename ST>
__host__ __device__ inline Layout layout(uint32_t k) {
    const uint32_t nb = k / 32;
    Layout L;
    uint32_t off = 16;  // mbarrier
    L.xs = off;
    off += k * 4;  // x hi [k] + lo [k] (f16)
    L.xpost = off;
    off += nb * 4;  // per-32-block activation post-scale 2^-s
    L.red = off;
    off += kRedFloats * 4;
    off = (off + 127) & ~127u;  // scales are bulk-copied: 16-byte aligned rows
    L.ssm = off;
    off += kRows * nb * (uint32_t)sizeof(ST);
    off = (off + 127) & ~127u;
    L.wt = off;
    off += kRows * padded_blocks(nb) * 16;
    L.total = off;
    return L;
}

// Source of activation element i (before the hi/lo split) and its elementwise
// factor: the RMSNorm weight, 1 without a norm.
template <int PRO, typename XT>
struct Prologue;

__device__ __forceinline__ float4 load4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float4 load4(const uint16_t *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xFFFF0000u));
}

template <typename XT>
struct Prologue<PRO_NONE, XT> {
    const XT *x;
    __device__ void init(const Args &a) { x = reinterpret_cast<const XT *>(a.x); }
    __device__ __forceinline__ float4 raw4(size_t i) const { return load4(x + i); }
    __device__ __forceinline__ float4 weight4(size_t) const { return make_float4(1.f, 1.f, 1.f, 1.f); }
};

template <typename XT>
struct Prologue<PRO_RMSNORM, XT> {
    const float *x, *w;
    __device__ void init(const Args &a) {
        x = reinterpret_cast<const float *>(a.x);
        w = a.norm_w;
    }
    __device__ __forceinline__ float4 raw4(size_t i) const { return load4(x + i); }
    __device__ __forceinline__ float4 weight4(size_t i) const { return load4(w + i); }
};

// Embedding row of the token at *tok (bf16 -> f32, llama_run:509-510 /
// llama_run:425), written to the residual stream by CTA 0, then RMSNorm.
template <typename XT>
struct Prologue<PRO_EMBED_RMSNORM, XT> {
    const uint16_t *row;
    const float *w;
    __device__ void init(const Args &a) {
        row = a.embed + (size_t)(*a.tok) * a.k;
        w = a.norm_w;
    }
    __device__ __forceinline__ float4 raw4(size_t i) const { return load4(row + i); }
    __device__ __forceinline__ float4 weight4(size_t i) const { return load4(w + i); }
};

// Split four consecutive activation values (this lane's share of a 32-block held
// by 8 lanes) into f16 hi/lo with a power-of-two prescale 2^s that puts the
// block's max magnitude in [2^14, 2^15): v*2^s = hi + lo carries ~22 bits of v;
// 2^-s is applied in fp32 after the mma.
__device__ __forceinline__ void split4(float4 v, uint32_t i, uint32_t b, int lane, bool valid, __half *xhi,
                                       __half *xlo, float *xpost) {
    // all 32 lanes take part (the shuffles stay inside each 8-lane block group)
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    const int ex = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;
    int s = (m > 0.0f && ex < 128 && ex > -127) ? 14 - ex : 0;
    s = max(-126, min(126, s));
    const float pre = __uint_as_float((uint32_t)(s + 127) << 23);
    const float a0 = v.x * pre, a1 = v.y * pre, a2 = v.z * pre, a3 = v.w * pre;
    const __half2 h01 = __floats2half2_rn(a0, a1), h23 = __floats2half2_rn(a2, a3);
    const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
    const __half2 l01 = __floats2half2_rn(a0 - f01.x, a1 - f01.y), l23 = __floats2half2_rn(a2 - f23.x, a3 - f23.y);
    if (!valid) return;
    *reinterpret_cast<uint2 *>(xhi + i) =
        make_uint2(*reinterpret_cast<const uint32_t *>(&h01), *reinterpret_cast<const uint32_t *>(&h23));
    *reinterpret_cast<uint2 *>(xlo + i) =
        make_uint2(*reinterpret_cast<const uint32_t *>(&l01), *reinterpret_cast<const uint32_t *>(&l23));
    if ((lane & 7) == 0) xpost[b] = __uint_as_float((uint32_t)(127 - s) << 23);
}

// Plain GEMVs (no fused prologue) are register-capped so that five CTAs fit an SM:
// a call's grid is ~2.4 CTAs per SM, so the next call's CTAs (launched early by
// programmatic dependent launch) can all be resident and stream their weights
// while this call finishes (config 0: 5.51 -> 4.68 us per call in a 64-call graph).
// The fused forms keep the default budget (capped, they would spill).
template <typename ST, typename XT, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, PRO == PRO_NONE ? 5 : 1) gemv_kernel(Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t k = a.k, n = a.n;
    const uint32_t nb = k / 32;
    const uint32_t row_stride = padded_blocks(nb) * 16;
    const Layout L = layout<ST>(k);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
    __half *xhi = reinterpret_cast<__half *>(smem + L.xs);
    __half *xlo = xhi + k;
    float *xpost = reinterpret_cast<float *>(smem + L.xpost);
    float *red = reinterpret_cast<float *>(smem + L.red);
    ST *ssm = reinterpret_cast<ST *>(smem + L.ssm);
    uint8_t *wt = smem + L.wt;
    const uint8_t *w = a.w;
    const ST *scales = reinterpret_cast<const ST *>(a.scales);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t row0 = blockIdx.x * kRows;
    const uint32_t rows = min((uint32_t)kRows, n - row0);

    // Let the next kernel's CTAs start (and stream their own weights) as soon
    // as there is room on the SMs; they wait for this grid before reading its output.
    pdl_launch_dependents();
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();

    // 1) weight stream (never depends on an earlier kernel): one bulk copy per row
    //    of nibbles and, when 16-byte granular, one per row of scales
    const uint32_t sbytes = nb * (uint32_t)sizeof(ST);
    const bool bulk_scales = (sbytes % 16 == 0) && aligned16(a.scales);
    if (warp == 0) {
        if (lane == 0) mbar_arrive_expect_tx(bar, rows * (nb * 16 + (bulk_scales ? sbytes : 0)));
        __syncwarp();
        const uint64_t pol = policy_evict_first();
        if (lane < (int)rows)
            bulk_g2s_hint(wt + lane * row_stride, w + (size_t)(row0 + lane) * (k / 2), nb * 16, bar, pol);
        else if (bulk_scales && lane >= 16 && lane - 16 < (int)rows)
            bulk_g2s_hint(ssm + (lane - 16) * nb, scales + (size_t)(row0 + lane - 16) * nb, sbytes, bar, pol);
    }
    if (!bulk_scales) {
        for (uint32_t i = tid; i < kRows * nb; i += kThreads) {
            const uint32_t r = i / nb, b = i % nb;
            ssm[i] = (r < rows) ? scales[(size_t)(row0 + r) * nb + b] : ST(0);
        }
    }
    // 2) activations written by the previous kernel are visible after this
    pdl_wait();

    Prologue<PRO, XT> pro;
    pro.init(a);
    float ss = 0.0f;
    if (PRO == PRO_NONE) {
        // No norm: each warp stages exactly the 128-k groups its MMAs read below, so
        // a warp barrier suffices and no warp waits for another's activation loads.
        const uint32_t ngr = (nb + 3) / 4, s0 = (ngr * warp) / kWarps, s1 = (ngr * (warp + 1)) / kWarps;
        constexpr int CH = 6;
        for (uint32_t c0 = s0; c0 < s1; c0 += CH) {
            float4 raw[CH];
#pragma unroll
            for (int u = 0; u < CH; ++u) {
                const uint32_t c = c0 + u, b = 4 * c + (lane >> 3);
                raw[u] = (c < s1 && b < nb) ? pro.raw4((size_t)c * 128 + lane * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < CH; ++u) {
                const uint32_t c = c0 + u, b = 4 * c + (lane >> 3);
                if (c < s1) split4(raw[u], c * 128 + lane * 4, b, lane, b < nb, xhi, xlo, xpost);  // warp-uniform
            }
        }
        __syncwarp();
    } else {
        // chunk = 128 consecutive elements = 4 blocks; lane owns 4 elements, 8 lanes a block
        const uint32_t nchunks = (nb + 3) / 4;
        constexpr int CH = 6;  // chunks in flight per warp (K <= 6144 in one batch)
        for (uint32_t c0 = warp; c0 < nchunks; c0 += CH * kWarps) {
            float4 raw[CH], wv[CH];
#pragma unroll
            for (int u = 0; u < CH; ++u) {
                const uint32_t c = c0 + u * kWarps, b = 4 * c + (lane >> 3);
                const size_t i = (size_t)c * 128 + lane * 4;
                const bool ok = c < nchunks && b < nb;
                raw[u] = ok ? pro.raw4(i) : make_float4(0.f, 0.f, 0.f, 0.f);
                wv[u] = ok ? pro.weight4(i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < CH; ++u) {
                const uint32_t c = c0 + u * kWarps, b = 4 * c + (lane >> 3);
                if (c < nchunks) {  // warp-uniform; lanes past nb only carry zeros
                    const uint32_t i = c * 128 + lane * 4;
                    const float4 r4 = raw[u];
                    if (PRO == PRO_EMBED_RMSNORM && blockIdx.x == 0 && b < nb)
                        *reinterpret_cast<float4 *>(a.x_out + i) = r4;
                    ss += r4.x * r4.x + r4.y * r4.y + r4.z * r4.z + r4.w * r4.w;
                    const float4 v = make_float4(r4.x * wv[u].x, r4.y * wv[u].y, r4.z * wv[u].z, r4.w * wv[u].w);
                    split4(v, i, b, lane, b < nb, xhi, xlo, xpost);
                }
            }
        }
    }
    float rms = 1.0f;  // RMSNorm's scalar is applied to the row results (W(x*w)*rms = W(x*rms*w))
    if (PRO != PRO_NONE) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int i = 0; i < kWarps; ++i) tot += red[i];
        rms = 1.0f / sqrtf(tot / (float)k + a.eps);
    }

    // 3) tensor-core tile dot products.  Groups of 4 blocks (128 k): the 8 mma
    //    columns carry (block j, hi) and (block j, lo) for j = 0..3, so one
    //    accumulator set covers the group and every lane holds useful sums:
    //    lane (g, t) ends with rows g, g+8 of block t, hi and lo.
    const uint32_t ng = (nb + 3) / 4;
    const uint32_t wg0 = (ng * warp) / kWarps, wg1 = (ng * (warp + 1)) / kWarps;
    const int g = lane >> 2, t = lane & 3, my_j = g >> 1;
    const __half *xmine = (g & 1) ? xlo : xhi;
    float acc0 = 0.0f, acc1 = 0.0f;  // rows g and g+8 over blocks = t (mod 4)
    if (mbar_wait_bounded(bar, 0)) {
        const int mj = lane >> 3, mi = lane & 7;
        const uint8_t *lrow = wt + (mi + 8 * (mj & 1)) * row_stride + (mj >> 1) * 16;
        for (uint32_t grp = wg0; grp < wg1; ++grp) {
            const uint32_t b = grp * 4;
            const uint32_t nv = min(4u, nb - b);  // valid blocks in this group (warp-uniform)
            uint32_t r[2][4];
            if (nv >= 2) {
                ldmatrix_x4(r[0], lrow + b * 16);
            } else {
                uint32_t q[2];
                ldmatrix_x2(q, lrow + b * 16);
                r[0][0] = q[0], r[0][1] = q[1];
            }
            if (nv == 4) {
                ldmatrix_x4(r[1], lrow + (b + 2) * 16);
            } else if (nv == 3) {
                uint32_t q[2];
                ldmatrix_x2(q, lrow + (b + 2) * 16);
                r[1][0] = q[0], r[1][1] = q[1];
            }
            uint4 xv = make_uint4(0, 0, 0, 0);
            if (my_j < (int)nv) xv = *reinterpret_cast<const uint4 *>(xmine + (b + my_j) * 32 + 8 * t);
            float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j < (int)nv) {
                    uint32_t ha[4], hb[4];
                    decode_word_f16(r[j >> 1][2 * (j & 1)], ha);      // row g
                    decode_word_f16(r[j >> 1][2 * (j & 1) + 1], hb);  // row g+8
                    const bool mine = (j == my_j);
                    const uint32_t a0[4] = {ha[0], hb[0], ha[1], hb[1]};
                    const uint32_t a1[4] = {ha[2], hb[2], ha[3], hb[3]};
                    mma_f16_16816(d, a0, mine ? xv.x : 0u, mine ? xv.y : 0u, d);
                    mma_f16_16816(d, a1, mine ? xv.z : 0u, mine ? xv.w : 0u, d);
                }
            }
            if (t < (int)nv) {
                const float xp = xpost[b + t];
                acc0 += load_scale(&ssm[g * nb + b + t]) * xp * (d[0] + d[1]);
                acc1 += load_scale(&ssm[(g + 8) * nb + b + t]) * xp * (d[2] + d[3]);
            }
        }
    }
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    float *part = red + 32;                 // [kWarps][16]
    float *yt = red + 32 + kWarps * kRows;  // final row values of this tile
    if (t == 0) {
        part[warp * kRows + g] = acc0;
        part[warp * kRows + g + 8] = acc1;
    }
    __syncthreads();
    float yv = 0.0f;  // row tid of the tile (tid < kRows)
    if (tid < kRows) {
        float s = part[tid];
#pragma unroll
        for (int i = 1; i < kWarps; ++i) s += part[i * kRows + tid];
        yv = s * rms;
        yt[tid] = yv;
    }
    if (EPI != EPI_STORE && EPI != EPI_RESIDUAL) __syncthreads();  // these two write only their own row

    // 4) epilogue
    if (EPI == EPI_STORE) {
        if (tid < (int)rows) a.y[row0 + tid] = yv;
    } else if (EPI == EPI_RESIDUAL) {
        if (tid < (int)rows) a.y[row0 + tid] = a.y[row0 + tid] + yv;  // llama_run:259
    } else if (EPI == EPI_SWIGLU) {
        // tile rows 0..7 = gate[8*tile ..], rows 8..15 = up[8*tile ..]
        if (tid < 8) {
            const float gv = yt[tid], uv = yt[tid + 8];
            a.y[blockIdx.x * 8 + tid] = gv / (1.0f + expf(-gv)) * uv;  // llama_run:248-250
        }
    } else if (EPI == EPI_QKV_ROPE) {
        const uint32_t pos = *a.pos;
        if (pos >= a.max_seq) return;  // never write past the cache (host also bounds positions)
        const uint32_t hd = a.head_dim, half = hd / 2, tiles_per_head = half / 8;
        const uint32_t tile = blockIdx.x;
        const uint32_t kvrow = a.n_kv * hd;  // elements per position of one layer's cache
        if (tile < a.q_tiles + a.k_tiles) {
            // rope-paired tile: rows 0..7 = j0..j0+7, rows 8..15 = j0+half..
            const bool is_q = tile < a.q_tiles;
            const uint32_t lt = is_q ? tile : tile - a.q_tiles;
            const uint32_t head = lt / tiles_per_head, j = (lt % tiles_per_head) * 8 + tid;
            if (tid < 8) {
                const float c = a.cos_t[(size_t)pos * half + j], s = a.sin_t[(size_t)pos * half + j];
                const float x0 = yt[tid], x1 = yt[tid + 8];
                const float o0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));  // llama_run:135-136
                const float o1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
                if (is_q) {
                    a.q_out[head * hd + j] = o0;
                    a.q_out[head * hd + j + half] = o1;
                } else {
                    uint16_t *dst = a.kc + (size_t)pos * kvrow + head * hd;
                    dst[j] = f32_to_bf16_bits(o0);
                    dst[j + half] = f32_to_bf16_bits(o1);
                }
            }
        } else if (tid < (int)rows) {
            const uint32_t vi = (tile - a.q_tiles - a.k_tiles) * kRows + tid;
            a.vc[(size_t)pos * kvrow + vi] = f32_to_bf16_bits(yt[tid]);
        }
    }
}

template <typename ST, typename XT, int PRO, int EPI>
int launch(cudaStream_t stream, const Args &a, bool pdl) {
    const Layout L = layout<ST>(a.k);
    auto kern = gemv_kernel<ST, XT, PRO, EPI>;
    if (L.total > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
        if (e != cudaSuccess) {
            set_error("fp4_gemv: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
            return FP4X_ECUDA;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.n + kRows - 1) / kRows);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) {
        set_error("fp4_gemv: launch: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    return FP4X_OK;
}

int validate(const Args &a, uint32_t kmax, bool needs_y = true) {
    FP4X_REQUIRE(a.w && a.scales && (a.y || !needs_y), "fp4_gemv: null pointer");
    FP4X_REQUIRE(a.n > 0, "fp4_gemv: n must be > 0");
    FP4X_REQUIRE(a.k >= 32 && a.k % 32 == 0 && a.k <= kmax, "fp4_gemv: k=%u must be a multiple of 32 in [32, %u]",
                 a.k, kmax);
    FP4X_REQUIRE(aligned16(a.w), "fp4_gemv: weights must be 16-byte aligned");
    return FP4X_OK;
}

// Engine entry: dispatch the fused variants on E8M0 scales and f32 activations.
int launch_fused(cudaStream_t stream, int pro, int epi, const Args &a, bool pdl) {
    int st = validate(a, kMaxK, epi != EPI_QKV_ROPE);
    if (st) return st;
    if (epi == EPI_QKV_ROPE)
        FP4X_REQUIRE(a.q_out && a.kc && a.vc && a.cos_t && a.sin_t && a.pos, "fp4_gemv (qkv): null pointer");
    if (pro == PRO_EMBED_RMSNORM) FP4X_REQUIRE(a.embed && a.tok && a.x_out, "fp4_gemv (embed): null pointer");
    if (pro != PRO_EMBED_RMSNORM) FP4X_REQUIRE(a.x, "fp4_gemv: null activation");
#define FP4X_CASE(P, E)                                                    \
    if (pro == P && epi == E) return launch<uint8_t, float, P, E>(stream, a, pdl);
    FP4X_CASE(PRO_NONE, EPI_STORE)
    FP4X_CASE(PRO_NONE, EPI_RESIDUAL)
    FP4X_CASE(PRO_RMSNORM, EPI_STORE)
    FP4X_CASE(PRO_RMSNORM, EPI_SWIGLU)
    FP4X_CASE(PRO_RMSNORM, EPI_QKV_ROPE)
    FP4X_CASE(PRO_EMBED_RMSNORM, EPI_QKV_ROPE)
#undef FP4X_CASE
    set_error("fp4_gemv: unsupported fused variant %d/%d", pro, epi);
    return FP4X_EUNSUPPORTED;
}

}  // namespace gemv
}  // namespace fp4x

using namespace fp4x;

extern "C" int fp4_gemv(fp4x_stream_t stream, uint32_t n, uint32_t k, const uint8_t *w, const uint8_t *scales,
                        const uint16_t *x, float *y) {
    gemv::Args a = {};
    a.n = n, a.k = k, a.w = w, a.scales = scales, a.x = x, a.y = y;
    int st = gemv::validate(a, gemv::kMaxK);
    if (!st) FP4X_REQUIRE(x, "fp4_gemv: null pointer");
    return st ? st : gemv::launch<uint8_t, uint16_t, gemv::PRO_NONE, gemv::EPI_STORE>((cudaStream_t)stream, a, true);
}

extern "C" int fp4_gemv_f32x(fp4x_stream_t stream, uint32_t n, uint32_t k, const uint8_t *w, const uint8_t *scales,
                             const float *x, float *y) {
    gemv::Args a = {};
    a.n = n, a.k = k, a.w = w, a.scales = scales, a.x = x, a.y = y;
    int st = gemv::validate(a, gemv::kMaxK);
    if (!st) FP4X_REQUIRE(x, "fp4_gemv: null pointer");
    return st ? st : gemv::launch<uint8_t, float, gemv::PRO_NONE, gemv::EPI_STORE>((cudaStream_t)stream, a, true);
}

extern "C" int fp4_gemv_ref(fp4x_stream_t stream, uint32_t n, uint32_t k, const uint32_t *w, const float *scales,
                            const float *x, float *y) {
    gemv::Args a = {};
    a.n = n, a.k = k, a.w = reinterpret_cast<const uint8_t *>(w), a.scales = scales, a.x = x, a.y = y;
    int st = gemv::validate(a, 8192);  // the reference's MAXK (llama_run:17)
    if (!st) FP4X_REQUIRE(x, "fp4_gemv: null pointer");
    return st ? st : gemv::launch<float, float, gemv::PRO_NONE, gemv::EPI_STORE>((cudaStream_t)stream, a, true);
}
