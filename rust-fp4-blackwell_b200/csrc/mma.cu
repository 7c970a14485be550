// mma.cu -- fp4_mma: block-scaled MXFP4 x MXFP4 GEMM on the sm_100a tensor cores.
//
//   D[t][r] = sum_k A[t][k] * W[r][k],  A: [m][k] tokens, W: [n][k] weight rows,
//   both packed E2M1 (k/2 bytes a row, low nibble = lower k) with one E8M0 scale
//   per 32 values ([rows][k/32] bytes); fp32 accumulation, bf16 or fp32 out.
//
// The reference has no GEMM on this path, only the single-warp all-ones
// known-answer test (examples/fp4_mma/src/main.rs:18-54: every D = 64.0) and
// the m16n8k64 operand/scale layout notes it pins (trackb/FP4_M16N8K64_LAYOUT.md).
// The CPU oracle's orc_mma_mxf4 restates the arithmetic.
//
// One CTA computes a 128-weight-row x NT-token tile (NT = 8..256) over a range
// of K stages (256 k each, split-K when the tile grid alone cannot fill the
// SMs).  Weights are the MMA's A operand (M = 128), tokens its B operand (N = NT):
//   warp 0     TMA producer: one 128-byte-swizzled box of each operand a stage;
//   warp 1     allocates tensor memory; lane 0 issues tcgen05.cp (scales) and
//              4 x tcgen05.mma.kind::mxf4 a stage, then tcgen05.commit;
//   warps 2-5  gather the stage's E8M0 scales into shared scale atoms, then run
//              the epilogue (tcgen05.ld -> bf16/fp32 stores or fp32 red.add).
#include "common.cuh"
#include "tc05.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

namespace fp4x {
namespace tc {

bool make_map_sw128(CUtensorMap *map, const void *base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!encode) return false;
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {128, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_out(CUtensorMap *map, void *base, uint32_t elem, uint64_t cols, uint64_t rows, uint64_t planes,
                  uint32_t box_cols, uint32_t box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!encode || (cols * elem) % 16 != 0 || (reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
    const cuuint64_t dims[3] = {cols, rows, planes};
    const cuuint64_t strides[2] = {cols * elem, cols * rows * elem};
    const cuuint32_t box[3] = {box_cols, box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return encode(map, elem == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                  planes > 1 ? 3 : 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc

namespace mma {

constexpr int kThreads = 192;

// Per-CTA timestamps (globaltimer, ns) only in builds compiled with
// -DFP4X_MMA_TIMING; a no-op otherwise.  Slot layout per CTA (linear block id
// < kMtCtas): 0 start, 1 setup done, 2 + i MMA lane saw stage i (i < 24),
// 26 last MMA commit, 27 epilogue start, 28 epilogue done, 29 SM id, 30 TMEM
// reads staged, 31 epilogue warps synchronised.
#ifdef FP4X_MMA_TIMING
constexpr uint32_t kMtCtas = 2048, kMtSlots = 32;
__device__ unsigned long long g_mma_ts[kMtCtas * kMtSlots];
__device__ __forceinline__ void mts(uint32_t i) {
    const uint32_t b = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    if (b < kMtCtas && i < kMtSlots) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g_mma_ts[b * kMtSlots + i] = t;
        if (i == 0) {
            uint32_t sm;
            asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
            g_mma_ts[b * kMtSlots + 29] = sm;
        }
    }
}
#else
__device__ __forceinline__ void mts(uint32_t) {}
#endif
constexpr uint32_t kStageK = 256;             // k per stage: one 128-byte swizzle row
constexpr uint32_t kTileA = 128 * 128;        // weight tile bytes per stage
constexpr uint32_t kMaxStages = 8;
constexpr uint32_t kSmemLimit = 227 * 1024;
constexpr uint32_t kBarBytes = 256;

// Final write of an output element: bf16 store, f32 store, or f32 add into the
// destination (a residual; one writer per element, so a plain load + store).
enum Mode : uint32_t { OUT_BF16 = 0, OUT_F32 = 1, OUT_ADD_F32 = 2 };

// ak = scale atoms per 256-k stage per 128 rows: 2 for MXFP4 (E8M0 per 32, an atom
// row holds 4 blocks = 128 k), 4 for NVFP4 (UE4M3 per 16, an atom row = 64 k).
struct Geo {
    uint32_t nt, ak, stages, sfb_atoms, stage_bytes, b_off, sfa_off, sfb_off, tmem_cols, sfa_col0, sfb_col0, smem;
    uint32_t per_sm;  // CTAs resident per SM (2 for tiles of <= 128 tokens: their MMA issue overlaps)
};

// Two CTAs share an SM when each needs at most half of its shared memory (228 KB,
// 1 KB reserved per CTA) and half of its 512 tensor-memory columns.
constexpr uint32_t kSmemHalf = 113 * 1024;

__host__ __device__ inline Geo geometry(uint32_t nt, bool nv = false) {
    Geo g;
    g.nt = nt;
    g.ak = nv ? 4 : 2;
    g.sfb_atoms = nt > 128 ? 2 : 1;
    g.b_off = kTileA;
    g.sfa_off = g.b_off + nt * 128;
    g.sfb_off = g.sfa_off + g.ak * 512;
    g.stage_bytes = (g.sfb_off + g.sfb_atoms * g.ak * 512 + 1023) / 1024 * 1024;
    for (g.per_sm = nt <= 128 ? 2u : 1u;; g.per_sm = 1) {
        const uint32_t lim = g.per_sm == 2 ? kSmemHalf : kSmemLimit;
        uint32_t s = (lim - 1024 - kBarBytes) / g.stage_bytes;
        g.stages = s > kMaxStages ? kMaxStages : s;
        g.sfa_col0 = nt;
        g.sfb_col0 = nt + g.stages * 4 * g.ak;
        const uint32_t cols = g.sfb_col0 + g.stages * 4 * g.ak * g.sfb_atoms;
        uint32_t c = 32;
        while (c < cols) c *= 2;
        g.tmem_cols = c;
        g.smem = g.stages * g.stage_bytes + 1024 + kBarBytes;
        if (g.per_sm == 1 || (g.stages >= 3 && g.tmem_cols <= 256)) break;
    }
    return g;
}

struct Args {
    uint32_t m, n, k, nt, kps;  // kps: K stages per split
    const uint8_t *sa, *sw;     // scales [m][k/32], [n][k/32]
    void *d;                    // [m / terms][n] bf16 or f32
    uint32_t mode;
    uint32_t terms;             // 1, 4 or 8: A rows T t .. T t + T - 1 are the MXFP4 terms of token t (summed)
    uint32_t splits;            // K splits (blockIdx.z); > 1: partial sums to ws, added by splitk_reduce_kernel
    float *ws;                  // [splits][m / terms][n] partial sums
    float alpha;                // output multiplier (NVFP4 per-tensor scales; 1 for MXFP4)
    // MXFP4 only: the scales already arranged as the kernel's 512-byte atoms
    // (scale_image_bytes layouts), loaded per stage by one bulk copy each instead of
    // gathered from sa / sw; both null = gather
    const uint8_t *sa_img, *sw_img;
    // 1: the epilogue writes its tile with one TMA store (or TMA reduce-add for
    // OUT_ADD_F32) through map_d; 0: coalesced thread stores
    uint32_t tma_out;
};

// Scale-atom image of a [rows][k/32] E8M0 matrix cut into tiles of `tile_rows`
// rows (128: weights; nt: tokens): [tile][stage of 256 k][tile_rows/128][2][512 B],
// atom h of a stage holding k-blocks 8 stage + 4h + j of row r at byte
// 16 (r % 32) + 4 (r / 32) + j (rows / blocks outside the matrix are 0).
__host__ __device__ inline size_t scale_image_bytes(uint32_t rows, uint32_t k, uint32_t tile_rows) {
    const uint32_t tiles = (rows + tile_rows - 1) / tile_rows, kst = (k + kStageK - 1) / kStageK;
    return (size_t)tiles * kst * ((tile_rows + 127) / 128) * 2 * 512;
}
__host__ __device__ inline size_t scale_image_offset(uint32_t row, uint32_t kb, uint32_t k, uint32_t tile_rows) {
    const uint32_t kst = (k + kStageK - 1) / kStageK, qn = (tile_rows + 127) / 128;
    const uint32_t tile = row / tile_rows, rr = row % tile_rows, q = rr / 128, r = rr % 128;
    const uint32_t stage = kb / 8, h = (kb % 8) / 4, j = kb % 4;
    return ((((size_t)tile * kst + stage) * qn + q) * 2 + h) * 512 + 16 * (r % 32) + 4 * (r / 32) + j;
}

__global__ void scale_image_kernel(const uint8_t *__restrict__ s, uint32_t rows, uint32_t k, uint32_t tile_rows,
                                   uint8_t *__restrict__ img) {
    const uint32_t kbt = k / 32, tiles = (rows + tile_rows - 1) / tile_rows;
    const size_t total = (size_t)tiles * tile_rows * kbt;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t row = (uint32_t)(i / kbt), kb = (uint32_t)(i % kbt);
        img[scale_image_offset(row, kb, k, tile_rows)] = row < rows ? s[(size_t)row * kbt + kb] : (uint8_t)0;
    }
}

__device__ __forceinline__ void emit(const Args &a, uint32_t tok, uint32_t row, float v) {
    const size_t o = (size_t)tok * a.n + row;
    if (a.mode == OUT_BF16)
        reinterpret_cast<uint16_t *>(a.d)[o] = f32_to_bf16_bits(v);
    else if (a.mode == OUT_F32)
        reinterpret_cast<float *>(a.d)[o] = v;
    else
        reinterpret_cast<float *>(a.d)[o] += v;
}

// Split-K: out[t][r] (final write of `mode`) = sum over splits, in split order.
__global__ void splitk_reduce_kernel(const float *__restrict__ ws, uint32_t splits, uint32_t tokens, uint32_t n,
                                     void *d, uint32_t mode) {
    pdl_launch_dependents();
    pdl_wait();
    const size_t total = (size_t)tokens * n, stride = (size_t)gridDim.x * blockDim.x;
    Args a{};
    a.n = n, a.d = d, a.mode = mode;
    if ((n & 3u) == 0) {
        const size_t q = total / 4;
        for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < q; i += stride) {
            float4 acc = __ldcg(reinterpret_cast<const float4 *>(ws) + i);
            for (uint32_t sp = 1; sp < splits; ++sp) {
                const float4 v = __ldcg(reinterpret_cast<const float4 *>(ws + sp * total) + i);
                acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
            }
            const uint32_t tk = (uint32_t)(4 * i / n), r = (uint32_t)(4 * i % n);
            emit(a, tk, r, acc.x), emit(a, tk, r + 1, acc.y), emit(a, tk, r + 2, acc.z), emit(a, tk, r + 3, acc.w);
        }
        return;
    }
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        float acc = __ldcg(ws + i);
        for (uint32_t sp = 1; sp < splits; ++sp) acc += __ldcg(ws + sp * total + i);
        emit(a, (uint32_t)(i / n), (uint32_t)(i % n), acc);
    }
}

__device__ __forceinline__ void sts_f32(uint32_t addr, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void sts_b16(uint32_t addr, uint16_t v) {
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}
__device__ __forceinline__ float4 lds_f32x4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr)
                 : "memory");
    return v;
}

// Accumulator -> outputs for the 128 epilogue threads (thread t: TMEM lane
// quarter q = warp % 4, tile row 32q + lane).  Column c of the tile is A row
// tok0 + c; T consecutive columns are the terms of one token and are added.
// The tile goes through shared memory (the stage buffers, idle once the last
// MMA has completed) as [token][128 rows] of the output type, and leaves with
// one TMA tile store (a TMA reduce-add for OUT_ADD_F32; the box is clipped at
// the tensor's edges), or -- when the output rows are not 16-byte granular --
// f32 staging and coalesced thread stores.  Writing straight from TMEM (one
// 2-byte store per element) took half of a CTA's lifetime at 256 tokens.  With
// split K the sums go to this split's partial slice.
template <uint32_t T>
__device__ void epilogue_tile(const Args &a, const CUtensorMap *map_d, uint32_t tbase, uint32_t q, uint32_t lane,
                              uint32_t t, uint32_t row0, uint32_t tok0, uint8_t *stg) {
    const uint32_t r = 32 * q + lane, ntok = a.nt / T, tokens = a.m / T, tk0 = tok0 / T;
    const bool bf = a.tma_out && a.splits == 1 && a.mode == OUT_BF16;  // bf16 staging image
    const uint32_t sbase = smem_u32(stg);
    for (uint32_t c0 = 0; c0 < a.nt; c0 += 32) {
        float v[4][8];
#pragma unroll
        for (uint32_t u = 0; u < 4; ++u)
            if (c0 + 8 * u < a.nt) tc::tmem_ld_x8(tbase + ((32 * q) << 16) + c0 + 8 * u, v[u]);
        tc::tmem_wait_ld();
#pragma unroll
        for (uint32_t u = 0; u < 4; ++u) {
            if (c0 + 8 * u >= a.nt) continue;
#pragma unroll
            for (uint32_t j = 0; j < 8; j += T) {
                float sum = v[u][j];
#pragma unroll
                for (uint32_t e = 1; e < T; ++e) sum += v[u][j + e];
                const uint32_t idx = ((c0 + 8 * u + j) / T) * 128 + r;
                if (bf)
                    sts_b16(sbase + 2 * idx, f32_to_bf16_bits(sum * a.alpha));
                else
                    sts_f32(sbase + 4 * idx, sum * a.alpha);
            }
        }
    }
    if (a.tma_out) {
        fence_proxy_async_smem();  // this thread's staging writes -> the TMA engine
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (t == 0) {
            if (a.splits > 1)
                tc::tma_store_3d(map_d, (int32_t)row0, (int32_t)tk0, (int32_t)blockIdx.z, stg);
            else if (a.mode == OUT_ADD_F32)
                tc::tma_reduce_add_2d(map_d, (int32_t)row0, (int32_t)tk0, stg);
            else
                tc::tma_store_2d(map_d, (int32_t)row0, (int32_t)tk0, stg);
            tc::bulk_commit();
            tc::bulk_wait_all();
        }
        return;
    }
    asm volatile("bar.sync 2, 128;" ::: "memory");
    const uint32_t rows = a.n - row0 < 128u ? a.n - row0 : 128u;
    const bool vec = (a.n & 3u) == 0 && rows == 128;
    for (uint32_t i = t; i < ntok * 32; i += 128) {
        const uint32_t tk = i / 32, c4 = i % 32, tok = tk0 + tk;
        if (tok >= tokens) continue;
        const float4 v = lds_f32x4(sbase + 16 * i);
        const uint32_t row = row0 + 4 * c4;
        const size_t o = (size_t)tok * a.n + row;
        if (vec && a.splits > 1) {
            *reinterpret_cast<float4 *>(a.ws + (size_t)blockIdx.z * tokens * a.n + o) = v;
        } else if (vec && a.mode == OUT_BF16) {
            const uint32_t lo = (uint32_t)f32_to_bf16_bits(v.x) | ((uint32_t)f32_to_bf16_bits(v.y) << 16);
            const uint32_t hi = (uint32_t)f32_to_bf16_bits(v.z) | ((uint32_t)f32_to_bf16_bits(v.w) << 16);
            *reinterpret_cast<uint2 *>(reinterpret_cast<uint16_t *>(a.d) + o) = make_uint2(lo, hi);
        } else if (vec && a.mode == OUT_F32) {
            *reinterpret_cast<float4 *>(reinterpret_cast<float *>(a.d) + o) = v;
        } else if (vec) {  // OUT_ADD_F32: one writer per element
            float4 *p = reinterpret_cast<float4 *>(reinterpret_cast<float *>(a.d) + o);
            float4 x = *p;
            x.x += v.x, x.y += v.y, x.z += v.z, x.w += v.w;
            *p = x;
        } else {
            const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (uint32_t k = 0; k < 4; ++k) {
                if (4 * c4 + k >= rows) break;
                if (a.splits > 1)
                    a.ws[(size_t)blockIdx.z * tokens * a.n + o + k] = e[k];
                else
                    emit(a, tok, row + k, e[k]);
            }
        }
    }
}

// Bounded wait that also gives up when another role of the CTA has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile uint32_t *abort) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
    }
    *abort = 1;
    raise_device_error(DEVERR_MBAR_TIMEOUT);
    return false;
}

// 8 scale bytes [kb0, kb0 + 8) of one row (0 outside the matrix).
__device__ __forceinline__ uint2 load_scales8(const uint8_t *s, uint32_t row, uint32_t rows, uint32_t kb0,
                                              uint32_t kbt) {
    if (row >= rows) return make_uint2(0, 0);
    const uint8_t *p = s + (size_t)row * kbt + kb0;
    if ((kbt & 7u) == 0 && kb0 + 8 <= kbt) return __ldg(reinterpret_cast<const uint2 *>(p));
    uint32_t w[2] = {0, 0};
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j)
        if (kb0 + j < kbt) w[j >> 2] |= (uint32_t)__ldg(p + j) << (8 * (j & 3));
    return make_uint2(w[0], w[1]);
}

// 16 scale bytes [kb0, kb0 + 16) of one row (0 outside the matrix).
__device__ __forceinline__ uint4 load_scales16(const uint8_t *s, uint32_t row, uint32_t rows, uint32_t kb0,
                                               uint32_t kbt) {
    if (row >= rows) return make_uint4(0, 0, 0, 0);
    const uint8_t *p = s + (size_t)row * kbt + kb0;
    if ((kbt & 15u) == 0 && kb0 + 16 <= kbt) return __ldg(reinterpret_cast<const uint4 *>(p));
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
    for (uint32_t j = 0; j < 16; ++j)
        if (kb0 + j < kbt) w[j >> 2] |= (uint32_t)__ldg(p + j) << (8 * (j & 3));
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// NV: NVFP4 operands (UE4M3 scales per 16, kind::mxf4nvf4); otherwise MXFP4.
template <bool NV>
__global__ void __launch_bounds__(kThreads, 1)
    mxf4_gemm_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_a,
                     const __grid_constant__ CUtensorMap map_d, Args a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const Geo G = geometry(a.nt, NV);
    const uint32_t S = G.stages;
    uint64_t *full_t = reinterpret_cast<uint64_t *>(smem + S * G.stage_bytes);  // TMA bytes landed
    uint64_t *full_s = full_t + kMaxStages;                                     // scale atoms written
    uint64_t *empty = full_s + kMaxStages;                                      // MMAs of the stage done
    uint64_t *accb = empty + kMaxStages;                                        // accumulator complete
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accb + 1);
    volatile uint32_t *abort = tmem_slot + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) mts(0);
    const uint32_t tok0 = blockIdx.x * a.nt, row0 = blockIdx.y * 128;
    const uint32_t kst = (a.k + kStageK - 1) / kStageK, kbt = a.k / (NV ? 16 : 32);
    const uint32_t s0 = blockIdx.z * a.kps, s1 = min(kst, s0 + a.kps);
    const uint32_t nst = s1 > s0 ? s1 - s0 : 0;
    const bool pre = !NV && a.sa_img != nullptr;  // scale atoms arrive by bulk copy with the tiles
    // CTAs walk their K stages in rotated order (start = weight tile index mod
    // stages) so that concurrent CTAs do not all read the same activation lines
    // of L2 at the same moment.
    const uint32_t rot = nst ? blockIdx.y % nst : 0;
    auto stage_of = [&](uint32_t i) { return s0 + (i + rot < nst ? i + rot : i + rot - nst); };

    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < S; ++i) {
            mbar_init(&full_t[i], 1);
            mbar_init(&full_s[i], 128);
            mbar_init(&empty[i], 1);
        }
        mbar_init(accb, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, G.tmem_cols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = *tmem_slot;
    // Launched with programmatic dependent launch: the setup above overlaps the
    // previous kernel's tail; nothing the previous kernel writes (operands, scales,
    // the output) is touched before it has completed.
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) mts(1);

    if (warp == 0) {
        if (lane == 0) {
            tc::tma_prefetch_desc(&map_w);
            tc::tma_prefetch_desc(&map_a);
            uint32_t issued = 0;
            for (uint32_t i = 0; i < nst; ++i) {
                const uint32_t slot = i % S;
                if (i >= S && !wait_or_abort(&empty[slot], ((i / S) - 1) & 1, abort)) break;
                uint8_t *st = smem + slot * G.stage_bytes;
                const uint32_t sw_bytes = G.ak * 512, sa_bytes = G.sfb_atoms * G.ak * 512;
                mbar_arrive_expect_tx(&full_t[slot], kTileA + a.nt * 128 + (pre ? sw_bytes + sa_bytes : 0u));
                const uint32_t sg = stage_of(i);
                const int32_t kx = (int32_t)(sg * 128);
                tc::tma_load_2d(st, &map_w, kx, (int32_t)row0, &full_t[slot]);
                tc::tma_load_2d(st + G.b_off, &map_a, kx, (int32_t)tok0, &full_t[slot]);
                if (pre) {
                    bulk_g2s(st + G.sfa_off, a.sw_img + ((size_t)blockIdx.y * kst + sg) * sw_bytes, sw_bytes, &full_t[slot]);
                    bulk_g2s(st + G.sfb_off, a.sa_img + ((size_t)blockIdx.x * kst + sg) * sa_bytes, sa_bytes, &full_t[slot]);
                }
                issued = i + 1;
            }
            // Never leave with copies in flight: wait for the last use of each slot.
            for (uint32_t i = issued > S ? issued - S : 0; i < issued; ++i)
                for (uint32_t it = 0; it < kSpinLimit && !mbar_try_wait(&full_t[i % S], (i / S) & 1); ++it) {
                }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = NV ? tc::idesc_nvf4(a.nt) : tc::idesc_mxf4(a.nt);
            for (uint32_t i = 0; i < nst; ++i) {
                const uint32_t slot = i % S, par = (i / S) & 1;
                if (!wait_or_abort(&full_t[slot], par, abort) || (!pre && !wait_or_abort(&full_s[slot], par, abort)))
                    break;
                mts(2 + i);
                tc::fence_after_sync();
                const uint8_t *st = smem + slot * G.stage_bytes;
                const uint32_t sa_col = tbase + G.sfa_col0 + slot * 4 * G.ak;
                const uint32_t sb_col = tbase + G.sfb_col0 + slot * 4 * G.ak * G.sfb_atoms;
                for (uint32_t at = 0; at < G.ak; ++at) {  // atom at covers k [at, at + 1) x 256 / ak of the stage
                    tc::utccp_scale_atom(sa_col + 4 * at, tc::desc_scale_atom(smem_u32(st + G.sfa_off + at * 512)));
                    for (uint32_t q = 0; q < G.sfb_atoms; ++q)
                        tc::utccp_scale_atom(sb_col + at * 4 * G.sfb_atoms + 4 * q,
                                             tc::desc_scale_atom(smem_u32(st + G.sfb_off + (q * G.ak + at) * 512)));
                }
                const uint32_t a_addr = smem_u32(st), b_addr = smem_u32(st + G.b_off);
#pragma unroll
                for (uint32_t kk = 0; kk < 4; ++kk) {
                    const uint64_t ad = tc::desc_sw128(a_addr + 32 * kk), bd = tc::desc_sw128(b_addr + 32 * kk);
                    if constexpr (NV) {  // one atom (4 UE4M3 bytes per row) per K=64
                        tc::mma_nvf4(tbase, ad, bd, idesc, sa_col + 4 * kk, sb_col + kk * 4 * G.sfb_atoms, (i | kk) != 0);
                    } else {  // one atom per K=128, scale ids 0/2 pick its byte pair
                        const uint32_t h = kk >> 1, sid = (kk & 1) * 2;
                        tc::mma_mxf4(tbase, ad, bd, idesc, (sa_col + 4 * h) | (sid << 30),
                                     (sb_col + h * 4 * G.sfb_atoms) | (sid << 30), (i | kk) != 0);
                    }
                }
                tc::commit(&empty[slot]);
            }
            mts(26);
            tc::commit(accb);  // also on abort: the epilogue then knows no MMA is in flight
        }
    } else {
        const uint32_t t = threadIdx.x - 64;  // 0..127
        // The scale bytes of stage i are loaded kScaleAhead stages early (a register
        // ring shifted every stage), so the global-load latency overlaps the MMAs
        // of the stages in between instead of adding to every stage.
        constexpr uint32_t kScaleAhead = 4;
        uint4 rw[kScaleAhead], rb0[kScaleAhead], rb1[kScaleAhead];
        auto load = [&](const uint8_t *sc, uint32_t row, uint32_t rows, uint32_t kb0) {
            if constexpr (NV) return load_scales16(sc, row, rows, kb0, kbt);
            const uint2 v = load_scales8(sc, row, rows, kb0, kbt);
            return make_uint4(v.x, v.y, 0u, 0u);
        };
        auto fetch = [&](uint32_t i, uint4 &w, uint4 &b0, uint4 &b1) {
            w = b0 = b1 = make_uint4(0, 0, 0, 0);
            if (i >= nst) return;
            const uint32_t kb0 = stage_of(i) * (NV ? 16 : 8);
            w = load(a.sw, row0 + t, a.n, kb0);
            if (t < a.nt) b0 = load(a.sa, tok0 + t, a.m, kb0);
            if (G.sfb_atoms > 1 && t + 128 < a.nt) b1 = load(a.sa, tok0 + t + 128, a.m, kb0);
        };
#pragma unroll
        for (uint32_t j = 0; j < kScaleAhead; ++j)
            if (!pre) fetch(j, rw[j], rb0[j], rb1[j]);
        for (uint32_t i = 0; i < (pre ? 0u : nst); ++i) {
            const uint32_t slot = i % S;
            if (i >= S && !wait_or_abort(&empty[slot], ((i / S) - 1) & 1, abort)) break;
            uint8_t *st = smem + slot * G.stage_bytes;
            const uint32_t off = tc::scale_atom_off(t, 0);
            const uint32_t wa[4] = {rw[0].x, rw[0].y, rw[0].z, rw[0].w};
            const uint32_t wb0[4] = {rb0[0].x, rb0[0].y, rb0[0].z, rb0[0].w};
            const uint32_t wb1[4] = {rb1[0].x, rb1[0].y, rb1[0].z, rb1[0].w};
#pragma unroll
            for (uint32_t at = 0; at < (NV ? 4u : 2u); ++at) {
                *reinterpret_cast<uint32_t *>(st + G.sfa_off + at * 512 + off) = wa[at];
                *reinterpret_cast<uint32_t *>(st + G.sfb_off + at * 512 + off) = wb0[at];
                if (G.sfb_atoms > 1) *reinterpret_cast<uint32_t *>(st + G.sfb_off + (G.ak + at) * 512 + off) = wb1[at];
            }
            fence_proxy_async_smem();
            mbar_arrive(&full_s[slot]);
#pragma unroll
            for (uint32_t j = 0; j + 1 < kScaleAhead; ++j) rw[j] = rw[j + 1], rb0[j] = rb0[j + 1], rb1[j] = rb1[j + 1];
            fetch(i + kScaleAhead, rw[kScaleAhead - 1], rb0[kScaleAhead - 1], rb1[kScaleAhead - 1]);
        }
        // epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31
        bool ok = wait_or_abort(accb, 0, abort);
        ok = __all_sync(0xffffffffu, ok);
        tc::fence_after_sync();
        // one decision for the 4 epilogue warps (the tile epilogue synchronises them)
        if (!ok && lane == 0) *abort = 1;
        asm volatile("bar.sync 2, 128;" ::: "memory");
        ok = *abort == 0;
        if (t == 0) mts(27);
        const uint32_t q = (uint32_t)warp & 3;
        uint8_t *stg = smem;  // stage buffers: every TMA copy and MMA has completed
        if (ok) {
            if (a.terms == 8) epilogue_tile<8>(a, &map_d, tbase, q, lane, t, row0, tok0, stg);
            else if (a.terms == 4) epilogue_tile<4>(a, &map_d, tbase, q, lane, t, row0, tok0, stg);
            else epilogue_tile<1>(a, &map_d, tbase, q, lane, t, row0, tok0, stg);
        }
        if (t == 0) mts(28);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, G.tmem_cols);
    }
}

// Known-answer kernel of the reference's fp4_mma_allones: A = B = 0x22 bytes
// (every E2M1 value 1.0), every scale 127 (2^0), K = 64 -> every D = 64.0.
// Operands are written straight into shared memory (no TMA), one MMA.
__global__ void __launch_bounds__(128, 1) allones_kernel(float *out) {
    __shared__ __align__(1024) uint8_t tile_a[128 * 128];
    __shared__ __align__(1024) uint8_t tile_b[8 * 128];
    __shared__ __align__(128) uint8_t atom_a[512], atom_b[512];
    __shared__ __align__(8) uint64_t done;
    __shared__ uint32_t tslot;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (uint32_t i = threadIdx.x; i < sizeof(tile_a) / 4; i += blockDim.x)
        reinterpret_cast<uint32_t *>(tile_a)[i] = 0x22222222u;
    for (uint32_t i = threadIdx.x; i < sizeof(tile_b) / 4; i += blockDim.x)
        reinterpret_cast<uint32_t *>(tile_b)[i] = 0x22222222u;
    reinterpret_cast<uint32_t *>(atom_a)[threadIdx.x] = 0x7F7F7F7Fu;
    reinterpret_cast<uint32_t *>(atom_b)[threadIdx.x] = 0x7F7F7F7Fu;
    if (threadIdx.x == 0) {
        mbar_init(&done, 1);
        fence_mbar_init();
    }
    fence_proxy_async_smem();
    if (warp == 0) {
        tc::tmem_alloc(&tslot, 32);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = tslot;
    if (threadIdx.x == 0) {
        tc::utccp_scale_atom(tbase + 8, tc::desc_scale_atom(smem_u32(atom_a)));
        tc::utccp_scale_atom(tbase + 12, tc::desc_scale_atom(smem_u32(atom_b)));
        tc::mma_mxf4(tbase, tc::desc_sw128(smem_u32(tile_a)), tc::desc_sw128(smem_u32(tile_b)), tc::idesc_mxf4(8),
                     tbase + 8, tbase + 12, 0);
        tc::commit(&done);
    }
    bool ok = true;
    for (uint32_t it = 0; !mbar_try_wait(&done, 0); ++it)
        if (it >= kSpinLimit) {
            ok = false;
            raise_device_error(DEVERR_MBAR_TIMEOUT);
            break;
        }
    ok = __all_sync(0xffffffffu, ok);
    tc::fence_after_sync();
    if (ok) {
        float v[8];
        tc::tmem_ld_x8(tbase + ((32 * warp) << 16), v);
        tc::tmem_wait_ld();
        const uint32_t r = 32 * warp + lane;
        if (r < 16)
#pragma unroll
            for (int j = 0; j < 8; ++j) out[r * 8 + j] = v[j];
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, 32);
    }
}

// Token rows per CTA tile for an m-row A operand.  128 (not 256): two CTAs share
// each SM, so one CTA's epilogue and K-stage waits overlap the other's MMA issue,
// and the grid's last partial wave is half as long (config 3 at M = 512: 824 ->
// 963 TFLOP/s aggregate).  Callers that pre-arrange activation scale images use the
// same tiling.
__host__ __device__ inline uint32_t token_tile(uint32_t m) { return m >= 128 ? 128u : (m + 7) / 8 * 8; }

struct Plan {
    uint32_t nt, m_tiles, n_tiles, kst, kps, splits;
    Geo g;
};

inline Plan plan(uint32_t m, uint32_t n, uint32_t k, bool allow_split = true, bool nv = false) {
    Plan p;
    p.nt = token_tile(m);
    p.m_tiles = (m + p.nt - 1) / p.nt;
    p.n_tiles = (n + 127) / 128;
    p.kst = (k + kStageK - 1) / kStageK;
    p.g = geometry(p.nt, nv);
    const uint32_t tiles = p.m_tiles * p.n_tiles, sms = (uint32_t)num_sms() * p.g.per_sm;
    // Time ~ waves x (stages per CTA + ~2 stages of pipeline fill and epilogue),
    // a wave being every CTA slot of the GPU.  Take the fewest splits that reach
    // the minimum (each split adds an fp32 partial per output).
    uint32_t splits = 1, best = ~0u;
    for (uint32_t s = 1; s <= (allow_split ? std::min(p.kst, 16u) : 1u); ++s) {
        const uint32_t waves = (tiles * s + sms - 1) / sms, per = (p.kst + s - 1) / s;
        const uint32_t cost = waves * (per + 2) + (s > 1 ? 2 : 0);
        if (cost < best) best = cost, splits = s;
    }
    p.kps = (p.kst + splits - 1) / splits;
    p.splits = (p.kst + p.kps - 1) / p.kps;
    return p;
}

int validate(uint32_t m, uint32_t n, uint32_t k, const void *a, const void *sa, const void *w, const void *sw,
             const void *d) {
    FP4X_REQUIRE(m > 0 && n > 0 && k > 0, "fp4_mma: empty shape m=%u n=%u k=%u", m, n, k);
    FP4X_REQUIRE(k % 64 == 0, "fp4_mma: k=%u must be a multiple of 64", k);
    FP4X_REQUIRE(a && sa && w && sw && d, "fp4_mma: null pointer");
    FP4X_REQUIRE(aligned16(a) && aligned16(w), "fp4_mma: packed operands must be 16-byte aligned");
    FP4X_REQUIRE(m <= (1u << 24) && n <= (1u << 24) && k <= (1u << 20), "fp4_mma: shape too large");
    return FP4X_OK;
}

// Split-K scratch: partials [splits][m / terms][n] f32.
inline size_t partials_bytes(const Plan &p, uint32_t m, uint32_t n, uint32_t terms) {
    return p.splits > 1 ? (size_t)p.splits * (m / terms) * n * sizeof(float) : 0;
}

// partials: split-K scratch of partials_bytes() (unused when p.splits == 1).
int launch(cudaStream_t s, uint32_t m, uint32_t n, uint32_t k, const uint8_t *a, const uint8_t *sa,
           const uint8_t *w, const uint8_t *sw, void *d, Mode mode, const Plan &p, uint32_t terms, float *partials,
           bool nv = false, float alpha = 1.0f, const uint8_t *sa_img = nullptr, const uint8_t *sw_img = nullptr) {
    CUtensorMap map_w, map_a;
    if (!tc::make_map_sw128(&map_w, w, k / 2, n, 128) || !tc::make_map_sw128(&map_a, a, k / 2, m, p.nt)) {
        set_error("fp4_mma: cuTensorMapEncodeTiled failed (m=%u n=%u k=%u)", m, n, k);
        return FP4X_ECUDA;
    }
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [] {
        attr_err = cudaFuncSetAttribute(mxf4_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kSmemLimit);
        if (attr_err == cudaSuccess)
            attr_err = cudaFuncSetAttribute(mxf4_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)kSmemLimit);
    });
    if (attr_err != cudaSuccess) {
        set_error("fp4_mma: cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
        return FP4X_ECUDA;
    }
    if (p.splits > 1 && !partials) {
        set_error("fp4_mma: split-K launch without a workspace");
        return FP4X_EINVAL;
    }
    if ((size_t)p.g.stages * p.g.stage_bytes < (size_t)p.nt * 128 * sizeof(float)) {  // epilogue staging tile
        set_error("fp4_mma: %u-token tile does not fit the epilogue staging area", p.nt);
        return FP4X_EUNSUPPORTED;
    }
    Args args{m, n, k, p.nt, p.kps, sa, sw, d, (uint32_t)mode, terms, p.splits, partials, alpha, sa_img, sw_img, 0};
    // output tile stores by TMA where the rows are 16-byte granular (the map encoder
    // checks the base alignment); otherwise coalesced thread stores
    CUtensorMap map_d;
    memset(&map_d, 0, sizeof(map_d));
    {
        const uint32_t tokens = m / terms, box_rows = p.nt / terms;
        bool ok;
        if (p.splits > 1)
            ok = tc::make_map_out(&map_d, partials, 4, n, tokens, p.splits, 128, box_rows);
        else
            ok = tc::make_map_out(&map_d, d, mode == OUT_BF16 ? 2 : 4, n, tokens, 1, 128, box_rows);
        args.tma_out = ok ? 1u : 0u;
    }
    // Both kernels wait (griddepcontrol.wait) before touching memory, so they are
    // launched with programmatic dependent launch: their launch and setup overlap
    // the previous kernel on the stream.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.m_tiles, p.n_tiles, p.splits);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.g.smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = nv ? cudaLaunchKernelEx(&cfg, mxf4_gemm_kernel<true>, map_w, map_a, map_d, args)
                       : cudaLaunchKernelEx(&cfg, mxf4_gemm_kernel<false>, map_w, map_a, map_d, args);
    if (e == cudaSuccess && p.splits > 1) {
        const size_t total = (size_t)(m / terms) * n;
        cfg.gridDim = dim3((uint32_t)std::min<size_t>((total / 4 + 255) / 256 + 1, 8u * (uint32_t)num_sms()));
        cfg.blockDim = dim3(256);
        cfg.dynamicSmemBytes = 0;
        e = cudaLaunchKernelEx(&cfg, splitk_reduce_kernel, (const float *)partials, p.splits, m / terms, n, d,
                               (uint32_t)mode);
    }
    if (e != cudaSuccess) {
        set_error("fp4_mma: launch: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    return check_launch("fp4_mma");
}

}  // namespace mma
}  // namespace fp4x

using namespace fp4x;

extern "C" size_t fp4_mma_workspace_size(uint32_t m, uint32_t n, uint32_t k) {
    if (m == 0 || n == 0 || k == 0) return 0;
    return mma::partials_bytes(mma::plan(m, n, k), m, n, 1);
}

extern "C" int fp4_mma(fp4x_stream_t stream, uint32_t m, uint32_t n, uint32_t k, const uint8_t *a,
                       const uint8_t *a_scales, const uint8_t *w, const uint8_t *w_scales, uint16_t *d_bf16,
                       void *workspace, size_t workspace_bytes) {
    if (int e = mma::validate(m, n, k, a, a_scales, w, w_scales, d_bf16)) return e;
    const mma::Plan p = mma::plan(m, n, k);
    cudaStream_t s = (cudaStream_t)stream;
    const size_t need = mma::partials_bytes(p, m, n, 1);
    if (p.splits > 1)
        FP4X_REQUIRE(workspace && workspace_bytes >= need && aligned16(workspace),
                     "fp4_mma: split-K needs a 16-byte aligned workspace of %zu bytes (fp4_mma_workspace_size)", need);
    return mma::launch(s, m, n, k, a, a_scales, w, w_scales, d_bf16, mma::OUT_BF16, p, 1,
                       static_cast<float *>(workspace));
}

// fp32 output without a workspace: one CTA per output tile over the whole K.
extern "C" int fp4_mma_f32(fp4x_stream_t stream, uint32_t m, uint32_t n, uint32_t k, const uint8_t *a,
                           const uint8_t *a_scales, const uint8_t *w, const uint8_t *w_scales, float *d) {
    if (int e = mma::validate(m, n, k, a, a_scales, w, w_scales, d)) return e;
    const mma::Plan p = mma::plan(m, n, k, false);
    return mma::launch((cudaStream_t)stream, m, n, k, a, a_scales, w, w_scales, d, mma::OUT_F32, p, 1, nullptr);
}

extern "C" size_t fp4_mma_nvf4_workspace_size(uint32_t m, uint32_t n, uint32_t k) {
    if (m == 0 || n == 0 || k == 0) return 0;
    return mma::partials_bytes(mma::plan(m, n, k, true, true), m, n, 1);
}

extern "C" int fp4_mma_nvf4(fp4x_stream_t stream, uint32_t m, uint32_t n, uint32_t k, const uint8_t *a,
                            const uint8_t *a_scales, const uint8_t *w, const uint8_t *w_scales, float alpha,
                            uint16_t *d_bf16, void *workspace, size_t workspace_bytes) {
    if (int e = mma::validate(m, n, k, a, a_scales, w, w_scales, d_bf16)) return e;
    const mma::Plan p = mma::plan(m, n, k, true, true);
    const size_t need = mma::partials_bytes(p, m, n, 1);
    if (p.splits > 1)
        FP4X_REQUIRE(workspace && workspace_bytes >= need && aligned16(workspace),
                     "fp4_mma_nvf4: split-K needs a 16-byte aligned workspace of %zu bytes", need);
    return mma::launch((cudaStream_t)stream, m, n, k, a, a_scales, w, w_scales, d_bf16, mma::OUT_BF16, p, 1,
                       static_cast<float *>(workspace), true, alpha);
}

extern "C" int fp4_mma_nvf4_f32(fp4x_stream_t stream, uint32_t m, uint32_t n, uint32_t k, const uint8_t *a,
                                const uint8_t *a_scales, const uint8_t *w, const uint8_t *w_scales, float alpha,
                                float *d) {
    if (int e = mma::validate(m, n, k, a, a_scales, w, w_scales, d)) return e;
    const mma::Plan p = mma::plan(m, n, k, false, true);
    return mma::launch((cudaStream_t)stream, m, n, k, a, a_scales, w, w_scales, d, mma::OUT_F32, p, 1, nullptr, true,
                       alpha);
}

#ifdef FP4X_MMA_TIMING
extern "C" FP4X_API int fp4x_mma_timestamps(unsigned long long *out, uint32_t n) {
    if (n == 0) {  // reset
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, mma::g_mma_ts) != cudaSuccess) return 2;
        return cudaMemset(p, 0, sizeof(mma::g_mma_ts)) == cudaSuccess ? 0 : 2;
    }
    n = std::min<uint32_t>(n, mma::kMtCtas * mma::kMtSlots);
    return cudaMemcpyFromSymbol(out, mma::g_mma_ts, n * sizeof(unsigned long long)) == cudaSuccess ? 0 : 2;
}
#endif

extern "C" int fp4_mma_allones(fp4x_stream_t stream, float *out) {
    FP4X_REQUIRE(out, "fp4_mma_allones: null pointer");
    mma::allones_kernel<<<1, 128, 0, (cudaStream_t)stream>>>(out);
    return check_launch("fp4_mma_allones");
}
