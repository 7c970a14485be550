// attention.cu -- split-KV GQA flash-decode (the llama_attn_decode operator).
//
// Replaces attn_decode, examples/llama_run/src/main.rs:148-242.  The reference
// runs one CTA per q head, keeps all scores of the sequence in shared memory
// (MAXSEQ cap) and accumulates P.V with 64 of 128 threads serially over t.
// Here:
//   * a CTA owns (batch b, a group of q heads sharing one KV head, a slice of
//     the sequence); each K/V row is read from HBM once per CTA for every q
//     head of the group (GQA reuse);
//   * each warp runs an online softmax over 32-token tiles (lane = token for
//     Q.K, lane = head-dim pair for P.V);
//   * with more than one slice, each CTA writes (m, l, o[hd]) partials to a
//     caller-provided workspace and a combine kernel merges them in slice
//     order (deterministic);
//   * head_dim 64 and 128 are template instances; no sequence cap.
// Bound: HBM.  Algorithmic bytes per call = 2 * B * seq * n_kv * hd * sizeof(kv)
//   (+ q and out); flops = 4 * B * n_heads * seq * hd.
#include "common.cuh"
#include "attention.cuh"

#include <algorithm>
#include <mutex>

namespace fp4x {
namespace attn {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 32;

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(uint16_t v) { return bf16_bits_to_f32(v); }
__device__ __forceinline__ void store_out(float *p, float v) { *p = v; }
__device__ __forceinline__ void store_out(uint16_t *p, float v) { *p = f32_to_bf16_bits(v); }

// Load head-dim elements 2*lane, 2*lane+1 (+64 for hd 128) of one row as f32.
template <int HD>
__device__ __forceinline__ void load_row_pairs(const float *row, int lane, float (&v)[HD / 32]) {
#pragma unroll
    for (int c = 0; c < HD / 64; ++c) {
        const float2 f = *reinterpret_cast<const float2 *>(row + 64 * c + 2 * lane);
        v[2 * c] = f.x, v[2 * c + 1] = f.y;
    }
}
template <int HD>
__device__ __forceinline__ void load_row_pairs(const uint16_t *row, int lane, float (&v)[HD / 32]) {
#pragma unroll
    for (int c = 0; c < HD / 64; ++c) {
        const uint32_t u = *reinterpret_cast<const uint32_t *>(row + 64 * c + 2 * lane);
        v[2 * c] = __uint_as_float(u << 16), v[2 * c + 1] = __uint_as_float(u & 0xFFFF0000u);
    }
}

// Eight consecutive elements of a row as f32 (one 16- or 32-byte vector load).
__device__ __forceinline__ void load_chunk8(const float *p, float (&k)[8]) {
    const float4 a = reinterpret_cast<const float4 *>(p)[0], b = reinterpret_cast<const float4 *>(p)[1];
    k[0] = a.x, k[1] = a.y, k[2] = a.z, k[3] = a.w, k[4] = b.x, k[5] = b.y, k[6] = b.z, k[7] = b.w;
}
__device__ __forceinline__ void load_chunk8(const uint16_t *p, float (&k)[8]) {
    const uint4 u = *reinterpret_cast<const uint4 *>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        k[2 * j] = __uint_as_float(w[j] << 16);
        k[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
}



// grid = (splits, n_heads / HPC, batch); HPC q heads (one KV head) per CTA.
template <int HD, int HPC, typename QT, typename KT, typename OT>
__global__ void __launch_bounds__(kThreads) attn_split_kernel(Params p) {
    constexpr int NV = HD / 32;  // head-dim values per lane in the P.V phase
    __shared__ __align__(16) float qs[HPC][HD];
    __shared__ float ps[kWarps][HPC][kTile];
    __shared__ float wm[kWarps][HPC], wl[kWarps][HPC];
    __shared__ float wo[kWarps][HPC][HD];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t split = blockIdx.x, hgrp = blockIdx.y, b = blockIdx.z;
    constexpr uint32_t H = HPC;
    const uint32_t h0 = hgrp * H;
    const uint32_t group = p.n_heads / p.n_kv, kvh = h0 / group;
    const uint32_t seq = seq_of(p, b);
    const uint32_t t_begin = split * p.split_len, t_end = min(seq, t_begin + p.split_len);
    if (t_begin >= seq) return;  // slice past the current position (whole CTA, before any barrier)

    const QT *q = reinterpret_cast<const QT *>(p.q) + ((size_t)b * p.n_heads + h0) * HD;
    for (uint32_t i = tid; i < H * HD; i += kThreads) qs[i / HD][i % HD] = to_f32(q[i]) * p.scale;
    __syncthreads();

    const size_t row_stride = (size_t)p.n_kv * HD;
    const KT *kbase = reinterpret_cast<const KT *>(p.kc) + cache_of(p, b) * p.max_seq * row_stride + (size_t)kvh * HD;
    const KT *vbase = reinterpret_cast<const KT *>(p.vc) + cache_of(p, b) * p.max_seq * row_stride + (size_t)kvh * HD;

    float m[HPC], l[HPC], o[HPC][NV];
#pragma unroll
    for (int h = 0; h < HPC; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; ++i) o[h][i] = 0.0f;
    }

    for (uint32_t t0 = t_begin + warp * kTile; t0 < t_end; t0 += kWarps * kTile) {
        const uint32_t t = t0 + lane;
        const bool live = t < t_end;
        float s[HPC];
#pragma unroll
        for (int h = 0; h < HPC; ++h) s[h] = 0.0f;
        if (live) {
            const KT *krow = kbase + (size_t)t * row_stride;
#pragma unroll
            for (int c = 0; c < HD / 8; ++c) {
                float kv[8];
                load_chunk8(krow + 8 * c, kv);
#pragma unroll
                for (int h = 0; h < HPC; ++h) {
                    const float4 qa = *reinterpret_cast<const float4 *>(&qs[h][8 * c]);
                    const float4 qb = *reinterpret_cast<const float4 *>(&qs[h][8 * c + 4]);
                    s[h] += qa.x * kv[0] + qa.y * kv[1] + qa.z * kv[2] + qa.w * kv[3] + qb.x * kv[4] +
                            qb.y * kv[5] + qb.z * kv[6] + qb.w * kv[7];
                }
            }
        }
#pragma unroll
        for (int h = 0; h < HPC; ++h) {
            const float sh = live ? s[h] : -INFINITY;
            const float mt = warp_max(sh);
            const float mn = fmaxf(m[h], mt);
            const float alpha = __expf(m[h] - mn);  // m = -inf on the first tile -> 0
            const float pr = live ? __expf(sh - mn) : 0.0f;
            l[h] = l[h] * alpha + warp_sum(pr);
            ps[warp][h][lane] = pr;
#pragma unroll
            for (int i = 0; i < NV; ++i) o[h][i] *= alpha;
            m[h] = mn;
        }
        __syncwarp();
        const uint32_t nt = min((uint32_t)kTile, t_end - t0);
        for (uint32_t j = 0; j < nt; ++j) {
            float v[NV];
            load_row_pairs<HD>(vbase + (size_t)(t0 + j) * row_stride, lane, v);
#pragma unroll
            for (int h = 0; h < HPC; ++h) {
                const float pr = ps[warp][h][j];
#pragma unroll
                for (int i = 0; i < NV; ++i) o[h][i] += pr * v[i];
            }
        }
        __syncwarp();
    }

    // merge the warps' states (fixed order)
#pragma unroll
    for (int h = 0; h < HPC; ++h) {
        if (lane == 0) {
            wm[warp][h] = m[h];
            wl[warp][h] = l[h];
        }
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
            wo[warp][h][64 * c + 2 * lane] = o[h][2 * c];
            wo[warp][h][64 * c + 2 * lane + 1] = o[h][2 * c + 1];
        }
    }
    __syncthreads();
    for (uint32_t i = tid; i < H * HD; i += kThreads) {
        const uint32_t h = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wm[w][h]);
        float L = 0.0f, O = 0.0f;
        for (int w = 0; w < kWarps; ++w) {
            const float f = (wm[w][h] == -INFINITY) ? 0.0f : __expf(wm[w][h] - M);
            L += wl[w][h] * f;
            O += wo[w][h][d] * f;
        }
        const size_t bh = (size_t)b * p.n_heads + h0 + h;
        if (p.splits == 1) {
            store_out(reinterpret_cast<OT *>(p.out) + bh * HD + d, O / L);
        } else {
            float *rec = p.ws + (bh * p.splits + split) * (HD + 2);
            rec[2 + d] = O;
            if (d == 0) {
                rec[0] = M;
                rec[1] = L;
            }
        }
    }
}

// ---------------------------------------------------------------- tensor-core flash-decode (bf16 caches)
// A CTA owns (batch b, the HPC q heads of one KV head, one slice of the sequence)
// like attn_split_kernel, but stages K/V in 64-token tiles with cp.async (16-byte
// pieces, 128-byte XOR swizzle, a multi-stage ring) and contracts on the tensor
// cores with mma.sync.m16n8k16 bf16 (f32 accumulate).  Warp w of a tile owns
// tokens 16w..16w+15:
//   S^T[token][head] = K[token][:] . q[head][:]  (A = K via ldmatrix, B = q, the
//     8 mma columns are the (up to 8) heads; q is split into bf16 hi + lo, so an
//     f32 q keeps ~16 bits and a bf16 q is exact);
//   online softmax per head over the warp's tokens (f32);
//   O^T[dim][head] += V^T[dim][token] . P^T[token][head]  (A = V^T via
//     ldmatrix.trans, B = P written as bf16 hi + lo through shared memory).
// The 4 warps' states are merged in warp order; slices write (m, l, o) partials
// for attn_combine_kernel exactly like attn_split_kernel.
__device__ __forceinline__ void cp_async16(void *dst_smem, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst_smem)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void *smem_row_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(smem_row_addr)));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
}

template <int HD>
struct MmaCfg {
    static constexpr int kTile = 64;
    // Two K/V stages at both head dims: at 64 dims the smaller ring fits about twice
    // the CTAs per SM, which the slice model turns into more, shorter slices (B200,
    // config 2: batch 1 / 8 at 32k 14.2 -> 13.1 / 55.7 -> 52.6 us, batch 64 at 2k / 8k
    // 34.5 -> 29.6 / 97.0 -> 91.7 us; batch 64 at 512 positions 11.3 -> 13.1 us)
    static constexpr int kStages = 2;
    static constexpr int kChunks = HD / 8;  // 16-byte pieces per row
    static constexpr size_t kStageElems = (size_t)kTile * HD;
    static constexpr size_t kSmem = (size_t)kStages * 2 * kStageElems * 2  // K and V ring
                                    + (size_t)4 * 2 * 8 * 16 * 2            // P^T hi/lo per warp
                                    + (size_t)4 * 8 * (HD + 2) * 4;         // warp merge
};

// 16-byte piece c of tile row r, swizzled within groups of 8 pieces.
template <int HD>
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) {
    return r * HD + (((c & ~7u) | ((c ^ r) & 7u)) * 8u);
}

template <int HD, int HPC, typename QT, typename OT>
__global__ void __launch_bounds__(kThreads) attn_mma_kernel(Params p) {
    using C = MmaCfg<HD>;
    constexpr int NT = HD / 16;
    extern __shared__ __align__(128) uint8_t sm_raw[];
    uint16_t *ks = reinterpret_cast<uint16_t *>(sm_raw);
    uint16_t *vs = ks + C::kStages * C::kStageElems;
    uint16_t *ps = vs + C::kStages * C::kStageElems;          // [warp][hi|lo][head 8][token 16]
    float *mrg = reinterpret_cast<float *>(ps + 4 * 2 * 8 * 16);  // [warp][head 8][HD + 2]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t split = blockIdx.x, hgrp = blockIdx.y, b = blockIdx.z;
    const uint32_t h0 = hgrp * HPC;
    const uint32_t group = p.n_heads / p.n_kv, kvh = h0 / group;
    const uint32_t seq = seq_of(p, b);
    const uint32_t t_begin = split * p.split_len, t_end = min(seq, t_begin + p.split_len);
    if (t_begin >= seq) return;
    const size_t row_stride = (size_t)p.n_kv * HD;
    const uint16_t *kbase = reinterpret_cast<const uint16_t *>(p.kc) + cache_of(p, b) * p.max_seq * row_stride + (size_t)kvh * HD;
    const uint16_t *vbase = reinterpret_cast<const uint16_t *>(p.vc) + cache_of(p, b) * p.max_seq * row_stride + (size_t)kvh * HD;

    // q fragments (B operand, column n = head g): dims 16kk + 2t (+1), +8
    uint32_t qh[NT][2], ql[NT][2];
    {
        const QT *q = reinterpret_cast<const QT *>(p.q) + ((size_t)b * p.n_heads + h0) * HD;
#pragma unroll
        for (int kk = 0; kk < NT; ++kk)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                float q0 = 0.0f, q1 = 0.0f;
                if (g < HPC) {
                    q0 = to_f32(q[g * HD + 16 * kk + 8 * r + 2 * t]);
                    q1 = to_f32(q[g * HD + 16 * kk + 8 * r + 2 * t + 1]);
                }
                const float h0f = bf16_bits_to_f32(f32_to_bf16_bits(q0)), h1f = bf16_bits_to_f32(f32_to_bf16_bits(q1));
                qh[kk][r] = pack_bf16x2(q0, q1);
                ql[kk][r] = pack_bf16x2(q0 - h0f, q1 - h1f);
            }
    }
    const uint32_t ntiles = (t_end - t_begin + C::kTile - 1) / C::kTile;
    auto load_tile = [&](uint32_t i) {
        const uint32_t st = i % C::kStages, t0 = t_begin + i * C::kTile;
        uint16_t *kd = ks + st * C::kStageElems, *vd = vs + st * C::kStageElems;
        for (uint32_t idx = tid; idx < (uint32_t)C::kTile * C::kChunks; idx += kThreads) {
            const uint32_t r = idx / C::kChunks, c = idx % C::kChunks, tok = t0 + r;
            const bool valid = tok < t_end;
            const size_t src = (size_t)(valid ? tok : t_begin) * row_stride + 8 * c;
            cp_async16(kd + swz<HD>(r, c), kbase + src, valid);
            cp_async16(vd + swz<HD>(r, c), vbase + src, valid);
        }
    };
#pragma unroll
    for (int i = 0; i < C::kStages - 1; ++i) {
        if ((uint32_t)i < ntiles) load_tile(i);
        cp_async_commit();
    }
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // heads 2t, 2t+1
    float o[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
    uint16_t *pw = ps + warp * (2 * 8 * 16);
    for (uint32_t i = 0; i < ntiles; ++i) {
        if (i + C::kStages - 1 < ntiles) load_tile(i + C::kStages - 1);
        cp_async_commit();
        cp_async_wait<C::kStages - 1>();
        __syncthreads();
        const uint32_t st = i % C::kStages, t0 = t_begin + i * C::kTile;
        const uint16_t *kt = ks + st * C::kStageElems, *vt = vs + st * C::kStageElems;
        // S^T for tokens 16w..16w+15
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t arow = 16 * warp + (lane & 15);
#pragma unroll
        for (int kk = 0; kk < NT; ++kk) {
            uint32_t a[4];
            ldmatrix_x4(a, kt + swz<HD>(arow, 2 * kk + (lane >> 4)));
            mma_bf16_16816(s, a, qh[kk][0], qh[kk][1], s);
            mma_bf16_16816(s, a, ql[kk][0], ql[kk][1], s);
        }
        const uint32_t tokA = t0 + 16 * warp + g, tokB = tokA + 8;
        const float sa0 = tokA < t_end ? s[0] * p.scale : -INFINITY, sa1 = tokA < t_end ? s[1] * p.scale : -INFINITY;
        const float sb0 = tokB < t_end ? s[2] * p.scale : -INFINITY, sb1 = tokB < t_end ? s[3] * p.scale : -INFINITY;
        float mx0 = fmaxf(sa0, sb0), mx1 = fmaxf(sa1, sb1);
#pragma unroll
        for (int o2 = 4; o2 < 32; o2 <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o2));
        }
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        // a warp whose tokens are all masked keeps -inf: guard the exponent base
        const float base0 = mn0 == -INFINITY ? 0.0f : mn0, base1 = mn1 == -INFINITY ? 0.0f : mn1;
        const float al0 = __expf(m0 - base0), al1 = __expf(m1 - base1);
        const float pa0 = __expf(sa0 - base0), pa1 = __expf(sa1 - base1);
        const float pb0 = __expf(sb0 - base0), pb1 = __expf(sb1 - base1);
        float sum0 = pa0 + pb0, sum1 = pa1 + pb1;
#pragma unroll
        for (int o2 = 4; o2 < 32; o2 <<= 1) {
            sum0 += __shfl_xor_sync(0xffffffffu, sum0, o2);
            sum1 += __shfl_xor_sync(0xffffffffu, sum1, o2);
        }
        l0 = l0 * al0 + sum0, l1 = l1 * al1 + sum1;
        m0 = mn0, m1 = mn1;
#pragma unroll
        for (int dm = 0; dm < NT; ++dm) o[dm][0] *= al0, o[dm][1] *= al1, o[dm][2] *= al0, o[dm][3] *= al1;
        // P^T -> shared as [head][token] bf16 hi and lo
        {
            const float pv[4] = {pa0, pa1, pb0, pb1};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t head = 2 * t + (j & 1), tok = g + 8 * (j >> 1);
                const uint16_t hi = f32_to_bf16_bits(pv[j]);
                pw[head * 16 + tok] = hi;
                pw[128 + head * 16 + tok] = f32_to_bf16_bits(pv[j] - bf16_bits_to_f32(hi));
            }
        }
        __syncwarp();
        const uint32_t bh0 = *reinterpret_cast<const uint32_t *>(pw + g * 16 + 2 * t);
        const uint32_t bh1 = *reinterpret_cast<const uint32_t *>(pw + g * 16 + 2 * t + 8);
        const uint32_t bl0 = *reinterpret_cast<const uint32_t *>(pw + 128 + g * 16 + 2 * t);
        const uint32_t bl1 = *reinterpret_cast<const uint32_t *>(pw + 128 + g * 16 + 2 * t + 8);
        // O^T += V^T P^T
        const uint32_t vrow = 16 * warp + (lane & 7) + ((lane >> 4) << 3);
#pragma unroll
        for (int dm = 0; dm < NT; ++dm) {
            uint32_t a[4];
            ldmatrix_x4_trans(a, vt + swz<HD>(vrow, 2 * dm + ((lane >> 3) & 1)));
            mma_bf16_16816(o[dm], a, bh0, bh1, o[dm]);
            mma_bf16_16816(o[dm], a, bl0, bl1, o[dm]);
        }
        __syncthreads();  // the stage is reloaded next iteration
    }
    // merge the 4 warps (fixed order): rows of o = dims 16dm + g (+8), columns = heads 2t, 2t+1
    float *mw = mrg + warp * 8 * (HD + 2);
    if (g == 0) {
        mw[(2 * t) * (HD + 2)] = m0, mw[(2 * t) * (HD + 2) + 1] = l0;
        mw[(2 * t + 1) * (HD + 2)] = m1, mw[(2 * t + 1) * (HD + 2) + 1] = l1;
    }
#pragma unroll
    for (int dm = 0; dm < NT; ++dm) {
        mw[(2 * t) * (HD + 2) + 2 + 16 * dm + g] = o[dm][0];
        mw[(2 * t + 1) * (HD + 2) + 2 + 16 * dm + g] = o[dm][1];
        mw[(2 * t) * (HD + 2) + 2 + 16 * dm + g + 8] = o[dm][2];
        mw[(2 * t + 1) * (HD + 2) + 2 + 16 * dm + g + 8] = o[dm][3];
    }
    __syncthreads();
    for (uint32_t i = tid; i < HPC * HD; i += kThreads) {
        const uint32_t h = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mrg[(w * 8 + h) * (HD + 2)]);
        float L = 0.0f, O = 0.0f;
        for (int w = 0; w < kWarps; ++w) {
            const float *r = mrg + (w * 8 + h) * (HD + 2);
            const float f = r[0] == -INFINITY ? 0.0f : __expf(r[0] - M);
            L += r[1] * f;
            O += r[2 + d] * f;
        }
        const size_t bh = (size_t)b * p.n_heads + h0 + h;
        if (p.splits == 1) {
            store_out(reinterpret_cast<OT *>(p.out) + bh * HD + d, O / L);
        } else {
            float *rec = p.ws + (bh * p.splits + split) * (HD + 2);
            rec[2 + d] = O;
            if (d == 0) rec[0] = M, rec[1] = L;
        }
    }
}

template <int HD, int HPC, typename QT, typename OT>
cudaError_t launch_mma(cudaStream_t stream, const Params &p, dim3 grid, bool pdl) {
    using C = MmaCfg<HD>;
    static bool attr_done = false;
    if (!attr_done) {
        const cudaError_t e = cudaFuncSetAttribute(attn_mma_kernel<HD, HPC, QT, OT>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_mma_kernel<HD, HPC, QT, OT>, p);
}

constexpr int kCombineThreads = 256, kCombineDims = 16;

// Block-wide max / sum of one value per thread, in a fixed order (the result does
// not depend on timing). `red` holds one float per warp.
__device__ __forceinline__ float block_reduce(float v, float *red, bool is_max) {
    for (int o = 16; o; o >>= 1) {
        const float w = __shfl_xor_sync(0xffffffffu, v, o);
        v = is_max ? fmaxf(v, w) : v + w;
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    v = red[0];
    for (int w = 1; w < kCombineThreads / 32; ++w) v = is_max ? fmaxf(v, red[w]) : v + red[w];
    return v;
}

// grid = (n_heads, batch, HD / kCombineDims), block = kCombineThreads: merge the
// slices of one (b, head) for kCombineDims of its output dims.  The block finds the
// slices' common max M, then walks the slices in chunks of kCombineThreads: each
// thread loads its kCombineDims slices' outputs (one dim each) first, turns one
// slice's max into its weight exp(m_s - M) (shared memory), and adds its weighted
// outputs; the per-thread sums of a dim are added in a fixed order at the end.
// Every load of a chunk is issued before the first one is used, so a few hundred
// slices cost about two L2 round trips, not one per slice.
template <int HD, typename OT>
__global__ void __launch_bounds__(kCombineThreads) attn_combine_kernel(Params p) {
    constexpr int T = kCombineThreads, DB = kCombineDims, G = T / DB;
    static_assert(HD % DB == 0 && T % DB == 0, "combine tiling");
    __shared__ float wgt[T];
    __shared__ float red[T / 32];
    __shared__ float part[G][DB];
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const uint32_t g = tid / DB, d = blockIdx.z * DB + tid % DB;
    const size_t bh = (size_t)b * p.n_heads + h;
    const float *rec = p.ws + bh * p.splits * (HD + 2);
    const uint32_t seq = seq_of(p, b);
    const uint32_t used = (seq + p.split_len - 1) / p.split_len;
    float m = -INFINITY;
    for (uint32_t s = tid; s < used; s += T) m = fmaxf(m, rec[(size_t)s * (HD + 2)]);
    const float M = block_reduce(m, red, true);
    float l = 0.0f, o = 0.0f;
    for (uint32_t base = 0; base < used; base += T) {
        const uint32_t cnt = min((uint32_t)T, used - base);
        const float *r = rec + (size_t)base * (HD + 2) + 2 + d;
        float v[T / G];
#pragma unroll
        for (int k = 0; k < T / G; ++k) {
            const uint32_t j = g + k * G;
            v[k] = j < cnt ? r[(size_t)j * (HD + 2)] : 0.0f;
        }
        float f = 0.0f;
        if (tid < cnt) {
            const float *rs = rec + (size_t)(base + tid) * (HD + 2);
            f = __expf(rs[0] - M);
            l += rs[1] * f;
        }
        __syncthreads();  // the previous chunk's weights are no longer read
        wgt[tid] = f;
        __syncthreads();
#pragma unroll
        for (int k = 0; k < T / G; ++k) {
            const uint32_t j = g + k * G;
            if (j < cnt) o += v[k] * wgt[j];
        }
    }
    const float L = block_reduce(l, red, false);
    part[g][tid % DB] = o;
    __syncthreads();
    if (tid < DB) {
        float O = part[0][tid];
#pragma unroll
        for (int k = 1; k < G; ++k) O += part[k][tid];
        store_out(reinterpret_cast<OT *>(p.out) + bh * HD + d, O / L);
    }
}

// grid = ceil(batch * n_heads / 8), block = 256: one warp per (b, head) merges all
// of that head's slices over all HD dims (lane k owns dims [k HD/32, (k+1) HD/32)).
// This is the form for many (b, head) rows with few slices each (batched decode):
// the dims-parallel kernel above launches HD/16 CTAs per row there, and at batch 64
// x 32 heads those 16k short CTAs cost ~50 us of launch waves for ~1 MB of records.
// Same arithmetic as above (common max, exp weights, sums over slices); the slices
// are summed in index order.
template <int HD, typename OT>
__global__ void __launch_bounds__(256) attn_combine_rows_kernel(Params p) {
    constexpr int VD = HD / 32, U = 8;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t bh = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (bh >= p.batch * p.n_heads) return;
    const float *rec = p.ws + (size_t)bh * p.splits * (HD + 2);
    const uint32_t seq = seq_of(p, bh / p.n_heads);
    const uint32_t used = (seq + p.split_len - 1) / p.split_len;
    float m = -INFINITY;
    for (uint32_t s = lane; s < used; s += 32) m = fmaxf(m, rec[(size_t)s * (HD + 2)]);
    m = warp_max(m);
    float l = 0.0f, o[VD];
#pragma unroll
    for (int i = 0; i < VD; ++i) o[i] = 0.0f;
    for (uint32_t base = 0; base < used; base += 32) {
        const uint32_t cnt = min(32u, used - base);
        float f = 0.0f;
        if (lane < cnt) {
            const float *rs = rec + (size_t)(base + lane) * (HD + 2);
            f = __expf(rs[0] - m);
            l += rs[1] * f;
        }
        // records are (HD + 2) floats, HD + 2 even: every output pair is 8-byte aligned
        const float *r = rec + (size_t)base * (HD + 2) + 2 + VD * lane;
        for (uint32_t j = 0; j < cnt; j += U) {
            float2 v[U][VD / 2];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int i = 0; i < VD / 2; ++i)
                    v[u][i] = j + u < cnt ? *reinterpret_cast<const float2 *>(r + (size_t)(j + u) * (HD + 2) + 2 * i)
                                          : make_float2(0.0f, 0.0f);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const float fj = __shfl_sync(0xffffffffu, f, (j + u) & 31);
                if (j + u < cnt)
#pragma unroll
                    for (int i = 0; i < VD / 2; ++i) o[2 * i] += v[u][i].x * fj, o[2 * i + 1] += v[u][i].y * fj;
            }
        }
    }
    const float L = warp_sum(l);
    OT *out = reinterpret_cast<OT *>(p.out) + (size_t)bh * HD + VD * lane;
#pragma unroll
    for (int i = 0; i < VD; ++i) store_out(out + i, o[i] / L);
}

// The slice merge for p: the dims-parallel kernel while its HD/16 CTAs per (b, head)
// fit about two waves of the GPU, else the warp-per-row kernel (at most 256 slices
// a row; more go to the dims-parallel form, whose chunks keep every load in flight).
// With pdl, the launch may be scheduled while the split kernel runs.
template <int HD, typename OT>
cudaError_t launch_combine(cudaStream_t stream, const Params &p, bool pdl) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const size_t rows = (size_t)p.batch * p.n_heads;
    const size_t wave = (size_t)num_sms() * (2048 / kCombineThreads);
    if (rows * (HD / kCombineDims) > 2 * wave && p.splits <= 256) {
        cfg.gridDim = dim3((unsigned)((rows + 7) / 8));
        cfg.blockDim = dim3(256);
        return cudaLaunchKernelEx(&cfg, attn_combine_rows_kernel<HD, OT>, p);
    }
    cfg.gridDim = dim3(p.n_heads, p.batch, HD / kCombineDims);
    cfg.blockDim = dim3(kCombineThreads);
    return cudaLaunchKernelEx(&cfg, attn_combine_kernel<HD, OT>, p);
}

// q heads per CTA: the whole GQA group when it is 4 or 8 (else 8 or 4 of it, else 1).
uint32_t heads_per_cta(uint32_t group, bool group_heads) {
    if (!group_heads) return 1;
    if (group % 8 == 0) return 8;
    if (group % 4 == 0) return 4;
    return 1;
}

size_t workspace_bytes(uint32_t batch, uint32_t n_heads, uint32_t head_dim, uint32_t splits) {
    return splits <= 1 ? 0 : (size_t)batch * n_heads * splits * (head_dim + 2) * sizeof(float);
}

// Slices per (row, head group), from a wave model of the split kernel: a CTA walks
// its slice one 64-token tile at a time, and a tile costs the larger of the CTA's
// own time per tile (0.9 us at head_dim 64, 1.17 us at 128: issue and latency
// bound) and the HBM time of one tile of every CTA resident in that wave (at
// 6.5 TB/s); each CTA adds a prologue/epilogue cost (1.5 / 3 us), CTAs past the
// resident slots (CTAs per SM, from the kernel's shared memory, x SMs) run in
// further waves, and more than one slice adds the combine launch.  The
// constants were fitted to split-count sweeps on B200 (batch 1 and 8, contexts
// 2k-32k); the model keeps the last wave from holding a handful of CTAs.
uint32_t choose_splits(uint32_t batch, uint32_t groups, uint32_t seq, uint32_t hd) {
    if (seq <= 64) return 1;
    const bool wide = hd > 64;
    const double smem = wide ? (double)MmaCfg<128>::kSmem : (double)MmaCfg<64>::kSmem;
    const double slots = std::max(1.0, std::floor(233472.0 / (smem + 1024.0))) * num_sms();
    const double tile_bytes = 64.0 * hd * 2 * 2, tile_own = wide ? 1.17 : 0.9, cta_fixed = wide ? 3.0 : 1.5;
    double best = 0.0;
    uint32_t pick = 1;
    for (uint32_t s = 1; s <= 256; ++s) {
        const uint32_t len = (seq + s - 1) / s;
        if (s > 1 && len < 64) break;
        const uint32_t used = (seq + len - 1) / len;
        if (used != s) continue;  // same geometry as a smaller count
        const double tiles = (double)((len + 63) / 64);
        double left = (double)batch * groups * s, t = s > 1 ? 1.0 + 0.01 * s : 0.0;
        while (left > 0) {
            const double n = std::min(left, slots);
            t += tiles * std::max(tile_own, n * tile_bytes / 6.5e6) + cta_fixed;
            left -= n;
        }
        if (s == 1 || t < best - 1e-9) best = t, pick = s;
    }
    return pick;
}

template <typename QT, typename KT, typename OT>
int run(cudaStream_t stream, uint32_t batch, uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t seq,
        uint32_t max_seq, const QT *q, const KT *kc, const KT *vc, OT *out, void *ws, size_t ws_bytes,
        bool group_heads) {
    FP4X_REQUIRE(q && kc && vc && out, "llama_attn_decode: null pointer");
    FP4X_REQUIRE(hd == 64 || hd == 128, "llama_attn_decode: head_dim %u not in {64, 128}", hd);
    FP4X_REQUIRE(n_kv > 0 && n_heads % n_kv == 0, "llama_attn_decode: n_heads %% n_kv_heads != 0");
    FP4X_REQUIRE(batch > 0 && seq > 0 && seq <= max_seq, "llama_attn_decode: need 0 < seq <= max_seq");
    const uint32_t group = n_heads / n_kv;
    const uint32_t hpc = heads_per_cta(group, group_heads);
    uint32_t splits = 1;
    if (ws) {
        splits = choose_splits(batch, n_heads / hpc, seq, hd);
        while (splits > 1 && workspace_bytes(batch, n_heads, hd, splits) > ws_bytes) splits /= 2;
    }
    Params p;
    p.batch = batch, p.n_heads = n_heads, p.n_kv = n_kv, p.seq = seq, p.max_seq = max_seq;
    p.split_len = (seq + splits - 1) / splits;
    p.splits = (seq + p.split_len - 1) / p.split_len;
    p.scale = 1.0f / sqrtf((float)hd);
    p.q = q, p.kc = kc, p.vc = vc, p.out = out, p.ws = static_cast<float *>(ws);
    p.pos_ptr = nullptr;
    dim3 grid(p.splits, n_heads / hpc, batch);
    if (sizeof(KT) == 2 && (hpc == 4 || hpc == 8)) {
        cudaError_t e = cudaSuccess;
        if (hd == 64 && hpc == 8) e = launch_mma<64, 8, QT, OT>(stream, p, grid, false);
        if (hd == 64 && hpc == 4) e = launch_mma<64, 4, QT, OT>(stream, p, grid, false);
        if (hd == 128 && hpc == 8) e = launch_mma<128, 8, QT, OT>(stream, p, grid, false);
        if (hd == 128 && hpc == 4) e = launch_mma<128, 4, QT, OT>(stream, p, grid, false);
        if (e == cudaSuccess && p.splits > 1)
            e = hd == 64 ? launch_combine<64, OT>(stream, p, true) : launch_combine<128, OT>(stream, p, true);
        if (e != cudaSuccess) {
            set_error("llama_attn_decode: %s", cudaGetErrorString(e));
            return FP4X_ECUDA;
        }
        return check_launch("llama_attn_decode");
    }
#define FP4X_ATTN_CASE(HD_, HPC_)                                                                       \
    if (hd == HD_ && hpc == HPC_) {                                                                   \
        attn_split_kernel<HD_, HPC_, QT, KT, OT><<<grid, kThreads, 0, stream>>>(p);                   \
        if (p.splits > 1) (void)launch_combine<HD_, OT>(stream, p, false);                           \
    }
    FP4X_ATTN_CASE(64, 1)
    FP4X_ATTN_CASE(64, 4)
    FP4X_ATTN_CASE(64, 8)
    FP4X_ATTN_CASE(128, 1)
    FP4X_ATTN_CASE(128, 4)
    FP4X_ATTN_CASE(128, 8)
#undef FP4X_ATTN_CASE
    return check_launch("llama_attn_decode");
}

// Engine form: f32 q/out, bf16 caches, seq from *pos_ptr + 1 on the device, a
// fixed grid of `splits` slices of `split_len` tokens (slices past seq exit),
// launched with programmatic dependent launch.
template <int HD, int HPC>
int launch_engine_t(cudaStream_t stream, const Params &p, bool pdl) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.splits, p.n_heads / HPC, p.batch);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = (HPC == 4 || HPC == 8) ? launch_mma<HD, HPC, float, float>(stream, p, cfg.gridDim, pdl)
                                            : cudaLaunchKernelEx(&cfg, attn_split_kernel<HD, HPC, float, uint16_t, float>, p);
    if (e == cudaSuccess && p.splits > 1) e = launch_combine<HD, float>(stream, p, pdl);
    if (e != cudaSuccess) {
        set_error("attention (engine): %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    return FP4X_OK;
}

int launch_engine(cudaStream_t stream, const Params &p, uint32_t head_dim, bool pdl) {
    const uint32_t hpc = heads_per_cta(p.n_heads / p.n_kv, true);
    if (head_dim == 64 && hpc == 8) return launch_engine_t<64, 8>(stream, p, pdl);
    if (head_dim == 64 && hpc == 4) return launch_engine_t<64, 4>(stream, p, pdl);
    if (head_dim == 64 && hpc == 1) return launch_engine_t<64, 1>(stream, p, pdl);
    if (head_dim == 128 && hpc == 8) return launch_engine_t<128, 8>(stream, p, pdl);
    if (head_dim == 128 && hpc == 4) return launch_engine_t<128, 4>(stream, p, pdl);
    if (head_dim == 128 && hpc == 1) return launch_engine_t<128, 1>(stream, p, pdl);
    set_error("attention (engine): unsupported head_dim %u", head_dim);
    return FP4X_EUNSUPPORTED;
}

}  // namespace attn
}  // namespace fp4x

using namespace fp4x;

extern "C" int llama_attn_decode(fp4x_stream_t stream, uint32_t n_heads, uint32_t n_kv_heads, uint32_t seq,
                                 const float *q, const float *kc, const float *vc, float *out) {
    // Reference signature (head_dim fixed at 64, llama_run/src/main.rs:19), no workspace:
    // one CTA per q head over the whole sequence.
    return attn::run<float, float, float>((cudaStream_t)stream, 1, n_heads, n_kv_heads, 64, seq, seq, q, kc, vc, out,
                                          nullptr, 0, false);
}

extern "C" int llama_attn_decode_hd(fp4x_stream_t stream, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                                    uint32_t seq, const float *q, const float *kc, const float *vc, float *out,
                                    void *workspace, size_t workspace_bytes) {
    return attn::run<float, float, float>((cudaStream_t)stream, 1, n_heads, n_kv_heads, head_dim, seq, seq, q, kc, vc,
                                          out, workspace, workspace_bytes, true);
}

extern "C" size_t llama_attn_workspace_size(uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                                            uint32_t seq) {
    if (n_kv_heads == 0 || n_heads % n_kv_heads) return 0;
    const uint32_t hpc = attn::heads_per_cta(n_heads / n_kv_heads, true);
    return attn::workspace_bytes(batch, n_heads, head_dim, attn::choose_splits(batch, n_heads / hpc, seq, head_dim));
}

extern "C" int llama_attn_decode_bf16(fp4x_stream_t stream, uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads,
                                      uint32_t head_dim, uint32_t seq, uint32_t max_seq, const uint16_t *q,
                                      const uint16_t *kc, const uint16_t *vc, uint16_t *out, void *workspace,
                                      size_t workspace_bytes) {
    return attn::run<uint16_t, uint16_t, uint16_t>((cudaStream_t)stream, batch, n_heads, n_kv_heads, head_dim, seq,
                                                   max_seq, q, kc, vc, out, workspace, workspace_bytes, true);
}

extern "C" int llama_attn_decode_f32q_bf16kv(fp4x_stream_t stream, uint32_t batch, uint32_t n_heads,
                                             uint32_t n_kv_heads, uint32_t head_dim, uint32_t seq, uint32_t max_seq,
                                             const float *q, const uint16_t *kc, const uint16_t *vc, float *out,
                                             void *workspace, size_t workspace_bytes) {
    return attn::run<float, uint16_t, float>((cudaStream_t)stream, batch, n_heads, n_kv_heads, head_dim, seq, max_seq,
                                             q, kc, vc, out, workspace, workspace_bytes, true);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of llama_attn_decode_bf16.
//
// Some callers cannot allocate device memory for the split-KV partials: a host
// whose device memory is owned by its own pool allocator and must not see a
// cudaMalloc from inside a plugin, or a latency-critical serving loop where
// cudaMalloc/cudaFree (which can synchronise the device) are not allowed.  For
// them the partials live in one file-scope __device__ array of fixed size,
// kNoAllocScratchFloats floats (4 MiB), which every GPU that loads this library
// holds until the process exits.  In host code the array's name is only a
// host-side stand-in, so its device address is looked up with
// cudaGetSymbolAddress on the first call made in each CUDA context (the device's
// primary context for runtime-API callers; make that first call before any
// stream capture) and cached per context: a caller that switches to another
// context, or resets the device, gets the address in the context it runs in.
//
// All calls share the array and it keeps the last call's contents.  Nothing in
// it has to start at zero: every slice record a call reads was written earlier
// in the same call.  Calls whose kernels overlap on the GPU (different streams,
// or host threads racing on one device) write the same memory and race; callers
// must serialise them, e.g. by issuing them on one stream.
namespace fp4x {
namespace attn {

constexpr size_t kNoAllocScratchFloats = size_t(1) << 20;  // 4 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// Addresses already looked up, keyed by the driver's context id (cuCtxGetId: unique
// for the life of the process, so a context created after a device reset never
// matches an entry of the one it replaced).
constexpr int kNoAllocMaxCtx = 64;
struct NoAllocEntry {
    unsigned long long id;
    float *ptr;
};
static NoAllocEntry g_noalloc_cache[kNoAllocMaxCtx] = {};
static int g_noalloc_n = 0, g_noalloc_next = 0;
static std::mutex g_noalloc_mu;

using PfnCtxGetCurrent = int (*)(void **);
using PfnCtxGetId = int (*)(void *, unsigned long long *);

// Id of the calling thread's current context; false if there is none (or the
// driver does not export the calls).
static bool current_context_id(unsigned long long *id) {
    static PfnCtxGetCurrent get = nullptr;
    static PfnCtxGetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get = reinterpret_cast<PfnCtxGetCurrent>(fn);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PfnCtxGetId>(fn);
    });
    void *ctx = nullptr;
    if (!get || !get_id || get(&ctx) != 0 || ctx == nullptr) return false;
    return get_id(ctx, id) == 0;
}

static int noalloc_scratch(float **out) {
    unsigned long long id = 0;
    bool have_id = current_context_id(&id);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (have_id)
        for (int i = 0; i < g_noalloc_n; ++i)
            if (g_noalloc_cache[i].id == id) {
                *out = g_noalloc_cache[i].ptr;
                return FP4X_OK;
            }
    // first call in this context (for a runtime-API caller with no context yet,
    // this lookup creates the device's primary context)
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
        set_error("llama_attn_decode_bf16_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    if (!have_id) have_id = current_context_id(&id);
    if (have_id) {  // no id (old driver): look the address up on every call
        const int slot = g_noalloc_n < kNoAllocMaxCtx ? g_noalloc_n++ : g_noalloc_next++ % kNoAllocMaxCtx;
        g_noalloc_cache[slot] = {id, static_cast<float *>(p)};
    }
    *out = static_cast<float *>(p);
    return FP4X_OK;
}

}  // namespace attn
}  // namespace fp4x

extern "C" size_t llama_attn_noalloc_max_bytes(void) { return attn::kNoAllocScratchFloats * sizeof(float); }

extern "C" int llama_attn_decode_bf16_noalloc(fp4x_stream_t stream, uint32_t batch, uint32_t n_heads,
                                              uint32_t n_kv_heads, uint32_t head_dim, uint32_t seq, uint32_t max_seq,
                                              const uint16_t *q, const uint16_t *kc, const uint16_t *vc,
                                              uint16_t *out) {
    FP4X_REQUIRE(n_kv_heads > 0 && n_heads % n_kv_heads == 0, "llama_attn_decode_bf16_noalloc: n_heads %% n_kv != 0");
    const size_t need = llama_attn_workspace_size(batch, n_heads, n_kv_heads, head_dim, seq);
    const size_t cap = attn::kNoAllocScratchFloats * sizeof(float);
    FP4X_REQUIRE(need <= cap,
                 "llama_attn_decode_bf16_noalloc: this shape needs %zu bytes of split-KV scratch, above the %zu-byte "
                 "static maximum; use llama_attn_decode_bf16 with a caller workspace",
                 need, cap);
    float *scratch = nullptr;
    if (need > 0) {
        const int st = attn::noalloc_scratch(&scratch);
        if (st) return st;
    }
    return attn::run<uint16_t, uint16_t, uint16_t>((cudaStream_t)stream, batch, n_heads, n_kv_heads, head_dim, seq,
                                                   max_seq, q, kc, vc, out, scratch, need ? cap : 0, true);
}
