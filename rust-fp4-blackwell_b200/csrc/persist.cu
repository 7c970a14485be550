// persist.cu -- persistent MXFP4 decode kernel for sm_100a.
//
// The reference runs a token as 377 host-issued launches of independent SIMT
// kernels (examples/llama_run/src/main.rs:512-534).  At batch 1 a token is a
// 549.5 MB weight stream and every linear is a few MB, far too small to keep
// HBM busy on its own (6.5 TB/s x ~1 us latency = ~8 MB must be in flight), so
// this kernel runs whole generations in ONE cooperative launch with one CTA per
// SM:
//   * producer warp: streams this CTA's pre-packed weight chunks (its fixed
//     share of every linear, in consumption order) into a ring of shared-memory
//     slots with cp.async.bulk; weights never depend on activations, so it runs
//     ahead across phases, layers and tokens, bounded only by the ring;
//   * 8 consumer warps: per layer three phases separated by grid barriers,
//       A  RMSNorm + QKV rows + RoPE + bf16 KV append            (llama_run:513-521)
//       B  attention of the heads whose O columns this CTA holds, then the O
//          projection restricted to those columns (split-K by head), added
//          into the residual stream with red.add                  (:522-524)
//       C  RMSNorm + gate/up rows of this CTA's FFN slice + SwiGLU, then the
//          down projection restricted to that slice (split-K by FFN index),
//          added into an FFN-delta buffer                          (:525-530)
//     and once per token: final RMSNorm + lm_head rows + per-CTA argmax, a
//     grid barrier, then every CTA reduces the 148 candidates itself (ties to
//     the lowest index, :287) and feeds the next token (:550-566).
//   * The residual stream after a layer is X + Y: phase C reads X while other
//     CTAs are still adding, so the FFN delta goes to Y, which the next layer's
//     phase B folds into X (red.add) and zeroes.  Summation order of those
//     atomics varies, so results are reproducible to ~1e-7 relative, not bits.
//
// Weight records ("fragment order"): for a 16-row tile and one 32-k block, 256
// bytes = lane (g = lane/4, t = lane%4) x 8 bytes, where byte h*4 + j feeds mma
// register a_j of half h: rows g (+8 for odd j), k = 8t + 4h + 2(j/2) + {0,1};
// then 16 E8M0 bytes (one per row).  A lane loads its 8 bytes with one LDS.64,
// decodes each byte with cvt.rn.f16x2.e2m1x2 straight into an mma.m16n8k16 A
// register, and the activation's matching pairs are the natural x[8t .. 8t+7]
// of the block (one LDS.128).  The 8 mma columns carry (block j of a 4-block
// group, hi | lo of the f16 split activation).
#include "common.cuh"
#include "persist.cuh"

#include <algorithm>
#include <vector>

namespace fp4x {
namespace persist {

constexpr uint32_t kBarLimit = 1u << 24;

// Phase timestamps of CTA 0 (globaltimer, ns), only in builds compiled with
// -DFP4X_PHASE_TIMING; a no-op otherwise.
#ifdef FP4X_PHASE_TIMING
constexpr uint32_t kStamps = 1u << 16;
__device__ unsigned long long g_phase_ts[kStamps];
__device__ __forceinline__ void stamp(uint32_t i) {
    if (blockIdx.x == 0 && threadIdx.x == 0 && i < kStamps) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g_phase_ts[i] = t;
    }
}
// producer issue times of chunks (CTA 0), from index kStamps / 2
__device__ __forceinline__ void pstamp(uint32_t seq) {
    if (blockIdx.x == 0 && (threadIdx.x & 31) == 0 && seq < kStamps / 4) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g_phase_ts[kStamps / 2 + seq] = t;
    }
}
// consumer chunk wait / compute times (CTA 0), from index 3 * kStamps / 4
__device__ __forceinline__ void cstamp(uint32_t i) {
    if (blockIdx.x == 0 && threadIdx.x == 0 && i < kStamps / 4) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g_phase_ts[3 * kStamps / 4 + i] = t;
    }
}
#else
__device__ __forceinline__ void stamp(uint32_t) {}
__device__ __forceinline__ void pstamp(uint32_t) {}
__device__ __forceinline__ void cstamp(uint32_t) {}
#endif

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); }

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_add(float *p, float v) {
    asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

struct Smem {
    uint32_t bars, red, xh, xl, xpost, ofl, oh, ol, opost, s16h, s16l, spost, qs, wst, ps, dacc, flag, sched, cbytes,
        ring, total;
};

__host__ __device__ inline Smem smem_layout(const Params &p) {
    Smem L;
    uint32_t off = 0;
    auto take = [&](uint32_t bytes, uint32_t align) {
        off = (off + align - 1) / align * align;
        const uint32_t o = off;
        off += bytes;
        return o;
    };
    const uint32_t hd = p.hd;
    L.bars = take(2 * kMaxSlots * 8, 16);
    L.red = take(512 * 4, 16);
    L.xh = take(p.dim * 2, 16);
    L.xl = take(p.dim * 2, 16);
    L.xpost = take(p.dim / 32 * 4, 16);
    L.ofl = take(kMaxBHeads * hd * 4, 16);
    L.oh = take(kMaxBHeads * hd * 2, 16);
    L.ol = take(kMaxBHeads * hd * 2, 16);
    L.opost = take(kMaxBHeads * hd / 32 * 4, 16);
    L.s16h = take(kMaxUnits * 16 * 2, 16);
    L.s16l = take(kMaxUnits * 16 * 2, 16);
    L.spost = take(kMaxUnits * 4, 16);
    L.qs = take(kMaxBHeads * hd * 4, 16);
    L.wst = take(kConsumerWarps * (hd + 2) * 4, 16);
    L.ps = 0;
    L.dacc = take(p.dim * 4, 16);
    L.flag = take(16, 16);  // [0] barrier verdict, [1] local failure
    L.sched = take(sizeof(CtaSched), 16);       // this CTA's schedule, staged once
    L.cbytes = take(p.chunk_stride * 4, 16);     // its chunk sizes, staged once
    L.ring = take(p.n_slots * p.slot_bytes, 128);
    L.total = off;
    return L;
}

// ---------------------------------------------------------------- consumer helpers

// float offsets inside the consumers' 512-float scratch (Ctx::red)
constexpr int kRedSS = 0;                                // [kConsumerWarps] sum-of-squares partials
constexpr int kRedPart = 32;                             // [kConsumerWarps][16] row partials
constexpr int kRedYT = kRedPart + kConsumerWarps * 16;   // [16] values of the current tile
constexpr int kRedSV = kRedYT + 32;                      // [16] SwiGLU values of the current unit
constexpr int kRedArg = kRedSV + 32;                     // argmax value, index
static_assert(kRedArg + 2 <= 512, "consumer scratch overflow");

struct Ctx {
    const Params *p;
    uint8_t *smem;
    Smem L;
    uint64_t *full, *empty;
    uint8_t *ring;
    float *red;
    uint32_t seq;       // next chunk to consume
    uint32_t nbar;      // grid barriers passed
    bool ok;
};

// All consumer threads call this; a thread whose bounded chunk wait failed
// (c.ok false) keeps going to here, so every exit decision is CTA-uniform.
__device__ bool grid_barrier(Ctx &c) {
    const Params &p = *c.p;
    volatile uint32_t *flag = reinterpret_cast<volatile uint32_t *>(c.smem + c.L.flag);
    if (!c.ok) flag[1] = 1;  // sticky local failure
    csync();
    c.nbar += 1;
    if (threadIdx.x == 0) {
        if (flag[1]) atomicExch(&p.bar[1], 1u);
        // release: the CTA's writes (ordered before this thread by the CTA barrier)
        // are visible before the arrival; one instruction instead of fence + add
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&p.bar[0]) : "memory");
        const uint32_t target = c.nbar * gridDim.x;
        uint32_t ok = 1;
        for (uint32_t i = 0;; ++i) {
            if (ld_acquire(&p.bar[0]) >= target) break;
            // the abort word is read every 64 polls: a second load per poll would
            // wait behind the acquire and double the poll period
            if ((i & 63) == 63 && ld_volatile(&p.bar[1])) {
                ok = 0;
                break;
            }
            if (i > kBarLimit) {
                atomicExch(&p.bar[1], 1u);
                raise_device_error(DEVERR_FLAG_TIMEOUT);
                ok = 0;
                break;
            }
            __nanosleep(64);
        }
        // the acquire load above already orders this CTA's later reads (the CTA
        // barrier below passes that on)
        flag[0] = ok;
    }
    csync();
    c.ok = flag[0] != 0;
    return c.ok;
}

// Wait for the next chunk.  A wait that runs out only marks this thread's
// context failed (no early return: the CTA decides to stop at its next grid
// barrier, uniformly); the slot is then read stale, never out of bounds.
__device__ const uint8_t *chunk_acquire(Ctx &c) {
    const Params &p = *c.p;
    const uint32_t slot = c.seq % p.n_slots, parity = (c.seq / p.n_slots) & 1;
    cstamp(3 * c.seq);
    if (c.ok && !mbar_wait_bounded(&c.full[slot], parity)) c.ok = false;
    cstamp(3 * c.seq + 1);
    return c.ring + (size_t)slot * p.slot_bytes;
}

__device__ void chunk_release(Ctx &c) {
    const Params &p = *c.p;
    cstamp(3 * c.seq + 2);
    csync();
    if (threadIdx.x == 0) mbar_arrive(&c.empty[c.seq % p.n_slots]);
    c.seq += 1;
}

// Stage RMSNorm's input: v = (src) * w as f16 hi/lo per 32-block (prescaled),
// returns rms = 1/sqrt(mean(src^2) + eps).  src = X (+ Y) or an embedding row;
// CTA 0 writes the embedding row to X when `x_out` is set.
template <int MODE>  // 0: X, 1: X + Y, 2: bf16 embedding row
__device__ float stage_norm(Ctx &c, const float *X, const float *Y, const uint16_t *erow, const float *w,
                            float *x_out) {
    const Params &p = *c.p;
    __half *xh = reinterpret_cast<__half *>(c.smem + c.L.xh);
    __half *xl = reinterpret_cast<__half *>(c.smem + c.L.xl);
    float *xpost = reinterpret_cast<float *>(c.smem + c.L.xpost);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t nb = p.dim / 32, nchunks = (nb + 3) / 4;
    float ss = 0.0f;
    constexpr int CH = 8;  // chunks per warp in flight (dim <= 8192 in one round)
    for (uint32_t ch0 = warp; ch0 < nchunks; ch0 += CH * kConsumerWarps) {
        float4 r[CH], wv[CH];
#pragma unroll
        for (int u = 0; u < CH; ++u) {
            const uint32_t ch = ch0 + u * kConsumerWarps, b = 4 * ch + (lane >> 3), i = ch * 128 + lane * 4;
            r[u] = wv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ch < nchunks && b < nb) {
                if (MODE == 2) {
                    const uint2 q = *reinterpret_cast<const uint2 *>(erow + i);
                    r[u] = make_float4(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xFFFF0000u),
                                       __uint_as_float(q.y << 16), __uint_as_float(q.y & 0xFFFF0000u));
                } else {
                    r[u] = __ldcg(reinterpret_cast<const float4 *>(X + i));
                    if (MODE == 1) {
                        const float4 y = __ldcg(reinterpret_cast<const float4 *>(Y + i));
                        r[u].x += y.x, r[u].y += y.y, r[u].z += y.z, r[u].w += y.w;
                    }
                }
                wv[u] = __ldg(reinterpret_cast<const float4 *>(w + i));
            }
        }
#pragma unroll
        for (int u = 0; u < CH; ++u) {
            const uint32_t ch = ch0 + u * kConsumerWarps, b = 4 * ch + (lane >> 3), i = ch * 128 + lane * 4;
            if (ch < nchunks) {  // warp-uniform
                const bool valid = b < nb;
                if (MODE == 2 && x_out && valid) *reinterpret_cast<float4 *>(x_out + i) = r[u];
                ss += r[u].x * r[u].x + r[u].y * r[u].y + r[u].z * r[u].z + r[u].w * r[u].w;
                gemv::split4(make_float4(r[u].x * wv[u].x, r[u].y * wv[u].y, r[u].z * wv[u].z, r[u].w * wv[u].w),
                             i, b, lane, valid, xh, xl, xpost);
            }
        }
    }
    ss = warp_sum(ss);
    if (lane == 0) c.red[kRedSS + warp] = ss;
    csync();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < kConsumerWarps; ++i) tot += c.red[kRedSS + i];
    csync();
    return 1.0f / sqrtf(tot / (float)p.dim + p.eps);
}

// Split `n` (<= 32 * kConsumerWarps) f32 values from shared memory into f16 hi/lo
// with a prescale per 32-block (one warp per block).
__device__ void stage_small(const float *v, uint32_t n, __half *xh, __half *xl, float *xpost) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (uint32_t b = warp; b * 32 < n; b += kConsumerWarps) {
        const uint32_t i = b * 32 + lane;
        const float x = i < n ? v[i] : 0.0f;
        const float m = warp_max(fabsf(x));
        const int ex = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;
        int s = (m > 0.0f && ex < 128 && ex > -127) ? 14 - ex : 0;
        s = max(-126, min(126, s));
        const float xs = x * __uint_as_float((uint32_t)(s + 127) << 23);
        const __half h = __float2half_rn(xs);
        if (i < n) {
            xh[i] = h;
            xl[i] = __float2half_rn(xs - __half2float(h));
        }
        if (lane == 0) xpost[b] = __uint_as_float((uint32_t)(127 - s) << 23);
    }
}

// Row sums of one 16-row record over the 4-block group starting at block b (nv
// valid blocks): the 8 mma columns carry (block j, hi|lo); block j accumulates in
// its own register set d[j] (chains of 2 mma, not 8), and lane (g, t) reads rows
// g, g+8 of block t from columns 2t, 2t+1 (the other d[j] are zero there).
__device__ __forceinline__ void group_dot(const uint8_t *nib, const uint8_t *sc, uint32_t b, uint32_t nv,
                                          const __half *xh, const __half *xl, const float *xpost, float &acc0,
                                          float &acc1) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, my_j = g >> 1;
    const __half *xmine = (g & 1) ? xl : xh;
    uint4 xv = make_uint4(0, 0, 0, 0);
    if (my_j < (int)nv) xv = *reinterpret_cast<const uint4 *>(xmine + (b + my_j) * 32 + 8 * t);
    uint2 wv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
        wv[j] = j < (int)nv ? *reinterpret_cast<const uint2 *>(nib + (b + j) * 256 + lane * 8) : make_uint2(0, 0);
    float d[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        d[j][0] = d[j][1] = d[j][2] = d[j][3] = 0.0f;
        if (j < (int)nv) {
            uint32_t a0[4], a1[4];
            decode_word_f16(wv[j].x, a0);
            decode_word_f16(wv[j].y, a1);
            const bool mine = (j == my_j);
            mma_f16_16816(d[j], a0, mine ? xv.x : 0u, mine ? xv.y : 0u, d[j]);
            mma_f16_16816(d[j], a1, mine ? xv.z : 0u, mine ? xv.w : 0u, d[j]);
        }
    }
    if (t < (int)nv) {
        const float h0 = (d[0][0] + d[1][0]) + (d[2][0] + d[3][0]), l0 = (d[0][1] + d[1][1]) + (d[2][1] + d[3][1]);
        const float h1 = (d[0][2] + d[1][2]) + (d[2][2] + d[3][2]), l1 = (d[0][3] + d[1][3]) + (d[2][3] + d[3][3]);
        const float xp = xpost[b + t];
        acc0 += e8m0_to_f32(sc[(b + t) * 16 + g]) * xp * (h0 + l0);
        acc1 += e8m0_to_f32(sc[(b + t) * 16 + g + 8]) * xp * (h1 + l1);
    }
}

// 16 row values (times rowscale) of a full-K tile record; all consumer warps
// split its 4-block groups, then reduce through shared memory in warp order.
__device__ void tile_rows(Ctx &c, const uint8_t *rec, uint32_t nb, float rowscale, float *yt) {
    const __half *xh = reinterpret_cast<const __half *>(c.smem + c.L.xh);
    const __half *xl = reinterpret_cast<const __half *>(c.smem + c.L.xl);
    const float *xpost = reinterpret_cast<const float *>(c.smem + c.L.xpost);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const uint32_t ng = (nb + 3) / 4;
    float acc0 = 0.0f, acc1 = 0.0f;
    for (uint32_t grp = warp; grp < ng; grp += kConsumerWarps)
        group_dot(rec, rec + nb * 256, grp * 4, min(4u, nb - grp * 4), xh, xl, xpost, acc0, acc1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    float *part = c.red + kRedPart;
    if (t == 0) {
        part[warp * 16 + g] = acc0;
        part[warp * 16 + g + 8] = acc1;
    }
    csync();
    if (threadIdx.x < 16) {
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < kConsumerWarps; ++i) s += part[i * 16 + threadIdx.x];
        yt[threadIdx.x] = s * rowscale;
    }
    csync();
}

// ---------------------------------------------------------------- phases

// A: RMSNorm + QKV rows of this CTA + RoPE + KV append (rope-paired tiles: rows
// 0..7 = head rows j0.., rows 8..15 = j0 + hd/2 ..).
__device__ void phase_qkv(Ctx &c, const CtaSched &S, uint32_t l, uint32_t tok, uint32_t pos) {
    const Params &p = *c.p;
    float rms;
    if (l == 0)
        rms = stage_norm<2>(c, nullptr, nullptr, p.embed + (size_t)tok * p.dim, p.attn_norm,
                            blockIdx.x == 0 ? p.X : nullptr);
    else
        rms = stage_norm<1>(c, p.X, p.Y, nullptr, p.attn_norm + (size_t)l * p.dim, nullptr);
    float *yt = c.red + kRedYT;
    const uint32_t hd = p.hd, half = hd / 2, tph = half / 8, kvrow = p.n_kv * hd;
    uint16_t *kc = p.kc + (size_t)l * p.max_seq * kvrow, *vc = p.vc + (size_t)l * p.max_seq * kvrow;
    for (uint32_t i = 0; i < S.n_a; ++i) {
        const uint8_t *rec = chunk_acquire(c);
        tile_rows(c, rec, p.dim / 32, rms, yt);
        chunk_release(c);
        const uint32_t tile = S.a_tile[i];
        const int tid = threadIdx.x;
        if (tile < p.q_tiles + p.k_tiles) {
            if (tid < 8) {
                const bool is_q = tile < p.q_tiles;
                const uint32_t lt = is_q ? tile : tile - p.q_tiles;
                const uint32_t head = lt / tph, j = (lt % tph) * 8 + tid;
                const float cs = p.cos_t[(size_t)pos * half + j], sn = p.sin_t[(size_t)pos * half + j];
                const float x0 = yt[tid], x1 = yt[tid + 8];
                const float o0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));  // llama_run:135-136
                const float o1 = __fadd_rn(__fmul_rn(x1, cs), __fmul_rn(x0, sn));
                if (is_q) {
                    p.q[head * hd + j] = o0;
                    p.q[head * hd + j + half] = o1;
                } else {
                    uint16_t *dst = kc + (size_t)pos * kvrow + head * hd;
                    dst[j] = f32_to_bf16_bits(o0);
                    dst[j + half] = f32_to_bf16_bits(o1);
                }
            }
        } else if (tid < 16) {
            const uint32_t vi = (tile - p.q_tiles - p.k_tiles) * 16 + tid;
            vc[(size_t)pos * kvrow + vi] = f32_to_bf16_bits(yt[tid]);
        }
        csync();
    }
}

// One step of a warp reduce-scatter: lanes whose bit `O` is set keep the upper
// half of v[0..N), the others the lower half, each adding the partner's copy.
template <int M, int N, int O>
__device__ __forceinline__ void rs_step(float (&v)[M], int lane) {
    const bool up = (lane & O) != 0;
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
        const float keep = up ? v[i + N / 2] : v[i];
        const float send = up ? v[i] : v[i + N / 2];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
    }
}

// Sum 32 per-lane values over the warp; lane L ends with element L.
__device__ __forceinline__ float reduce_scatter32(float (&v)[32], int lane) {
    rs_step<32, 32, 16>(v, lane);
    rs_step<32, 16, 8>(v, lane);
    rs_step<32, 8, 4>(v, lane);
    rs_step<32, 4, 2>(v, lane);
    rs_step<32, 2, 1>(v, lane);
    return v[0];
}

// Attention of heads h0 .. h0+nh-1 over positions 0..pos (llama_run:148-242
// semantics, 1/sqrt(hd) scale), the heads in parallel on groups of warps; each
// warp runs an online softmax over 32-token tiles with lane = token for both
// Q.K and P.V (K and V rows fetched with 16-byte loads, the P.V sums
// reduce-scattered so lane L keeps dims 32c + L), then the group's warps are
// merged and the result is staged as f16 hi/lo into head slots 0..nh-1.
template <int HD>
__device__ void attend(Ctx &c, uint32_t l, uint32_t h0, uint32_t nh, uint32_t pos) {
    const Params &p = *c.p;
    constexpr int NC = HD / 32;  // 32-dim chunks per head
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, tid = threadIdx.x;
    const uint32_t wpg = nh <= 1 ? kConsumerWarps : (nh == 2 ? kConsumerWarps / 2 : kConsumerWarps / 4);
    const uint32_t grp = warp / wpg, wl = warp % wpg;
    float *qs = reinterpret_cast<float *>(c.smem + c.L.qs);    // [kMaxBHeads][HD]
    float *wst = reinterpret_cast<float *>(c.smem + c.L.wst);  // [warp][HD + 2]
    const uint32_t kvrow = p.n_kv * HD, seq = pos + 1, group = p.n_heads / p.n_kv;
    const float scale = 1.0f / sqrtf((float)HD);
    for (uint32_t i = tid; i < nh * HD; i += kConsumers) qs[i] = __ldcg(p.q + h0 * HD + i) * scale;
    csync();
    float m = -INFINITY, lsum = 0.0f, o[NC];
#pragma unroll
    for (int i = 0; i < NC; ++i) o[i] = 0.0f;
    if (grp < nh) {
        const uint32_t head = h0 + grp, kvh = head / group;
        const float *q = qs + grp * HD;
        const uint16_t *kb = p.kc + (size_t)l * p.max_seq * kvrow + kvh * HD;
        const uint16_t *vb = p.vc + (size_t)l * p.max_seq * kvrow + kvh * HD;
        for (uint32_t t0 = wl * 32; t0 < seq; t0 += wpg * 32) {
            const uint32_t t = t0 + lane;
            const bool live = t < seq;
            const uint4 *kr = reinterpret_cast<const uint4 *>(kb + (size_t)(live ? t : 0) * kvrow);
            const uint4 *vr = reinterpret_cast<const uint4 *>(vb + (size_t)(live ? t : 0) * kvrow);
            float s = 0.0f;
#pragma unroll
            for (int h = 0; h < HD / 64; ++h) {
                uint4 kv4[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) kv4[i] = __ldcg(kr + 8 * h + i);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t wv[4] = {kv4[i].x, kv4[i].y, kv4[i].z, kv4[i].w};
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq)
                        s += q[64 * h + 8 * i + 2 * qq] * __uint_as_float(wv[qq] << 16) +
                             q[64 * h + 8 * i + 2 * qq + 1] * __uint_as_float(wv[qq] & 0xFFFF0000u);
                }
            }
            const float sh = live ? s : -INFINITY;
            const float mn = fmaxf(m, warp_max(sh));
            const float alpha = __expf(m - mn);
            const float pr = live ? __expf(sh - mn) : 0.0f;
            lsum = lsum * alpha + warp_sum(pr);
            m = mn;
#pragma unroll
            for (int cc = 0; cc < NC; ++cc) {
                uint4 vv4[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) vv4[i] = __ldcg(vr + 4 * cc + i);
                float pv[32];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t wv[4] = {vv4[i].x, vv4[i].y, vv4[i].z, vv4[i].w};
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq) {
                        pv[8 * i + 2 * qq] = pr * __uint_as_float(wv[qq] << 16);
                        pv[8 * i + 2 * qq + 1] = pr * __uint_as_float(wv[qq] & 0xFFFF0000u);
                    }
                }
                o[cc] = o[cc] * alpha + reduce_scatter32(pv, lane);
            }
        }
        float *ws = wst + warp * (HD + 2);
        if (lane == 0) {
            ws[0] = m;
            ws[1] = lsum;
        }
#pragma unroll
        for (int cc = 0; cc < NC; ++cc) ws[2 + 32 * cc + lane] = o[cc];
    }
    csync();
    float *ofl = reinterpret_cast<float *>(c.smem + c.L.ofl);  // [kMaxBHeads][HD]
    for (uint32_t i = tid; i < nh * HD; i += kConsumers) {
        const uint32_t gh = i / HD, d = i % HD, w0 = gh * wpg;
        float M = -INFINITY;
        for (uint32_t w = w0; w < w0 + wpg; ++w) M = fmaxf(M, wst[w * (HD + 2)]);
        float L = 0.0f, O = 0.0f;
        for (uint32_t w = w0; w < w0 + wpg; ++w) {
            const float mw = wst[w * (HD + 2)];
            const float f = (mw == -INFINITY) ? 0.0f : __expf(mw - M);
            L += wst[w * (HD + 2) + 1] * f;
            O += wst[w * (HD + 2) + 2 + d] * f;
        }
        ofl[i] = O / L;
    }
    csync();
    stage_small(ofl, nh * HD, reinterpret_cast<__half *>(c.smem + c.L.oh),
                reinterpret_cast<__half *>(c.smem + c.L.ol), reinterpret_cast<float *>(c.smem + c.L.opost));
    csync();
}

// B: fold the FFN delta of the previous layer into X (this CTA's slice), attend
// the heads of this CTA's O pairs, then add W_o[rows, head cols] . o_head into X.
__device__ void phase_attn_o(Ctx &c, const CtaSched &S, uint32_t l, uint32_t pos) {
    const Params &p = *c.p;
    {
        const uint32_t per = (p.dim + gridDim.x - 1) / gridDim.x;
        const uint32_t e0 = blockIdx.x * per, e1 = min(p.dim, e0 + per);
        for (uint32_t e = e0 + threadIdx.x; e < e1; e += kConsumers) {
            if (l > 0) red_add(&p.X[e], __ldcg(&p.Y[e]));
            p.Y[e] = 0.0f;
        }
    }
    if (S.b_p1 <= S.b_p0) return;
    const uint32_t h0 = S.b_p0 / p.o_tiles, h1 = (S.b_p1 - 1) / p.o_tiles;
    if (p.hd == 64) attend<64>(c, l, h0, h1 - h0 + 1, pos);
    else attend<128>(c, l, h0, h1 - h0 + 1, pos);
    const uint32_t nkb = p.hd / 32, prec = nkb * kBlockRec;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    for (uint32_t q0 = S.b_p0; q0 < S.b_p1; q0 += p.pairs_per_chunk) {
        const uint32_t n = min(p.pairs_per_chunk, S.b_p1 - q0);
        const uint8_t *chunk = chunk_acquire(c);
        for (uint32_t i = warp; i < n; i += kConsumerWarps) {
            const uint32_t pair = q0 + i, head = pair / p.o_tiles, rt = pair % p.o_tiles, hs = head - h0;
            const uint8_t *rec = chunk + (size_t)i * prec;
            float acc0 = 0.0f, acc1 = 0.0f;
            group_dot(rec, rec + nkb * 256, 0, nkb, reinterpret_cast<const __half *>(c.smem + c.L.oh) + hs * p.hd,
                      reinterpret_cast<const __half *>(c.smem + c.L.ol) + hs * p.hd,
                      reinterpret_cast<const float *>(c.smem + c.L.opost) + hs * nkb, acc0, acc1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
            if (t == 0) {
                red_add(&p.X[rt * 16 + g], acc0);
                red_add(&p.X[rt * 16 + g + 8], acc1);
            }
        }
        chunk_release(c);
    }
}

// C: RMSNorm + gate/up rows of this CTA's FFN units + SwiGLU, then the down
// projection restricted to those FFN indices, accumulated in shared memory and
// added into Y.  Unit u = (block b, half h) covers FFN 32b + 8t + 4h + i
// (t, i < 4); its two gate/up tiles p = 0, 1 hold rows for t = 2p, 2p+1, and
// s16[8p + r] = silu(gate_r) * up_r is laid out so mma lane t reads s16[4t..4t+3].
__device__ void phase_ffn(Ctx &c, const CtaSched &S, uint32_t l) {
    const Params &p = *c.p;
    const float rms = stage_norm<0>(c, p.X, nullptr, nullptr, p.ffn_norm + (size_t)l * p.dim, nullptr);
    float *yt = c.red + kRedYT;
    float *sv = c.red + kRedSV;  // 16 SwiGLU values of the current unit
    __half *s16h = reinterpret_cast<__half *>(c.smem + c.L.s16h);
    __half *s16l = reinterpret_cast<__half *>(c.smem + c.L.s16l);
    float *spost = reinterpret_cast<float *>(c.smem + c.L.spost);
    float *dacc = reinterpret_cast<float *>(c.smem + c.L.dacc);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    for (uint32_t e = tid; e < p.dim; e += kConsumers) dacc[e] = 0.0f;
    const uint32_t ntiles = p.dim / 16;
    for (uint32_t u = 0; u < S.n_c; ++u) {
        for (int pt = 0; pt < 2; ++pt) {
            const uint8_t *rec = chunk_acquire(c);
            tile_rows(c, rec, p.dim / 32, rms, yt);
            chunk_release(c);
            if (tid < 8) {
                const float gv = yt[tid], uv = yt[tid + 8];
                sv[8 * pt + tid] = gv / (1.0f + expf(-gv)) * uv;  // llama_run:248-250
            }
            csync();
        }
        if (warp == 0) {  // unit prescale over its 16 values
            const float x = lane < 16 ? sv[lane] : 0.0f;
            const float m = warp_max(fabsf(x));
            const int ex = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;
            int s = (m > 0.0f && ex < 128 && ex > -127) ? 14 - ex : 0;
            s = max(-126, min(126, s));
            const float xs = x * __uint_as_float((uint32_t)(s + 127) << 23);
            const __half h = __float2half_rn(xs);
            if (lane < 16) {
                s16h[u * 16 + lane] = h;
                s16l[u * 16 + lane] = __float2half_rn(xs - __half2float(h));
            }
            if (lane == 0) spost[u] = __uint_as_float((uint32_t)(127 - s) << 23);
        }
        csync();
        const uint8_t *drec = chunk_acquire(c);
        uint2 xs = make_uint2(0, 0);
        if (g < 2) xs = *reinterpret_cast<const uint2 *>(((g & 1) ? s16l : s16h) + u * 16 + 4 * t);
        const float post = spost[u];
        const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
        for (uint32_t r0 = warp; r0 < ntiles; r0 += 4 * kConsumerWarps) {
            uint32_t wv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {  // 4 independent row tiles in flight
                const uint32_t r = r0 + u * kConsumerWarps;
                wv[u] = r < ntiles ? *reinterpret_cast<const uint32_t *>(drec + (size_t)r * kHalfRec + lane * 4) : 0u;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t r = r0 + u * kConsumerWarps;
                if (r < ntiles) {  // warp-uniform
                    const uint8_t *rec = drec + (size_t)r * kHalfRec;
                    uint32_t a[4];
                    decode_word_f16(wv[u], a);
                    float d[4];
                    mma_f16_16816(d, a, xs.x, xs.y, zero4);
                    if (t == 0) {
                        dacc[r * 16 + g] += e8m0_to_f32(rec[128 + g]) * post * (d[0] + d[1]);
                        dacc[r * 16 + g + 8] += e8m0_to_f32(rec[128 + g + 8]) * post * (d[2] + d[3]);
                    }
                }
            }
        }
        chunk_release(c);
    }
    csync();
    if (S.n_c > 0)
        for (uint32_t e = tid; e < p.dim; e += kConsumers) red_add(&p.Y[e], dacc[e]);
}

// L: final RMSNorm + this CTA's lm_head rows -> logits + a per-CTA argmax candidate.
__device__ void phase_lm(Ctx &c, const CtaSched &S) {
    const Params &p = *c.p;
    const float rms = stage_norm<1>(c, p.X, p.Y, nullptr, p.final_norm, nullptr);
    float *yt = c.red + kRedYT;
    float bv = -1e30f;
    uint32_t bi = 0;
    for (uint32_t i = 0; i < S.n_l; ++i) {
        const uint8_t *rec = chunk_acquire(c);
        tile_rows(c, rec, p.dim / 32, rms, yt);
        chunk_release(c);
        const uint32_t row0 = S.l_tile[i] * 16;
        if (threadIdx.x < 32) {
            const int lane = threadIdx.x;
            const uint32_t row = row0 + lane;
            if (lane < 16 && row < p.vocab) p.logits[row] = yt[lane];
            // llama_run:283-292: larger value wins, ties to the lower index
            float wv = (lane < 16 && row < p.vocab) ? yt[lane] : -INFINITY;
            uint32_t wi = row;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, wv, o);
                const uint32_t oi = __shfl_xor_sync(0xffffffffu, wi, o);
                if (ov > wv || (ov == wv && oi < wi)) {
                    wv = ov;
                    wi = oi;
                }
            }
            if (wv > bv || (wv == bv && wi < bi)) {
                bv = wv;
                bi = wi;
            }
        }
        csync();
    }
    if (threadIdx.x == 0) {
        p.cand_val[blockIdx.x] = bv;
        p.cand_idx[blockIdx.x] = bi;
    }
}

__device__ void producer(const Params &p, const CtaSched &S, const uint32_t *cb, uint64_t *full, uint64_t *empty,
                         uint8_t *ring) {
    const int lane = threadIdx.x & 31;
    const uint8_t *stream = p.arena + S.stream_off;
    const uint64_t pol = policy_evict_first();
    uint32_t seq = 0;
    bool abort = false;
    // same token count as the consumers: never past the cache capacity
    const uint32_t pos0 = p.state[1];
    const uint32_t n_eff = pos0 < p.max_seq ? min(p.n_tokens, p.max_seq - pos0) : 0u;
    for (uint32_t tok = 0; tok < n_eff && !abort; ++tok) {
        size_t off = 0;
        for (uint32_t i = 0; i < S.n_chunks; ++i, ++seq) {
            const uint32_t slot = seq % p.n_slots, bytes = cb[i];
            if (seq >= p.n_slots) {
                const uint32_t parity = ((seq / p.n_slots) - 1) & 1;
                bool got = false;
                for (uint32_t it = 0; it < kSpinLimit && !got; ++it) {
                    got = mbar_try_wait(&empty[slot], parity);
                    if (!got && (it & 63) == 63 && ld_volatile(&p.bar[1])) break;
                }
                if (!got) {
                    abort = true;
                    break;
                }
            }
            // one bulk copy per chunk: per-op overhead makes several small copies
            // much slower than one large one (measured: 18 KB x 1 streams ~47 GB/s
            // per SM, 4 KB pieces ~12 GB/s)
            if (lane == 0) {
                pstamp(seq);
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_g2s_hint(ring + (size_t)slot * p.slot_bytes, stream + off, bytes, &full[slot], pol);
            }
            __syncwarp();
            off += bytes;
        }
    }
    if (abort) {
        // let every copy already issued land before the CTA's shared memory goes away
        const uint32_t issued = seq;
        for (uint32_t s = 0; s < p.n_slots && s < issued; ++s) {
            const uint32_t last = issued - 1 - ((issued - 1 - s) % p.n_slots);  // last seq that used slot s
            mbar_wait_bounded(&full[last % p.n_slots], (last / p.n_slots) & 1);
        }
    }
}

__global__ void __maxnreg__(96) decode_kernel(Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const Smem L = smem_layout(p);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *empty = full + kMaxSlots;
    uint8_t *ring = smem + L.ring;
    // stage the schedule and chunk-size table: per-chunk global loads would put an
    // L2 round trip on every producer issue and consumer step
    {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(&p.sched[blockIdx.x]);
        uint32_t *dst = reinterpret_cast<uint32_t *>(smem + L.sched);
        for (uint32_t i = threadIdx.x; i < sizeof(CtaSched) / 4; i += blockDim.x) dst[i] = src[i];
        const uint32_t *cb = p.chunk_bytes + (size_t)blockIdx.x * p.chunk_stride;
        uint32_t *cbs = reinterpret_cast<uint32_t *>(smem + L.cbytes);
        for (uint32_t i = threadIdx.x; i < p.chunk_stride; i += blockDim.x) cbs[i] = cb[i];
    }
    const CtaSched &S = *reinterpret_cast<const CtaSched *>(smem + L.sched);
    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < p.n_slots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        fence_mbar_init();
        reinterpret_cast<volatile uint32_t *>(smem + L.flag)[0] = 1;
        reinterpret_cast<volatile uint32_t *>(smem + L.flag)[1] = 0;
    }
    __syncthreads();
    if (threadIdx.x >= kConsumers) {
        producer(p, S, reinterpret_cast<const uint32_t *>(smem + L.cbytes), full, empty, ring);
        return;
    }
    Ctx c;
    c.p = &p, c.smem = smem, c.L = L, c.full = full, c.empty = empty, c.ring = ring;
    c.red = reinterpret_cast<float *>(smem + L.red);
    c.seq = 0, c.nbar = 0, c.ok = true;
    uint32_t tok = p.state[0], pos = p.state[1];
    const uint32_t n_prompt = p.state[3], cap = p.state[4];
    // never index the cache past its capacity (the host bounds positions too)
    const uint32_t n_eff = pos < p.max_seq ? min(p.n_tokens, p.max_seq - pos) : 0u;
    const uint32_t per_tok = 7 * p.n_layers + 3;
    for (uint32_t it = 0; it < n_eff; ++it) {
        const uint32_t sb = it * per_tok;
        for (uint32_t l = 0; l < p.n_layers; ++l) {
            stamp(sb + 7 * l);
            phase_qkv(c, S, l, tok, pos);
            stamp(sb + 7 * l + 1);
            if (!grid_barrier(c)) return;
            stamp(sb + 7 * l + 2);
            phase_attn_o(c, S, l, pos);
            stamp(sb + 7 * l + 3);
            if (!grid_barrier(c)) return;
            stamp(sb + 7 * l + 4);
            phase_ffn(c, S, l);
            stamp(sb + 7 * l + 5);
            if (!grid_barrier(c)) return;
            stamp(sb + 7 * l + 6);
        }
        stamp(sb + 7 * p.n_layers);
        phase_lm(c, S);
        stamp(sb + 7 * p.n_layers + 1);
        if (!grid_barrier(c)) return;
        stamp(sb + 7 * p.n_layers + 2);
        // every CTA reduces the candidates itself (same order -> same token)
        float *rv = c.red + kRedArg;
        uint32_t *ri = reinterpret_cast<uint32_t *>(c.red + kRedArg + 1);
        if (threadIdx.x < 32) {
            const int lane = threadIdx.x;
            float bv = -1e30f;
            uint32_t bi = 0;
            for (uint32_t i = lane; i < gridDim.x; i += 32) {
                const float v = __ldcg(&p.cand_val[i]);
                const uint32_t ix = __ldcg(&p.cand_idx[i]);
                if (v > bv || (v == bv && ix < bi)) bv = v, bi = ix;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
            }
            if (lane == 0) {
                rv[0] = bv;
                ri[0] = bi;
            }
        }
        csync();
        const uint32_t next = ri[0];
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            p.state[2] = next;
            if (pos + 1 >= n_prompt && pos + 1 - n_prompt < cap) p.out[pos + 1 - n_prompt] = next;
            p.state[0] = (pos + 1 < n_prompt) ? p.prompt[pos + 1] : next;
            p.state[1] = pos + 1;
        }
        tok = (pos + 1 < n_prompt) ? p.prompt[pos + 1] : next;
        pos += 1;
        csync();
    }
}

}  // namespace persist
}  // namespace fp4x

// ---------------------------------------------------------------- host side
namespace fp4x {
namespace persist {

struct Tensor {
    const uint8_t *w = nullptr, *s = nullptr;
    uint32_t n = 0, k = 0;
};

struct BuildIn {
    fp4x_llama_config cfg;
    std::vector<Tensor> qkv, o, gu, down;  // per layer, engine row orders
    Tensor lm;
    const float *attn_norm = nullptr, *ffn_norm = nullptr, *final_norm = nullptr;
    const uint16_t *embed = nullptr;
    const float *cos_t = nullptr, *sin_t = nullptr;
    uint16_t *kc = nullptr, *vc = nullptr;
    float *q = nullptr, *logits = nullptr;
    uint32_t *state = nullptr;
    const uint32_t *prompt = nullptr;
    uint32_t *out = nullptr;
};

struct Engine {
    Params p;
    int grid = 0;
    size_t smem = 0;
    size_t arena_bytes = 0;
    std::vector<void *> allocs;
};

// rows[16] of one tile + n_rt consecutive tiles (rows + 16 each) -> records at dst.
struct PackJobH {
    const uint8_t *w, *s;
    uint32_t K;
    int32_t rows[16];
    uint32_t n_rt, kb0, nkb;
    int32_t half;
    uint64_t dst;
};

__global__ void pack_jobs_kernel(const PackJobH *jobs, uint8_t *arena) {
    const PackJobH &J = jobs[blockIdx.x];
    const uint32_t rowbytes = J.K / 2, nbk = J.K / 32;
    const uint32_t recb = J.half < 0 ? J.nkb * kBlockRec : kHalfRec;
    for (uint32_t rt = 0; rt < J.n_rt; ++rt) {
        uint8_t *dst = arena + J.dst + (size_t)rt * recb;
        for (uint32_t i = threadIdx.x; i < recb; i += blockDim.x) {
            uint8_t v = 0;
            if (J.half < 0) {
                const uint32_t nib = J.nkb * 256;
                if (i < nib) {
                    const uint32_t b = i / 256, r = i % 256, lane = r / 8, h = (r % 8) / 4, j = r % 4;
                    const uint32_t g = lane / 4, t = lane % 4;
                    const int32_t row = J.rows[g + 8 * (j & 1)];
                    if (row >= 0)
                        v = J.w[(size_t)(row + 16 * rt) * rowbytes + (J.kb0 + b) * 16 + 4 * t + 2 * h + (j >> 1)];
                } else {
                    const uint32_t q = i - nib, b = q / 16, r = q % 16;
                    const int32_t row = J.rows[r];
                    if (row >= 0) v = J.s[(size_t)(row + 16 * rt) * nbk + J.kb0 + b];
                }
            } else {
                if (i < 128) {
                    const uint32_t lane = i / 4, j = i % 4, g = lane / 4, t = lane % 4;
                    const int32_t row = J.rows[g + 8 * (j & 1)];
                    if (row >= 0)
                        v = J.w[(size_t)(row + 16 * rt) * rowbytes + J.kb0 * 16 + 4 * t + 2 * J.half + (j >> 1)];
                } else {
                    const int32_t row = J.rows[i - 128];
                    if (row >= 0) v = J.s[(size_t)(row + 16 * rt) * nbk + J.kb0];
                }
            }
            dst[i] = v;
        }
    }
}

static int fail(const char *what, cudaError_t e) {
    set_error("persistent decode: %s: %s", what, cudaGetErrorString(e));
    return FP4X_ECUDA;
}

void destroy(Engine *e) {
    if (!e) return;
    for (void *q : e->allocs) cudaFree(q);
    delete e;
}

template <typename T>
static int dalloc(Engine *e, T **p, size_t count) {
    void *q = nullptr;
    cudaError_t err = cudaMalloc(&q, count * sizeof(T) + 16);
    if (err != cudaSuccess) {
        set_error("persistent decode: cudaMalloc(%zu): %s", count * sizeof(T), cudaGetErrorString(err));
        return FP4X_ENOMEM;
    }
    e->allocs.push_back(q);
    *p = static_cast<T *>(q);
    return FP4X_OK;
}

// Returns FP4X_EUNSUPPORTED (with a message) when the shape does not fit the
// kernel's static limits; the caller keeps the graph path then.
int build(const BuildIn &in, cudaStream_t st, Engine **out) {
    const fp4x_llama_config &c = in.cfg;
    const uint32_t hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
    int dev = 0, G = 0, coop = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&G, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    if (!coop || G <= 0) {
        set_error("persistent decode: cooperative launch unavailable");
        return FP4X_EUNSUPPORTED;
    }
    if (c.dim % 128 || c.ffn % 32 || (hd != 64 && hd != 128) || qd % 16 || kvd % 16 || c.dim > 8192) {
        set_error("persistent decode: unsupported shape");
        return FP4X_EUNSUPPORTED;
    }
    Params P = {};
    P.n_layers = c.n_layers, P.dim = c.dim, P.ffn = c.ffn, P.n_heads = c.n_heads, P.n_kv = c.n_kv_heads;
    P.hd = hd, P.vocab = c.vocab, P.max_seq = c.max_seq, P.eps = c.eps;
    P.q_tiles = qd / 16, P.k_tiles = kvd / 16, P.o_tiles = c.dim / 16;
    const uint32_t qkv_tiles = (qd + 2 * kvd) / 16, pairs = c.n_heads * P.o_tiles, units = c.ffn / 16;
    const uint32_t lm_tiles = (c.vocab + 15) / 16;
    const uint32_t T = c.dim / 32 * kBlockRec, PB = hd / 32 * kBlockRec, D = c.dim / 16 * kHalfRec;
    P.slot_bytes = std::max(std::max(T, D), PB);
    P.pairs_per_chunk = P.slot_bytes / PB;
    int max_smem = 0;
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    P.n_slots = 0;
    const uint32_t base = smem_layout(P).total;
    const uint32_t room = max_smem > (int)base + 256 ? (uint32_t)max_smem - base - 256 : 0;
    P.n_slots = std::min<uint32_t>(kMaxSlots, room / P.slot_bytes);
    if (P.n_slots < 3) {
        set_error("persistent decode: shared memory too small for the weight ring");
        return FP4X_EUNSUPPORTED;
    }
    // static schedule
    std::vector<CtaSched> S(G);
    for (auto &s : S) s = CtaSched{};
    for (uint32_t i = 0; i < qkv_tiles; ++i) {
        CtaSched &s = S[i % G];
        if (s.n_a >= (uint32_t)kMaxA) {
            set_error("persistent decode: too many QKV tiles per CTA");
            return FP4X_EUNSUPPORTED;
        }
        s.a_tile[s.n_a++] = i;
    }
    for (int g = 0; g < G; ++g) {
        S[g].b_p0 = (uint32_t)((uint64_t)pairs * g / G);
        S[g].b_p1 = (uint32_t)((uint64_t)pairs * (g + 1) / G);
        if (S[g].b_p1 > S[g].b_p0 &&
            (S[g].b_p1 - 1) / P.o_tiles - S[g].b_p0 / P.o_tiles + 1 > (uint32_t)kMaxBHeads) {
            set_error("persistent decode: a CTA spans too many attention heads");
            return FP4X_EUNSUPPORTED;
        }
    }
    for (uint32_t u = 0; u < units; ++u) {
        CtaSched &s = S[u % G];
        if (s.n_c >= (uint32_t)kMaxUnits) {
            set_error("persistent decode: too many FFN units per CTA");
            return FP4X_EUNSUPPORTED;
        }
        s.c_unit[s.n_c++] = u;
    }
    for (uint32_t i = 0; i < lm_tiles; ++i) {
        CtaSched &s = S[i % G];
        if (s.n_l >= (uint32_t)kMaxL) {
            set_error("persistent decode: too many lm_head tiles per CTA");
            return FP4X_EUNSUPPORTED;
        }
        s.l_tile[s.n_l++] = i;
    }
    // chunk streams + packing jobs, in consumption order
    std::vector<std::vector<uint32_t>> cbytes(G);
    std::vector<PackJobH> jobs;
    uint64_t off = 0;
    auto job = [&](const Tensor &t, const int32_t *rows, uint32_t n_rt, uint32_t kb0, uint32_t nkb, int32_t half,
                   uint64_t dst) {
        PackJobH j;
        j.w = t.w, j.s = t.s, j.K = t.k, j.n_rt = n_rt, j.kb0 = kb0, j.nkb = nkb, j.half = half, j.dst = dst;
        for (int r = 0; r < 16; ++r) j.rows[r] = rows[r];
        jobs.push_back(j);
    };
    int32_t rows[16];
    for (int g = 0; g < G; ++g) {
        CtaSched &s = S[g];
        s.stream_off = off;
        auto &cb = cbytes[g];
        for (uint32_t l = 0; l < c.n_layers; ++l) {
            for (uint32_t i = 0; i < s.n_a; ++i) {
                for (int r = 0; r < 16; ++r) rows[r] = (int32_t)(16 * s.a_tile[i] + r);
                job(in.qkv[l], rows, 1, 0, c.dim / 32, -1, off);
                cb.push_back(T), off += T;
            }
            for (uint32_t q0 = s.b_p0; q0 < s.b_p1; q0 += P.pairs_per_chunk) {
                const uint32_t n = std::min(P.pairs_per_chunk, s.b_p1 - q0);
                uint32_t i = 0;
                while (i < n) {  // runs of pairs of the same head: consecutive O row tiles
                    const uint32_t head = (q0 + i) / P.o_tiles;
                    uint32_t j = i;
                    while (j < n && (q0 + j) / P.o_tiles == head) ++j;
                    const uint32_t rt0 = (q0 + i) % P.o_tiles;
                    for (int r = 0; r < 16; ++r) rows[r] = (int32_t)(16 * rt0 + r);
                    job(in.o[l], rows, j - i, head * hd / 32, hd / 32, -1, off + (uint64_t)i * PB);
                    i = j;
                }
                cb.push_back(n * PB), off += (uint64_t)n * PB;
            }
            for (uint32_t ui = 0; ui < s.n_c; ++ui) {
                const uint32_t u = s.c_unit[ui], b = u / 2, h = u % 2;
                for (uint32_t pt = 0; pt < 2; ++pt) {
                    for (int r = 0; r < 16; ++r) {
                        const uint32_t rr = r % 8, f = 32 * b + 8 * (2 * pt + rr / 4) + 4 * h + rr % 4;
                        rows[r] = (int32_t)((f / 8) * 16 + f % 8 + (r >= 8 ? 8 : 0));
                    }
                    job(in.gu[l], rows, 1, 0, c.dim / 32, -1, off);
                    cb.push_back(T), off += T;
                }
                for (int r = 0; r < 16; ++r) rows[r] = r;
                job(in.down[l], rows, P.o_tiles, b, 1, (int32_t)h, off);
                cb.push_back(D), off += D;
            }
        }
        for (uint32_t i = 0; i < s.n_l; ++i) {
            for (int r = 0; r < 16; ++r) {
                const uint32_t row = 16 * s.l_tile[i] + r;
                rows[r] = row < c.vocab ? (int32_t)row : -1;
            }
            job(in.lm, rows, 1, 0, c.dim / 32, -1, off);
            cb.push_back(T), off += T;
        }
        s.n_chunks = (uint32_t)cb.size();
    }
    uint32_t stride = 0;
    for (auto &cb : cbytes) stride = std::max<uint32_t>(stride, (uint32_t)cb.size());
    std::vector<uint32_t> cbflat((size_t)G * stride, 0);
    for (int g = 0; g < G; ++g) std::copy(cbytes[g].begin(), cbytes[g].end(), cbflat.begin() + (size_t)g * stride);

    Engine *e = new Engine();
    int rc = FP4X_OK;
    uint8_t *arena = nullptr;
    uint32_t *dcb = nullptr, *bar = nullptr, *cidx = nullptr;
    CtaSched *dsched = nullptr;
    PackJobH *djobs = nullptr;
    float *X = nullptr, *Y = nullptr, *cval = nullptr;
    rc = dalloc(e, &arena, off);
    if (!rc) rc = dalloc(e, &dcb, cbflat.size());
    if (!rc) rc = dalloc(e, &dsched, (size_t)G);
    if (!rc) rc = dalloc(e, &bar, 4);
    if (!rc) rc = dalloc(e, &X, c.dim);
    if (!rc) rc = dalloc(e, &Y, c.dim);
    if (!rc) rc = dalloc(e, &cval, (size_t)G);
    if (!rc) rc = dalloc(e, &cidx, (size_t)G);
    if (!rc) rc = dalloc(e, &djobs, jobs.size());
    if (rc) {
        destroy(e);
        return rc;
    }
    cudaError_t err = cudaMemcpyAsync(dcb, cbflat.data(), cbflat.size() * 4, cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess)
        err = cudaMemcpyAsync(dsched, S.data(), S.size() * sizeof(CtaSched), cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess)
        err = cudaMemcpyAsync(djobs, jobs.data(), jobs.size() * sizeof(PackJobH), cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(Y, 0, c.dim * 4, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(bar, 0, 16, st);
    if (err == cudaSuccess) {
        for (size_t j0 = 0; j0 < jobs.size() && err == cudaSuccess; j0 += 65535) {
            const unsigned nj = (unsigned)std::min<size_t>(65535, jobs.size() - j0);
            pack_jobs_kernel<<<nj, 256, 0, st>>>(djobs + j0, arena);
            err = cudaGetLastError();
        }
    }
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);  // host vectors / job table go away
    if (err != cudaSuccess) {
        destroy(e);
        return fail("build", err);
    }
    cudaFree(djobs);
    e->allocs.pop_back();
    P.arena = arena, P.chunk_bytes = dcb, P.chunk_stride = stride, P.sched = dsched;
    P.attn_norm = in.attn_norm, P.ffn_norm = in.ffn_norm, P.final_norm = in.final_norm;
    P.embed = in.embed, P.cos_t = in.cos_t, P.sin_t = in.sin_t, P.kc = in.kc, P.vc = in.vc;
    P.X = X, P.Y = Y, P.q = in.q, P.logits = in.logits, P.cand_val = cval, P.cand_idx = cidx;
    P.state = in.state, P.prompt = in.prompt, P.out = in.out, P.bar = bar, P.n_tokens = 0;
    e->p = P;
    e->grid = G;
    e->smem = smem_layout(P).total;
    e->arena_bytes = off;
    err = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)e->smem);
    int per_sm = 0;
    if (err == cudaSuccess)
        err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel, kThreads, e->smem);
    if (err != cudaSuccess || per_sm < 1) {
        cudaFuncAttributes fa = {};
        cudaFuncGetAttributes(&fa, decode_kernel);
        const size_t smem = e->smem;
        destroy(e);
        if (err != cudaSuccess) return fail("occupancy", err);
        set_error("persistent decode: kernel does not fit one CTA per SM (%d threads, %d regs, %zu B dynamic + %zu B "
                  "static shared, max %d threads)",
                  kThreads, fa.numRegs, smem, fa.sharedSizeBytes, fa.maxThreadsPerBlock);
        return FP4X_EUNSUPPORTED;
    }
    *out = e;
    return FP4X_OK;
}

#ifdef FP4X_PHASE_TIMING
extern "C" FP4X_API int fp4x_phase_timestamps(unsigned long long *out, uint32_t n) {
    n = std::min<uint32_t>(n, kStamps);
    return cudaMemcpyFromSymbol(out, g_phase_ts, n * sizeof(unsigned long long)) == cudaSuccess ? 0 : 2;
}
#endif

int launch(Engine *e, cudaStream_t st, uint32_t n_tokens) {
    if (n_tokens == 0) return FP4X_OK;
    cudaError_t err = cudaMemsetAsync(e->p.bar, 0, 16, st);
    if (err != cudaSuccess) return fail("barrier reset", err);
    Params p = e->p;
    p.n_tokens = n_tokens;
    void *args[] = {&p};
    err = cudaLaunchCooperativeKernel((const void *)decode_kernel, dim3(e->grid), dim3(kThreads), args, e->smem, st);
    if (err != cudaSuccess) return fail("cooperative launch", err);
    return FP4X_OK;
}

}  // namespace persist
}  // namespace fp4x
