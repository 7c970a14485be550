// persist_tc.cu -- persistent MXFP4 decode kernel on the sm_100a tensor cores.
//
// Same job and phase structure as persist.cu (one cooperative launch runs whole
// generations, one CTA per SM, three grid-barrier phases per layer + lm_head;
// the reference's per-token loop is examples/llama_run/src/main.rs:492-587),
// but every linear layer runs on tcgen05.mma.kind::mxf4.block_scale:
//   * the weights are the MMA's A operand (128 rows); the batch-1 activation is
//     written as a sum of 8 MXFP4 terms that form the B operand's 8 columns
//     (N = 8), so the tensor core sums all terms at once and the epilogue adds
//     the 8 accumulator columns of a row: exact E2M1 x E2M1 products, fp32
//     accumulation, activation represented to ~1e-7 of its block maximum;
//   * warp 17 streams this CTA's pre-packed chunks through a shared-memory ring
//     with one cp.async.bulk per chunk (running ahead across phases, layers and
//     tokens); warp 16 allocates tensor memory and one lane of it copies scale
//     atoms into TMEM (tcgen05.cp) and issues the MMAs of each chunk as soon as
//     the chunk and the phase's activation are present; warps 0-15 build the
//     activation operands, read accumulators (tcgen05.ld) and run attention;
//   * per layer:  A  RMSNorm -> QKV (tile, k-range) units, partial sums added
//                    into a QKV vector (red.add);
//                 B  fold the FFN delta into the residual, RoPE + bf16 KV append
//                    for the attended KV heads, attention of this CTA's heads,
//                    O projection of their columns, added into the residual;
//                 C  RMSNorm -> gate/up rows of this CTA's FFN slice -> SwiGLU
//                    -> the down projection of those FFN indices, added into
//                    the FFN delta;
//     then final RMSNorm -> lm_head tiles -> per-CTA argmax candidates.
#include "common.cuh"
#include "persist_tc.cuh"
#include "tc05.cuh"

#include <algorithm>
#include <array>
#include <cstring>
#include <vector>

namespace fp4x {
namespace ptc {

constexpr uint32_t kBarLimit = 1u << 24;

// Timestamps (globaltimer, ns) of CTA 0 and the last CTA, only in builds
// compiled with -DFP4X_PHASE_TIMING; a no-op otherwise.  kTsPerLayer slots per
// layer (and the lm_head) per token: consumer steps 0..18, MMA lane 19..23,
// operand build split (decomposition done / fence done) 24..31, split-attention
// unit steps 32..34 (q staged, warp 0's positions done, warps merged), RMSNorm
// inputs loaded 35, normaliser known 36, K/V appended 37 (the last norm of a
// layer overwrites 35/36), split-attention warp 0's scores done 38 and softmax
// done 39 (its last tile).
constexpr uint32_t kTsPerLayer = 40;
#ifdef FP4X_PHASE_TIMING
constexpr uint32_t kTcStamps = 1u << 15;
__device__ unsigned long long g_tc_ts[2][kTcStamps];
__device__ __forceinline__ void tstamp(uint32_t i) {
    const int which = blockIdx.x == 0 ? 0 : (blockIdx.x == gridDim.x - 1 ? 1 : -1);
    if (which >= 0 && i < kTcStamps) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g_tc_ts[which][i] = t;
    }
}
// per-chunk MMA-lane times: [2 * chunk] full-wait done, [2 * chunk + 1] commit issued
constexpr uint32_t kMts = 1u << 16;
__device__ unsigned long long g_tc_mts[2][kMts];
__device__ __forceinline__ void mstamp(uint32_t i) {
    const int which = blockIdx.x == 0 ? 0 : (blockIdx.x == gridDim.x - 1 ? 1 : -1);
    if (which >= 0 && i < kMts) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g_tc_mts[which][i] = t;
    }
}
#else
__device__ __forceinline__ void tstamp(uint32_t) {}
__device__ __forceinline__ void mstamp(uint32_t) {}
#endif
#define CST(i)                                   \
    do {                                         \
        if (threadIdx.x == 0) tstamp(c.tsb + (i)); \
    } while (0)

struct Smem {
    uint32_t bars, flag, red, sched, xv, bx, sfbx, bo, sfbo, bh, sfbh, qs, wst, gu, ps, ring, total;
};

__host__ __device__ inline uint32_t attn_k(const Params &p) { return kMaxHeads * p.hd; }

__host__ __device__ inline Smem smem_layout(const Params &p) {
    Smem L;
    uint32_t off = 0;
    auto take = [&](uint32_t bytes, uint32_t align) {
        off = (off + align - 1) / align * align;
        const uint32_t o = off;
        off += bytes;
        return o;
    };
    L.bars = take((2 * kMaxSlots + 2 * PH_N + 1) * 8 + 16, 16);  // + TMEM base and abort words
    L.flag = take(16, 16);
    L.red = take(512 * 4, 16);
    L.sched = take(sizeof(Sched), 16);
    L.xv = take(p.dim * 4, 16);                      // f32 staging of the activation being decomposed
    L.bx = take(p.dim / 32 * 128, 128);              // 8 terms x dim: [k/32][8 rows][16 B]
    L.sfbx = take((p.dim / 128 + 3) * 128, 128);     // 128-byte scale atoms (+3: copy window)
    L.bo = take(attn_k(p) / 32 * 128, 128);
    L.sfbo = take((attn_k(p) / 128 + 1 + 3) * 128, 128);
    L.bh = take(5 * 128, 128);                       // U <= 128: 4 k32 columns, then a zero column
    L.sfbh = take((2 + 3) * 128, 128);
    L.qs = take(kMaxGroup * (p.hd + p.hd / 8) * 4, 16);  // split attention pads 4 floats per 32 dims
    L.wst = take(kCW * (p.hd + 2) * 4, 16);
    L.gu = take(256 * 4, 16);
    L.ps = take(kCW * kMaxGroup * 32 * 4, 16);  // split attention: per-warp probabilities
    L.ring = take(p.ring_bytes, 1024);
    L.total = off + 4096;  // MMA windows of partial tiles read up to 2 KB past a chunk
    return L;
}

// barrier area: full[kMaxSlots] empty[kMaxSlots] bready[PH_N] accr[PH_N] fin, tmem base, abort
struct Bars {
    uint64_t *full, *empty, *bready, *accr, *fin;
    uint32_t *tmem;
    volatile uint32_t *abort;
};

__device__ __forceinline__ Bars bars_of(uint8_t *smem, const Smem &L) {
    Bars B;
    uint64_t *b = reinterpret_cast<uint64_t *>(smem + L.bars);
    B.full = b;
    B.empty = b + kMaxSlots;
    B.bready = b + 2 * kMaxSlots;
    B.accr = B.bready + PH_N;
    B.fin = B.accr + PH_N;
    B.tmem = reinterpret_cast<uint32_t *>(B.fin + 1);
    B.abort = B.tmem + 1;
    return B;
}

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kCons) : "memory"); }

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
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t *p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded mbarrier wait that also gives up when the launch has aborted.
__device__ bool wait_bar(uint64_t *bar, uint32_t parity, const Params &p, volatile uint32_t *abort) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15) == 15 && (*abort || ld_volatile(&p.bar[1]))) return false;
    }
    *abort = 1;
    atomicExch(&p.bar[1], 1u);
    raise_device_error(DEVERR_MBAR_TIMEOUT);
    return false;
}

// ---------------------------------------------------------------- consumer context
struct Ctx {
    const Params *p;
    const Sched *S;
    uint8_t *smem;
    Smem L;
    Bars B;
    uint32_t tbase;
    float *red;
    uint32_t nbar;
    uint32_t tsb;  // timestamp slot base of the current layer
    uint32_t epoch0;  // cross-rank barrier epochs before this launch
    uint32_t xn;      // row-parallel exchanges of each kind done (tensor parallel)
    bool ok;
};

// All consumer threads call this; a failed wait earlier only marks the context,
// so the decision to stop is CTA-uniform here.  With `cross` (and more than one
// rank) the barrier spans every rank's grid; otherwise it is this GPU's grid.
__device__ bool grid_barrier(Ctx &c, bool cross = false) {
    const Params &p = *c.p;
    const bool xrank = cross && p.tp_size > 1;
    volatile uint32_t *flag = reinterpret_cast<volatile uint32_t *>(c.smem + c.L.flag);
    if (!c.ok) flag[1] = 1;
    csync();
    c.nbar += 1;
    if (threadIdx.x == 0) {
        if (flag[1]) atomicExch(&p.bar[1], 1u);
        if (xrank) {
            __threadfence_system();  // this CTA's writes into peer memory are visible before it arrives
            atomicAdd(&p.bar[0], 1u);
        } else {
            // release: the CTA's writes (ordered before this thread by the CTA barrier)
            // are visible before the arrival; one instruction instead of fence + add
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&p.bar[0]) : "memory");
        }
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
            __nanosleep(32);
        }
        if (ok && xrank) {
            // cross-rank step: CTA 0 tells every rank this rank's grid arrived, waits for
            // all ranks, then releases its own CTAs; epochs keep increasing across launches
            const uint32_t ep = c.epoch0 + c.nbar;
            const uint32_t lim = flag_wait_limit(kBarLimit);
            if (blockIdx.x == 0) {
                __threadfence_system();
                for (uint32_t r = 0; r < p.tp_size; ++r) st_release_sys(p.flagr[r] + 32 * p.tp_rank, ep);
                for (uint32_t src = 0; src < p.tp_size && ok; ++src)
                    for (uint32_t i = 0; ld_acquire_sys(p.flagr[p.tp_rank] + 32 * src) < ep; ++i)
                        if (i > lim || ld_volatile(&p.bar[1])) {
                            raise_device_error(DEVERR_FLAG_TIMEOUT);
                            ok = 0;
                            break;
                        }
                if (!ok) atomicExch(&p.bar[1], 1u);
                st_release_gpu(&p.bar[2], ok ? ep : 0xFFFFFFFFu);
            } else {
                for (uint32_t i = 0; ld_acquire(&p.bar[2]) < ep; ++i) {
                    if (ld_volatile(&p.bar[1]) || i > lim) {
                        if (i > lim) raise_device_error(DEVERR_FLAG_TIMEOUT);
                        ok = 0;
                        break;
                    }
                    __nanosleep(32);
                }
            }
        }
        // one GPU: the acquire load above already orders this CTA's later reads (the
        // CTA barrier below passes that on); the cross-rank path keeps its fence
        if (xrank) __threadfence();
        flag[0] = ok;
        if (!ok) *c.B.abort = 1;
    }
    csync();
    c.ok = flag[0] != 0;
    return c.ok;
}

// Row-parallel reduction under tensor parallelism (kind 0: the O-projection
// partials in tpo, 1: the down-projection partials in tpd), added into X.  CTA i
// owns slice i of the vector on every rank: each of its threads pushes one
// element of this rank's partial into every peer's receive slot as a 64-bit word
// {value, tag} (a single-copy-atomic store over NVLink, tag = n + 1), clears the
// element of the partial, then polls its own slots until every peer's word carries
// the tag and adds the ranks' values in rank order (the same bits on every rank).
// The tag makes each word self-validating, so no fence or flag orders the data.
// `n` numbers the exchanges of a kind (slot parity n & 1: a rank reaches exchange
// n + 2 of a kind only after every rank has finished exchange n, through the
// exchanges in between); a local grid barrier must follow before X is read.
// llama_run/src/main.rs:522-530 with the contraction split across ranks.
__device__ bool tp_exchange(Ctx &c, uint32_t kind, uint32_t n) {
    const Params &p = *c.p;
    const uint32_t T = p.tp_size, me = p.tp_rank, dim = p.dim, par = n & 1u, tag = n + 1;
    const uint32_t per = ((dim + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
    const uint32_t e0 = min(dim, blockIdx.x * per), e1 = min(dim, e0 + per);
    float *part = kind ? p.tpd : p.tpo;
    volatile uint32_t *flag = reinterpret_cast<volatile uint32_t *>(c.smem + c.L.flag);
    float own[2] = {0.f, 0.f};  // per <= 2 * kCons: dim <= 2 * kCons * grid
#pragma unroll
    for (uint32_t u = 0; u < 2; ++u) {
        const uint32_t i = e0 + threadIdx.x + u * kCons;
        if (i < e1) {
            own[u] = __ldcg(part + i);
            part[i] = 0.0f;
            const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(own[u]);
            for (uint32_t r = 0; r < T; ++r)
                if (r != me) {
                    uint64_t *dst = (kind ? p.trd[r] : p.tro[r]) + ((size_t)par * kMaxTp + me) * dim + i;
                    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(dst), "l"(w) : "memory");
                }
        }
    }
    const uint64_t *recv = kind ? p.trd[me] : p.tro[me];
    const uint32_t lim = flag_wait_limit(kBarLimit);
    bool ok = c.ok;
#pragma unroll
    for (uint32_t u = 0; u < 2; ++u) {
        const uint32_t i = e0 + threadIdx.x + u * kCons;
        if (i >= e1 || !ok) continue;
        // every peer's word is loaded at once; the ones without the tag are polled again
        uint64_t w[kMaxTp] = {};
        uint32_t pending = ((1u << T) - 1u) & ~(1u << me);
        for (uint32_t it = 0; pending; ++it) {
#pragma unroll
            for (uint32_t r = 0; r < kMaxTp; ++r)
                if ((pending >> r) & 1u)
                    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];"
                                 : "=l"(w[r])
                                 : "l"(recv + ((size_t)par * kMaxTp + r) * dim + i)
                                 : "memory");
#pragma unroll
            for (uint32_t r = 0; r < kMaxTp; ++r)
                if (((pending >> r) & 1u) && (uint32_t)(w[r] >> 32) == tag) pending &= ~(1u << r);
            if (pending && (((it & 63) == 63 && ld_volatile(&p.bar[1])) || it > lim)) {
                if (it > lim) {
                    raise_device_error(DEVERR_FLAG_TIMEOUT);
                    atomicExch(&p.bar[1], 1u);
                }
                ok = false;
                break;
            }
        }
        if (!ok) continue;
        float acc = 0.0f;
#pragma unroll
        for (uint32_t r = 0; r < kMaxTp; ++r)
            if (r < T) acc += r == me ? own[u] : __uint_as_float((uint32_t)w[r]);
        p.X[i] = __ldcg(p.X + i) + acc;  // this CTA alone writes its slice
    }
    if (threadIdx.x == 0) flag[2] = 1;
    csync();
    if (!ok) flag[2] = 0;
    csync();
    c.ok = flag[2] != 0;
    if (!c.ok && threadIdx.x == 0) *c.B.abort = 1;
    return c.ok;
}

// Consumers wait for the phase's accumulators (all threads poll; uniform result).
__device__ void wait_acc(Ctx &c, int ph, uint32_t parity) {
    if (c.ok && !wait_bar(&c.B.accr[ph], parity, *c.p, c.B.abort)) c.ok = false;
    tc::fence_after_sync();
}

// Activation operand ready: generic-proxy writes -> async proxy, then one arrive.
__device__ void signal_operand(Ctx &c, int ph) {
#ifdef FP4X_PHASE_TIMING
    csync();
    CST(24 + 2 * (ph == PH_LM ? 0 : ph));
#endif
    fence_proxy_async_smem();
#ifdef FP4X_PHASE_TIMING
    CST(25 + 2 * (ph == PH_LM ? 0 : ph));
#endif
    csync();
    if (threadIdx.x == 0) mbar_arrive(&c.B.bready[ph]);
}

// Sum of the 8 term columns of accumulator column `col` for row
// 32*(warp%4) + lane (smallest terms first).
__device__ __forceinline__ float acc_row(uint32_t tbase, uint32_t col) {
    const uint32_t warp = threadIdx.x >> 5;
    float v[8];
    tc::tmem_ld_x8(tbase + ((32u * (warp & 3u)) << 16) + col, v);
    tc::tmem_wait_ld();
    float s = v[7];
#pragma unroll
    for (int i = 6; i >= 0; --i) s += v[i];
    return s;
}

// Eight E2M1 values -> one packed word (low nibble = lower k), round to nearest
// even, saturating; cvt takes (upper, lower) pairs.
__device__ __forceinline__ uint32_t pack_e2m1x8(const float (&y)[8]) {
    uint32_t w;
    asm("{\n\t.reg .b8 q0, q1, q2, q3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q0, %2, %1;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q1, %4, %3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q2, %6, %5;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 q3, %8, %7;\n\t"
        "mov.b32 %0, {q0, q1, q2, q3};\n\t}"
        : "=r"(w)
        : "f"(y[0]), "f"(y[1]), "f"(y[2]), "f"(y[3]), "f"(y[4]), "f"(y[5]), "f"(y[6]), "f"(y[7]));
    return w;
}

// 8-term MXFP4 decomposition (operand rows 0..7 of B, [K/32][8][16 B], low nibble
// = lower k) of the 8 values x[] that this thread owns: word w (0..3) of 32-block b.
// The 4 threads of a block must sit in adjacent lanes (4b'..4b'+3 of the warp) and
// every lane of the warp must call (valid = false for padding lanes).  Scales go to
// sfb in 128-byte atoms (row t at 16t): block b at atom b/4 byte b%4 (natural), or
// at atom b/2 bytes 2(b%2), 2(b%2)+1 (pairs, for K32 blocks).
// Scale schedule per block with maximum a: e1 = the smallest exponent with
// a <= 6 * 2^e1, then e1 - 2, then 3 less per term.  Rounding to nearest keeps the
// residual after term 1 within 2^e1 and after each later term within half its
// scale, so every term stays inside +-6 and the 8-term sum equals the input to
// 2^(e1-21) (~1.6e-7 of the block maximum); every step is exact in fp32.
// Exponent of term t of a block whose first-term exponent is e1.
__device__ __forceinline__ int term_exp(int e1, int t) { return max(-126, min(125, t == 0 ? e1 : e1 + 1 - 3 * t)); }

// The terms themselves: words[t] = the 8 E2M1 codes of term t for x[] (x is
// consumed); returns e1.  The block maximum is taken over lanes l, l^1, l^2.
__device__ __forceinline__ int term_words8(float (&x)[8], uint32_t (&words)[8]) {
    float a = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) a = fmaxf(a, fabsf(x[j]));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    const uint32_t bits = __float_as_uint(a);
    int e1 = (int)((bits >> 23) & 0xFFu) - 127;
    e1 = (bits & 0x7FFFFFu) <= 0x400000u ? e1 - 2 : e1 - 1;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const int e = term_exp(e1, t);
        const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
        const float s = __uint_as_float((uint32_t)(127 + e) << 23);
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = x[j] * inv;
        words[t] = pack_e2m1x8(y);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t hv = e2m1x2_to_f16x2((words[t] >> (8 * j)) & 0xFFu);
            const __half2 q = *reinterpret_cast<const __half2 *>(&hv);
            x[2 * j] = fmaf(-__low2float(q), s, x[2 * j]);
            x[2 * j + 1] = fmaf(-__high2float(q), s, x[2 * j + 1]);
        }
    }
    return e1;
}

// The same 8-term decomposition with one value per lane (warp w: 32-blocks w,
// w + kCW, ...; same arithmetic per value as term_words8, so the same bits), for
// short vectors: the serial term chain per thread is 8x shorter and 8x more
// threads share the work.  Nibbles are gathered into words by three xor-shuffles
// within each 8-lane group.
__device__ void decompose_lanes(const float *v, uint32_t K, uint8_t *B, uint8_t *sfb, bool pairs) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (uint32_t b = warp; b < K / 32; b += kCW) {
        float x = v[b * 32 + lane];
        const float a = warp_max(fabsf(x));
        const uint32_t bits = __float_as_uint(a);
        int e1 = (int)((bits >> 23) & 0xFFu) - 127;
        e1 = (bits & 0x7FFFFFu) <= 0x400000u ? e1 - 2 : e1 - 1;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const int e = term_exp(e1, t);
            const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
            const float s = __uint_as_float((uint32_t)(127 + e) << 23);
            uint32_t code, hv;  // the code (low nibble; upper nibble 0) and its value as f16x2
            asm("{\n\t.reg .b8 q0;\n\t"
                "cvt.rn.satfinite.e2m1x2.f32 q0, %3, %2;\n\t"
                "cvt.u32.u8 %0, q0;\n\t"
                "cvt.rn.f16x2.e2m1x2 %1, q0;\n\t}"
                : "=r"(code), "=r"(hv)
                : "f"(x * inv), "f"(0.0f));
            const __half2 q = *reinterpret_cast<const __half2 *>(&hv);
            x = fmaf(-__low2float(q), s, x);
            uint32_t part = (code & 0xFu) << (4 * (lane & 7));
            part |= __shfl_xor_sync(0xffffffffu, part, 1);
            part |= __shfl_xor_sync(0xffffffffu, part, 2);
            part |= __shfl_xor_sync(0xffffffffu, part, 4);
            if ((lane & 7) == 0) *reinterpret_cast<uint32_t *>(B + b * 128 + t * 16 + (lane >> 3) * 4) = part;
        }
        if (lane < 8) {
            const uint8_t sb = (uint8_t)(term_exp(e1, (int)lane) + 127);
            if (!pairs) {
                sfb[(b >> 2) * 128 + lane * 16 + (b & 3)] = sb;
            } else {
                uint8_t *q2 = sfb + (b >> 1) * 128 + lane * 16 + 2 * (b & 1);
                q2[0] = sb;
                q2[1] = sb;
            }
        }
    }
}

// Half-word form: 4 values per thread (thread j of a 32-block owns values
// [4j, 4j + 4): the 8 threads of a block in adjacent lanes, j even = low half of
// word j / 2).  Same arithmetic per value as term_words8 (same bits); the term
// chain is half as long and twice as many threads share the vector.
__device__ __forceinline__ void decompose_half8(float (&x)[4], uint32_t b, uint32_t j, bool valid, uint8_t *B,
                                                uint8_t *sfb) {
    float a = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
    const uint32_t bits = __float_as_uint(a);
    int e1 = (int)((bits >> 23) & 0xFFu) - 127;
    e1 = (bits & 0x7FFFFFu) <= 0x400000u ? e1 - 2 : e1 - 1;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const int e = term_exp(e1, t);
        const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
        const float s = __uint_as_float((uint32_t)(127 + e) << 23);
        // the 4 codes (low 16 bits of h) and their values as two f16x2, from the
        // byte registers the encode leaves (no re-extraction of the bytes)
        uint32_t h, hvs[2];
        asm("{\n\t.reg .b8 q0, q1;\n\t.reg .b16 c;\n\t"
            "cvt.rn.satfinite.e2m1x2.f32 q0, %4, %3;\n\t"
            "cvt.rn.satfinite.e2m1x2.f32 q1, %6, %5;\n\t"
            "mov.b16 c, {q0, q1};\n\t"
            "cvt.u32.u16 %0, c;\n\t"
            "cvt.rn.f16x2.e2m1x2 %1, q0;\n\t"
            "cvt.rn.f16x2.e2m1x2 %2, q1;\n\t}"
            : "=r"(h), "=r"(hvs[0]), "=r"(hvs[1])
            : "f"(x[0] * inv), "f"(x[1] * inv), "f"(x[2] * inv), "f"(x[3] * inv));
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const uint32_t hv = hvs[q];
            const __half2 d = *reinterpret_cast<const __half2 *>(&hv);
            x[2 * q] = fmaf(-__low2float(d), s, x[2 * q]);
            x[2 * q + 1] = fmaf(-__high2float(d), s, x[2 * q + 1]);
        }
        const uint32_t other = __shfl_xor_sync(0xffffffffu, h, 1);
        if (valid && (j & 1) == 0) *reinterpret_cast<uint32_t *>(B + b * 128 + t * 16 + (j >> 1) * 4) = h | (other << 16);
    }
    if (valid && j == 0)
#pragma unroll
        for (int t = 0; t < 8; ++t) sfb[(b >> 2) * 128 + t * 16 + (b & 3)] = (uint8_t)(term_exp(e1, t) + 127);
}

// RMSNorm + decomposition in registers: thread i owns values [4i, 4i+4) (and
// [4(i+kCons), ...) when dim > 4 * kCons).  xn = (src * rms) * w
// (llama_run:79-116), src = X (MODE 0), X + Y (1) or the bf16 embedding row (2;
// CTA 0 writes it to X).  With `decompose` false only the CTA-0 embedding copy runs.
template <int MODE>
__device__ void norm_decompose(Ctx &c, const uint16_t *erow, const float *w, bool decompose) {
    const Params &p = *c.p;
    const uint32_t nw = p.dim / 8, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (!decompose) {
        if (MODE == 2 && blockIdx.x == 0)
            for (uint32_t i = threadIdx.x; i < nw; i += kCons) {
                const uint4 q = *reinterpret_cast<const uint4 *>(erow + 8 * i);
                const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    *reinterpret_cast<float2 *>(p.X + 8 * i + 2 * j) =
                        make_float2(__uint_as_float(u[j] << 16), __uint_as_float(u[j] & 0xFFFF0000u));
            }
        return;
    }
    // thread i owns the 4-value groups i, i + kCons, ... (values [4g, 4g + 4))
    constexpr int R4 = 4;  // dim <= 16 * kCons
    const uint32_t ng = p.dim / 4;
    float x[R4][4], g[R4][4];
    float ss = 0.0f;
#pragma unroll
    for (int r = 0; r < R4; ++r) {
        const uint32_t i = threadIdx.x + r * kCons;
#pragma unroll
        for (int j = 0; j < 4; ++j) x[r][j] = 0.0f, g[r][j] = 0.0f;
        if (i < ng) {
            float4 v;
            if (MODE == 2) {
                const uint2 q = *reinterpret_cast<const uint2 *>(erow + 4 * i);
                v = make_float4(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xFFFF0000u),
                                __uint_as_float(q.y << 16), __uint_as_float(q.y & 0xFFFF0000u));
                if (blockIdx.x == 0) *reinterpret_cast<float4 *>(p.X + 4 * i) = v;
            } else {
                v = __ldcg(reinterpret_cast<const float4 *>(p.X + 4 * i));
                if (MODE == 1) {
                    const float4 y = __ldcg(reinterpret_cast<const float4 *>(p.Y + 4 * i));
                    v.x += y.x, v.y += y.y, v.z += y.z, v.w += y.w;
                }
            }
            const float4 gw = __ldg(reinterpret_cast<const float4 *>(w + 4 * i));
            x[r][0] = v.x, x[r][1] = v.y, x[r][2] = v.z, x[r][3] = v.w;
            g[r][0] = gw.x, g[r][1] = gw.y, g[r][2] = gw.z, g[r][3] = gw.w;
#pragma unroll
            for (int j = 0; j < 4; ++j) ss += x[r][j] * x[r][j];
        }
    }
    CST(35);
    ss = warp_sum(ss);
    if (lane == 0) c.red[warp] = ss;
    csync();
    CST(36);
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < kCW; ++i) tot += c.red[i];
    const float rms = 1.0f / sqrtf(tot / (float)p.dim + p.eps);
    uint8_t *B = c.smem + c.L.bx, *sfb = c.smem + c.L.sfbx;
#pragma unroll
    for (int r = 0; r < R4; ++r) {
        const uint32_t i = threadIdx.x + r * kCons;
        if (i - lane >= ng) break;  // warp-uniform
        const bool valid = i < ng;
#pragma unroll
        for (int j = 0; j < 4; ++j) x[r][j] = x[r][j] * rms * g[r][j];
        decompose_half8(x[r], i >> 3, i & 7, valid, B, sfb);
    }
}

// Split attention, issued during layer l's QKV phase: L2 prefetch of the K and V
// rows (positions before pos) that this CTA's attention unit reads after the QKV
// barrier, so the unit's loads meet L2 instead of HBM.  One bulk prefetch per
// cached row (a KV head's HD bf16 values; rows of one head are n_kv * HD apart),
// spread over the consumer threads.
__device__ void prefetch_unit_kv(Ctx &c, uint32_t l, uint32_t pos) {
    const Params &p = *c.p;
    const uint32_t slices = p.attn_slices, u = blockIdx.x;
    if (u >= p.n_kv * slices) return;
    const uint32_t g = u / slices, sl = u % slices, seq = pos + 1;
    const uint32_t len = (seq + slices - 1) / slices, t_begin = min(seq, sl * len), t_end = min(pos, t_begin + len);
    if (t_begin >= t_end) return;
    const size_t base = (size_t)l * p.max_seq * p.kvd + (size_t)g * p.hd;
    const uint32_t n = t_end - t_begin, bytes = p.hd * 2;
    for (uint32_t i = threadIdx.x; i < 2 * n; i += kCons) {
        const uint16_t *src = (i < n ? p.kc : p.vc) + base + (size_t)(t_begin + (i < n ? i : i - n)) * p.kvd;
        prefetch_l2_bulk(src, bytes);
    }
}

// ---------------------------------------------------------------- phases

// A: normed input -> 8 terms -> QKV unit MMAs -> partial row sums into p.qkv.
// With kv_pos >= 0 (split attention this layer) the CTA's attention-unit K/V rows
// are prefetched into L2 while the QKV MMAs run.
__device__ void phase_qkv(Ctx &c, uint32_t l, uint32_t tok, uint32_t lay_count, int kv_pos) {
    const Params &p = *c.p;
    const Sched &S = *c.S;
    if (l == 0)
        norm_decompose<2>(c, p.embed + (size_t)tok * p.dim, p.attn_norm, S.n_a > 0);
    else if (p.tp_size > 1)  // the exchanges have already added every partial into X
        norm_decompose<0>(c, nullptr, p.attn_norm + (size_t)l * p.dim, S.n_a > 0);
    else
        norm_decompose<1>(c, nullptr, p.attn_norm + (size_t)l * p.dim, S.n_a > 0);
    CST(1);
    if (S.n_a > 0) signal_operand(c, PH_QKV);
    if (kv_pos >= 0) prefetch_unit_kv(c, l, (uint32_t)kv_pos);
    if (S.n_a == 0) return;
    CST(2);
    wait_acc(c, PH_QKV, lay_count & 1);
    CST(3);
    if (!c.ok) return;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, rows = p.qd + 2 * p.kvd;
    for (uint32_t u = warp >> 2; u < S.n_a; u += kCW / 4) {
        const float s = acc_row(c.tbase, 8 * u);
        const uint32_t row = S.a_tile[u] * 128 + 32 * (warp & 3) + lane;
        if (row < rows) red_add(&p.qkv[row], s);
    }
    CST(4);
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

__device__ __forceinline__ float reduce_scatter32(float (&v)[32], int lane) {
    rs_step<32, 32, 16>(v, lane);
    rs_step<32, 16, 8>(v, lane);
    rs_step<32, 8, 4>(v, lane);
    rs_step<32, 4, 2>(v, lane);
    rs_step<32, 2, 1>(v, lane);
    return v[0];
}

// RoPE'd, bf16-rounded K and bf16 V of KV head g at `pos` from the QKV sums into
// the cache (every CTA attending g writes the same bytes), then q of the
// attended heads (RoPE'd, pre-scaled) into qs.  llama_run:118-138 semantics.
template <int HD>
__device__ void stage_qkv(Ctx &c, uint32_t l, uint32_t pos) {
    const Params &p = *c.p;
    const Sched &S = *c.S;
    constexpr uint32_t half = HD / 2;
    const uint32_t group = p.n_heads / p.n_kv, g0 = S.h0 / group, g1 = (S.h0 + S.nh - 1) / group;
    const float *cs = p.cos_t + (size_t)pos * half, *sn = p.sin_t + (size_t)pos * half;
    uint16_t *kc = p.kc + ((size_t)l * p.max_seq + pos) * p.kvd, *vc = p.vc + ((size_t)l * p.max_seq + pos) * p.kvd;
    for (uint32_t i = threadIdx.x; i < (g1 - g0 + 1) * half; i += kCons) {
        const uint32_t g = g0 + i / half, j = i % half;
        const float *kr = p.qkv + p.qd + g * HD;
        const float k0 = __ldcg(kr + j), k1 = __ldcg(kr + j + half);
        kc[g * HD + j] = f32_to_bf16_bits(__fsub_rn(__fmul_rn(k0, cs[j]), __fmul_rn(k1, sn[j])));
        kc[g * HD + j + half] = f32_to_bf16_bits(__fadd_rn(__fmul_rn(k1, cs[j]), __fmul_rn(k0, sn[j])));
        const float *vr = p.qkv + p.qd + p.kvd + g * HD;
        vc[g * HD + j] = f32_to_bf16_bits(__ldcg(vr + j));
        vc[g * HD + j + half] = f32_to_bf16_bits(__ldcg(vr + j + half));
    }
    CST(37);
    float *qs = reinterpret_cast<float *>(c.smem + c.L.qs);
    const float scale = 1.0f / sqrtf((float)HD);
    for (uint32_t i = threadIdx.x; i < S.nh * half; i += kCons) {
        const uint32_t hs = i / half, j = i % half;
        const float *qr = p.qkv + (S.h0 + hs) * HD;
        const float q0 = __ldcg(qr + j), q1 = __ldcg(qr + j + half);
        qs[hs * HD + j] = __fsub_rn(__fmul_rn(q0, cs[j]), __fmul_rn(q1, sn[j])) * scale;
        qs[hs * HD + j + half] = __fadd_rn(__fmul_rn(q1, cs[j]), __fmul_rn(q0, sn[j])) * scale;
    }
    csync();
}

// Attention of heads h0 .. h0+nh-1 over positions 0..pos (llama_run:148-242,
// 1/sqrt(hd) scale folded into q): heads in parallel on groups of warps, each
// warp an online softmax over 32-token tiles (lane = token for Q.K and P.V, the
// P.V sums reduce-scattered so lane L keeps dims 32c + L); the group is merged
// into xv[head slot][HD] (f32).
template <int HD>
__device__ void attend(Ctx &c, uint32_t l, uint32_t pos) {
    const Params &p = *c.p;
    const Sched &S = *c.S;
    constexpr int NC = HD / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, tid = threadIdx.x;
    const uint32_t nh = S.nh;
    const uint32_t wpg = nh <= 1 ? kCW : (nh == 2 ? kCW / 2 : kCW / 4);
    const uint32_t grp = warp / wpg, wl = warp % wpg;
    const float *qs = reinterpret_cast<const float *>(c.smem + c.L.qs);
    float *wst = reinterpret_cast<float *>(c.smem + c.L.wst);
    const uint32_t kvrow = p.kvd, seq = pos + 1, group = p.n_heads / p.n_kv;
    float m = -INFINITY, lsum = 0.0f, o[NC];
#pragma unroll
    for (int i = 0; i < NC; ++i) o[i] = 0.0f;
    if (grp < nh) {
        const uint32_t head = S.h0 + grp, kvh = head / group;
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
    float *xv = reinterpret_cast<float *>(c.smem + c.L.xv);
    // warps past the last position of the sequence hold nothing (m = -inf)
    const uint32_t act = min(wpg, (seq + 31) / 32);
    for (uint32_t i = tid; i < nh * HD; i += kCons) {
        const uint32_t gh = i / HD, d = i % HD, w0 = gh * wpg;
        float M = -INFINITY;
        for (uint32_t w = w0; w < w0 + act; ++w) M = fmaxf(M, wst[w * (HD + 2)]);
        float L = 0.0f, O = 0.0f;
        for (uint32_t w = w0; w < w0 + act; ++w) {
            const float mw = wst[w * (HD + 2)];
            const float f = (mw == -INFINITY) ? 0.0f : __expf(mw - M);
            L += wst[w * (HD + 2) + 1] * f;
            O += wst[w * (HD + 2) + 2 + d] * f;
        }
        xv[i] = O / L;
    }
    csync();
}

// Fold the previous layer's FFN delta into X (a slice per CTA) and clear it.
__device__ void fold_delta(Ctx &c, uint32_t l) {
    const Params &p = *c.p;
    if (p.tp_size > 1) return;  // tensor parallel: the down exchange adds into X itself
    const uint32_t per = (p.dim + gridDim.x - 1) / gridDim.x;
    const uint32_t e0 = blockIdx.x * per, e1 = min(p.dim, e0 + per);
    for (uint32_t e = e0 + threadIdx.x; e < e1; e += kCons) {
        if (l > 0) red_add(&p.X[e], __ldcg(&p.Y[e]));
        p.Y[e] = 0.0f;
    }
}

// O projection of the attention output staged in xv ([head slot][hd] f32).  With
// fold_l >= 0 the previous layer's FFN delta is folded into X (fold_delta) while
// the O MMAs run: nothing in phase B reads X before the O epilogue, and both add
// into X.
__device__ void o_projection(Ctx &c, uint32_t lay_count, int fold_l = -1) {
    const Params &p = *c.p;
    const Sched &S = *c.S;
    decompose_lanes(reinterpret_cast<const float *>(c.smem + c.L.xv), S.nh * p.hd, c.smem + c.L.bo,
                    c.smem + c.L.sfbo, false);
    signal_operand(c, PH_O);
    CST(8);
    if (fold_l >= 0) fold_delta(c, (uint32_t)fold_l);
    wait_acc(c, PH_O, lay_count & 1);
    CST(9);
    if (!c.ok) return;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (uint32_t i = warp >> 2; i < S.n_pairs; i += kCW / 4) {
        const float s = acc_row(c.tbase, 8 * i);
        const uint32_t row = S.pair_tile[i] * 128 + 32 * (warp & 3) + lane;
        red_add((p.tp_size > 1 ? p.tpo : p.X) + row, s);  // this rank's partial under TP
    }
    CST(10);
}

// B (short contexts): fold the FFN delta, attention of this CTA's heads over the
// whole sequence, O-projection pairs (head, O tile) added into X.
__device__ void phase_attn_o(Ctx &c, uint32_t l, uint32_t pos, uint32_t lay_count) {
    const Params &p = *c.p;
    const Sched &S = *c.S;
    if (S.n_pairs == 0) {
        fold_delta(c, l);
        return;
    }
    if (p.hd == 64) {
        stage_qkv<64>(c, l, pos);
        CST(6);
        attend<64>(c, l, pos);
    } else {
        stage_qkv<128>(c, l, pos);
        CST(6);
        attend<128>(c, l, pos);
    }
    CST(7);
    o_projection(c, lay_count, (int)l);
}

// Split attention for long contexts, part 1: unit u = (KV head g, slice s) of the
// sequence (one unit per CTA, units = n_kv * attn_slices), all q heads of the GQA
// group at once (each K/V row read once per unit).  The unit holding the current
// position also RoPEs and appends its K/V (bf16).  Writes per head the slice's
// (max, sum, unnormalised output) to attn_part[head][slice].
//
// Every consumer warp takes RW consecutive rows of a pass of kCW * RW positions
// (RW the smallest of 2, 4, 8 that covers the unit in one pass, else 8 and more
// passes, so a short slice still spreads over all warps): a row's Q.K is split
// over 32 / RW lanes (HD * RW / 32 dims each, vector loads of K and of the padded
// q) and summed with xor shuffles; the warp's V rows are loaded with its K rows;
// the softmax uses the CTA-wide maximum of each head (one exchange per pass), so
// the warps' outputs and sums merge by plain addition, done as a fixed-order tree
// in shared memory; P.V has lane = head-dim pair.
template <int HD, int GRP, int RW>
__device__ void unit_scan(Ctx &c, const float *qs, const uint16_t *kb, const uint16_t *vb, size_t row,
                          uint32_t t_begin, uint32_t t_end, float *rec0, uint32_t rec_stride) {
    constexpr int LPR = 32 / RW, DPL = HD / LPR, NV = HD / 32, QP = HD + HD / 8;
    static_assert(DPL % 4 == 0, "unit_scan: at least 4 dims per lane");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t r_in = lane / LPR, seg = lane % LPR;
    float *ps = reinterpret_cast<float *>(c.smem + c.L.ps) + warp * (kMaxGroup * 32);
    float *wmax = c.red, *wsum = c.red + kCW * kMaxGroup;  // [kCW][GRP] each
    float M[GRP], lsum[GRP], o[GRP][NV];
#pragma unroll
    for (int h = 0; h < GRP; ++h) {
        M[h] = -INFINITY, lsum[h] = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; ++i) o[h][i] = 0.0f;
    }
    for (uint32_t base = t_begin; base < t_end; base += kCW * RW) {  // uniform over the CTA
        const uint32_t t0 = base + warp * RW, t = t0 + r_in;
        const bool live = t < t_end;
        const uint32_t nt = t0 < t_end ? min((uint32_t)RW, t_end - t0) : 0u;
        // this warp's V rows (lane = head-dim pair), loaded before the scores exist
        uint32_t vw[RW][HD / 64];
#pragma unroll
        for (int j = 0; j < RW; ++j)
#pragma unroll
            for (int cc = 0; cc < HD / 64; ++cc)
                vw[j][cc] = (uint32_t)j < nt ? __ldcg(reinterpret_cast<const uint32_t *>(vb + (size_t)(t0 + j) * row) + 32 * cc + lane) : 0u;
        float sc[GRP];
#pragma unroll
        for (int h = 0; h < GRP; ++h) sc[h] = 0.0f;
        if (live) {
            const uint32_t d0 = seg * DPL;
            const uint16_t *kr = kb + (size_t)t * row + d0;
#pragma unroll
            for (int cc = 0; cc < (DPL + 7) / 8; ++cc) {
                float kv[8];
                if (DPL >= 8) {
                    const uint4 kq = __ldcg(reinterpret_cast<const uint4 *>(kr) + cc);
                    const uint32_t wv[4] = {kq.x, kq.y, kq.z, kq.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        kv[2 * j] = __uint_as_float(wv[j] << 16), kv[2 * j + 1] = __uint_as_float(wv[j] & 0xFFFF0000u);
                } else {
                    const uint2 kq = __ldcg(reinterpret_cast<const uint2 *>(kr));
                    kv[0] = __uint_as_float(kq.x << 16), kv[1] = __uint_as_float(kq.x & 0xFFFF0000u);
                    kv[2] = __uint_as_float(kq.y << 16), kv[3] = __uint_as_float(kq.y & 0xFFFF0000u);
                }
                const uint32_t d = d0 + 8 * cc, qo = d + (d >> 5) * 4;  // padded q index of dim d
#pragma unroll
                for (int h = 0; h < GRP; ++h) {
                    const float4 qa = *reinterpret_cast<const float4 *>(qs + h * QP + qo);
                    sc[h] += qa.x * kv[0] + qa.y * kv[1] + qa.z * kv[2] + qa.w * kv[3];
                    if (DPL >= 8) {
                        const float4 qb = *reinterpret_cast<const float4 *>(qs + h * QP + qo + 4);
                        sc[h] += qb.x * kv[4] + qb.y * kv[5] + qb.z * kv[6] + qb.w * kv[7];
                    }
                }
            }
        }
#pragma unroll
        for (int h = 0; h < GRP; ++h) {
#pragma unroll
            for (int off = LPR / 2; off > 0; off >>= 1) sc[h] += __shfl_xor_sync(0xffffffffu, sc[h], off);
            const float wm = warp_max(live ? sc[h] : -INFINITY);
            if (lane == 0) wmax[warp * GRP + h] = wm;
        }
        CST(38);
        csync();
        float mn[GRP];
#pragma unroll
        for (int h = 0; h < GRP; ++h) {
            mn[h] = M[h];
            for (int w = 0; w < kCW; ++w) mn[h] = fmaxf(mn[h], wmax[w * GRP + h]);
            const float alpha = __expf(M[h] - mn[h]);  // M = -inf on the first pass -> 0
            const float pr = live ? __expf(sc[h] - mn[h]) : 0.0f;
            lsum[h] = lsum[h] * alpha + warp_sum(seg == 0 ? pr : 0.0f);
            if (seg == 0) ps[h * 32 + r_in] = pr;
#pragma unroll
            for (int i = 0; i < NV; ++i) o[h][i] *= alpha;
            M[h] = mn[h];
        }
        __syncwarp();
        CST(39);
#pragma unroll
        for (int j = 0; j < RW; ++j) {
            if ((uint32_t)j >= nt) break;
            float v[NV];
#pragma unroll
            for (int cc = 0; cc < HD / 64; ++cc) {
                v[2 * cc] = __uint_as_float(vw[j][cc] << 16);
                v[2 * cc + 1] = __uint_as_float(vw[j][cc] & 0xFFFF0000u);
            }
#pragma unroll
            for (int h = 0; h < GRP; ++h) {
                const float pr = ps[h * 32 + j];
#pragma unroll
                for (int i = 0; i < NV; ++i) o[h][i] += pr * v[i];
            }
        }
        csync();  // wmax and ps are rewritten by the next pass (or the merge)
    }
    CST(33);
    // warps w and w + half merge (w < half), half = 8, 4, 2, 1: outputs through the
    // probability area (kCW * kMaxGroup * 32 floats), HC heads per tree so that 8
    // warps x HC x HD values fit it; sums through wsum.  Every warp takes part; warps
    // without rows add zeros.
    constexpr int HC = (kCW * kMaxGroup * 32) / (kCW / 2 * HD) < GRP ? (kCW * kMaxGroup * 32) / (kCW / 2 * HD) : GRP;
    static_assert(HC >= 1 && GRP % HC == 0, "unit_scan: merge chunking");
    float *mrg = reinterpret_cast<float *>(c.smem + c.L.ps);
#pragma unroll
    for (int hb = 0; hb < GRP; hb += HC) {
#pragma unroll 1
        for (int half = kCW / 2; half > 0; half >>= 1) {
            if (warp >= half && warp < 2 * half) {
                float *dst = mrg + (warp - half) * (HC * HD);
#pragma unroll
                for (int h = hb; h < hb + HC; ++h) {
#pragma unroll
                    for (int cc = 0; cc < HD / 64; ++cc)
                        *reinterpret_cast<float2 *>(dst + (h - hb) * HD + 64 * cc + 2 * lane) =
                            make_float2(o[h][2 * cc], o[h][2 * cc + 1]);
                    if (lane == 0) wsum[(warp - half) * GRP + h] = lsum[h];
                }
            }
            csync();
            if (warp < half) {
                const float *src = mrg + warp * (HC * HD);
#pragma unroll
                for (int h = hb; h < hb + HC; ++h) {
#pragma unroll
                    for (int cc = 0; cc < HD / 64; ++cc) {
                        const float2 v = *reinterpret_cast<const float2 *>(src + (h - hb) * HD + 64 * cc + 2 * lane);
                        o[h][2 * cc] += v.x, o[h][2 * cc + 1] += v.y;
                    }
                    lsum[h] += wsum[warp * GRP + h];
                }
            }
            csync();
        }
    }
    if (warp == 0) {
#pragma unroll
        for (int h = 0; h < GRP; ++h) {
            float *r = rec0 + (size_t)h * rec_stride;
            if (lane == 0) r[0] = M[h], r[1] = lsum[h];
#pragma unroll
            for (int cc = 0; cc < HD / 64; ++cc)
                *reinterpret_cast<float2 *>(r + 2 + 64 * cc + 2 * lane) = make_float2(o[h][2 * cc], o[h][2 * cc + 1]);
        }
    }
}

template <int HD, int GRP>
__device__ void attend_unit(Ctx &c, uint32_t l, uint32_t pos) {
    const Params &p = *c.p;
    constexpr uint32_t half = HD / 2;
    const int tid = threadIdx.x;
    const uint32_t slices = p.attn_slices, u = blockIdx.x;
    if (u >= p.n_kv * slices) return;
    const uint32_t g = u / slices, sl = u % slices, seq = pos + 1;
    const uint32_t len = (seq + slices - 1) / slices, t_begin = min(seq, sl * len), t_end = min(seq, t_begin + len);
    const uint32_t h0 = g * GRP;
    // [GRP][HD + HD / 8]: 4 floats of padding after every 32 dims, so the lanes of a
    // warp that read different dims of q hit different banks
    float *qs = reinterpret_cast<float *>(c.smem + c.L.qs);
    constexpr uint32_t QP = HD + HD / 8;
    const float *cs = p.cos_t + (size_t)pos * half, *sn = p.sin_t + (size_t)pos * half;
    const float scale = 1.0f / sqrtf((float)HD);
    for (uint32_t i = tid; i < GRP * half; i += kCons) {
        const uint32_t hh = i / half, j = i % half, j2 = j + half;
        const float *qr = p.qkv + (h0 + hh) * HD;
        const float q0 = __ldcg(qr + j), q1 = __ldcg(qr + j2);
        qs[hh * QP + j + (j >> 5) * 4] = __fsub_rn(__fmul_rn(q0, cs[j]), __fmul_rn(q1, sn[j])) * scale;
        qs[hh * QP + j2 + (j2 >> 5) * 4] = __fadd_rn(__fmul_rn(q1, cs[j]), __fmul_rn(q0, sn[j])) * scale;
    }
    const size_t row = p.kvd;
    uint16_t *kb = p.kc + (size_t)l * p.max_seq * row + g * HD, *vb = p.vc + (size_t)l * p.max_seq * row + g * HD;
    if (t_end == seq && t_begin < seq && tid < half) {  // this unit holds the current position: append its K/V
        const float *kr = p.qkv + p.qd + g * HD, *vr = p.qkv + p.qd + p.kvd + g * HD;
        const uint32_t j = tid;
        const float k0 = __ldcg(kr + j), k1 = __ldcg(kr + j + half);
        kb[(size_t)pos * row + j] = f32_to_bf16_bits(__fsub_rn(__fmul_rn(k0, cs[j]), __fmul_rn(k1, sn[j])));
        kb[(size_t)pos * row + j + half] = f32_to_bf16_bits(__fadd_rn(__fmul_rn(k1, cs[j]), __fmul_rn(k0, sn[j])));
        vb[(size_t)pos * row + j] = f32_to_bf16_bits(__ldcg(vr + j));
        vb[(size_t)pos * row + j + half] = f32_to_bf16_bits(__ldcg(vr + j + half));
    }
    csync();
    CST(32);
    // heads scanned together: at most 4 of 128 dims (8 would hold 32 more
    // accumulators per lane than the kernel's register budget leaves)
    constexpr int GS = HD * GRP > 512 ? 512 / HD : GRP;
    const uint32_t n = t_end - t_begin, stride = slices * (HD + 2);
#pragma unroll 1
    for (int hs = 0; hs < GRP; hs += GS) {
        float *rec0 = p.attn_part + ((size_t)(h0 + hs) * slices + sl) * (HD + 2);
        const float *q = qs + hs * QP;
        if (n <= 2u * kCW) unit_scan<HD, GS, 2>(c, q, kb, vb, row, t_begin, t_end, rec0, stride);
        else if (n <= 4u * kCW) unit_scan<HD, GS, 4>(c, q, kb, vb, row, t_begin, t_end, rec0, stride);
        else unit_scan<HD, GS, 8>(c, q, kb, vb, row, t_begin, t_end, rec0, stride);
    }
    CST(34);
}

// Split attention, part 1 (every CTA): fold the FFN delta, then this CTA's unit.
__device__ void phase_attn_units(Ctx &c, uint32_t l, uint32_t pos) {
    const Params &p = *c.p;
    fold_delta(c, l);
    const uint32_t group = p.n_heads / p.n_kv;
    if (p.hd == 64) {
        if (group == 8) attend_unit<64, 8>(c, l, pos);
        else if (group == 4) attend_unit<64, 4>(c, l, pos);
        else attend_unit<64, 2>(c, l, pos);
    } else {
        if (group == 8) attend_unit<128, 8>(c, l, pos);
        else if (group == 4) attend_unit<128, 4>(c, l, pos);
        else attend_unit<128, 2>(c, l, pos);
    }
    CST(6);
}

// Split attention, part 2 (after a grid barrier): combine the slices of this CTA's
// heads into xv, then the O projection.
__device__ void phase_attn_combine_o(Ctx &c, uint32_t lay_count) {
    const Params &p = *c.p;
    const Sched &S = *c.S;
    if (S.n_pairs == 0) return;
    const uint32_t hd = p.hd, NS = p.attn_slices, nh = S.nh, tid = threadIdx.x;
    const uint32_t warp = tid >> 5, lane = tid & 31;
    float *xv = reinterpret_cast<float *>(c.smem + c.L.xv);
    // the split-attention probability area is free here: [nh][NS] slice maxima (then
    // their factors), [nh][NS] slice sums, [G][nh * hd] partial outputs
    float *fm = reinterpret_cast<float *>(c.smem + c.L.ps), *fl = fm + nh * NS, *part = fl + nh * NS;
    auto rec = [&](uint32_t hs, uint32_t s) { return p.attn_part + ((size_t)(S.h0 + hs) * NS + s) * (hd + 2); };
    for (uint32_t i = tid; i < nh * NS; i += kCons) {
        const float *r = rec(i / NS, i % NS);
        fm[i] = __ldcg(r);
        fl[i] = __ldcg(r + 1);
    }
    csync();
    if (warp < nh) {  // warp hs: the head's maximum, slice factors and normaliser
        float M = -INFINITY;
        for (uint32_t s = lane; s < NS; s += 32) M = fmaxf(M, fm[warp * NS + s]);
        M = warp_max(M);
        float L = 0.0f;
        for (uint32_t s = lane; s < NS; s += 32) {
            const float ms = fm[warp * NS + s];
            const float f = ms == -INFINITY ? 0.0f : __expf(ms - M);
            fm[warp * NS + s] = f;
            L += fl[warp * NS + s] * f;
        }
        L = warp_sum(L);
        if (lane == 0) c.red[warp] = L;
    }
    csync();
    // G slice groups per output column, each summing its slices with independent loads
    const uint32_t cols = nh * hd, G = max(1u, min(kCons / cols, NS));
    for (uint32_t i = tid; i < G * cols; i += kCons) {
        const uint32_t g = i / cols, col = i % cols, hs = col / hd, d = col % hd;
        float O = 0.0f;
#pragma unroll 16
        for (uint32_t s2 = g; s2 < NS; s2 += G) O += fm[hs * NS + s2] * __ldcg(rec(hs, s2) + 2 + d);
        part[i] = O;
    }
    csync();
    for (uint32_t i = tid; i < cols; i += kCons) {
        float O = 0.0f;
        for (uint32_t g = 0; g < G; ++g) O += part[g * cols + i];
        xv[i] = O / c.red[i / hd];
    }
    csync();
    CST(7);
    o_projection(c, lay_count);
}

// The two CTAs of a K-split FFN pair meet: row r's partial gate/up sum of each CTA
// travels as one 64-bit word {tag, value} in its half of p.ffx, tag = (launch << 20)
// | barrier count, so every word validates itself (no flag, no fence: the previous
// use of a slot carries another tag).  Warps 0-3 (rows 0..127) store their word,
// poll the partner's (bounded, abort-aware) and add the halves in K order into
// gu (identical bits in both CTAs).  Uniform result over the CTA.
__device__ bool ffn_pair_exchange(Ctx &c, const Sched &S, float *gu) {
    const Params &p = *c.p;
    volatile uint32_t *flag = reinterpret_cast<volatile uint32_t *>(c.smem + c.L.flag);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = 32 * warp + lane;
    const uint32_t tag = (p.launch_seq << 20) | (c.nbar & 0xFFFFFu);
    if (threadIdx.x == 0) flag[2] = 1;
    csync();
    if (warp < 4) {
        const float own = acc_row(c.tbase, 0);
        uint64_t *pair = p.ffx + (size_t)(S.f0 / 64) * 2 * 128;
        const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(own);
        asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(pair + S.kh * 128 + r), "l"(w) : "memory");
        const uint64_t *src = pair + (S.kh ^ 1u) * 128 + r;
        uint64_t v = 0;
        bool ok = true;
        for (uint32_t it = 0;; ++it) {
            asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(src) : "memory");
            if ((uint32_t)(v >> 32) == tag) break;
            if (((it & 63) == 63 && ld_volatile(&p.bar[1])) || it > kBarLimit) {
                if (it > kBarLimit) {
                    atomicExch(&p.bar[1], 1u);
                    raise_device_error(DEVERR_FLAG_TIMEOUT);
                }
                ok = false;
                break;
            }
        }
        const float other = __uint_as_float((uint32_t)v);
        if (ok && r < 2 * S.U) gu[r] = S.kh == 0 ? own + other : other + own;
        if (!ok) flag[2] = 0;
    }
    csync();
    c.ok = c.ok && flag[2] != 0;
    if (!c.ok && threadIdx.x == 0) *c.B.abort = 1;
    return c.ok;
}

// C: zero a slice of the QKV sums (read in B, next written in the next layer's
// A), RMSNorm -> gate/up rows of FFN [f0, f0+U) -> SwiGLU -> down projection of
// those U indices, added into Y.
__device__ void phase_ffn(Ctx &c, uint32_t l, uint32_t lay_count) {
    const Params &p = *c.p;
    const Sched &S = *c.S;
    {
        const uint32_t n = p.qd + 2 * p.kvd, per = (n + gridDim.x - 1) / gridDim.x;
        const uint32_t e0 = blockIdx.x * per, e1 = min(n, e0 + per);
        for (uint32_t e = e0 + threadIdx.x; e < e1; e += kCons) p.qkv[e] = 0.0f;
    }
    norm_decompose<0>(c, nullptr, p.ffn_norm + (size_t)l * p.dim, S.U > 0);
    CST(12);
    if (S.U == 0) return;
    signal_operand(c, PH_GU);
    CST(13);
    wait_acc(c, PH_GU, lay_count & 1);
    CST(14);
    if (!c.ok) return;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, U = S.U;
    float *gu = reinterpret_cast<float *>(c.smem + c.L.gu);
    const uint32_t ngu = (2 * U + 127) / 128;  // gate/up tiles: rows [gate 0..U) [up 0..U)
    if (S.ks > 1) {
        // K-split pair: publish this CTA's partial sums, wait for the partner's, and
        // add the two halves in K order (identical bits in both CTAs)
        if (!ffn_pair_exchange(c, S, gu)) return;
    } else {
        for (uint32_t t = warp >> 2; t < ngu; t += kCW / 4) {
            const float s = acc_row(c.tbase, 8 * t);
            const uint32_t r = t * 128 + 32 * (warp & 3) + lane;
            if (r < 2 * U) gu[r] = s;
        }
    }
    csync();
    float *h = reinterpret_cast<float *>(c.smem + c.L.xv);
    for (uint32_t i = threadIdx.x; i < U; i += kCons) {
        const float gv = gu[i], uv = gu[U + i];
        h[i] = gv / (1.0f + expf(-gv)) * uv;  // llama_run:245-253
    }
    csync();
    decompose_lanes(h, U, c.smem + c.L.bh, c.smem + c.L.sfbh, (U % 64) != 0);
    signal_operand(c, PH_DOWN);
    CST(15);
    wait_acc(c, PH_DOWN, lay_count & 1);
    CST(16);
    if (!c.ok) return;
    const uint32_t mt = p.dim / 128;
    // The CTA's whole down partial (dim values) is added into Y (this rank's partial
    // accumulator under TP) by one bulk reduction: the L2 applies it a sector at a
    // time instead of one element per red.add (148 CTAs x dim element updates per
    // layer otherwise).  The staging buffer (the activation staging area, free once
    // the down MMAs are done) is read by the bulk copy before this thread reaches
    // the next grid barrier.
    float *stg = reinterpret_cast<float *>(c.smem + c.L.xv);
    const uint32_t ta = mt * S.kh / S.ks, tb = mt * (S.kh + 1) / S.ks;  // this CTA's down tiles
    for (uint32_t t = ta + (warp >> 2); t < tb; t += kCW / 4)
        stg[t * 128 + 32 * (warp & 3) + lane] = acc_row(c.tbase, 8 * t);
    fence_proxy_async_smem();
    csync();
    if (threadIdx.x == 0) {
        tc::bulk_reduce_add_f32((p.tp_size > 1 ? p.tpd : p.Y) + ta * 128, stg + ta * 128, (tb - ta) * 128 * 4);
        tc::bulk_commit();
        tc::bulk_wait_all();
    }
    CST(17);
}

// L: final RMSNorm -> lm_head tiles -> logits + this CTA's argmax candidate.
__device__ void phase_lm(Ctx &c, uint32_t tok_count) {
    const Params &p = *c.p;
    const Sched &S = *c.S;
    if (p.tp_size > 1)
        norm_decompose<0>(c, nullptr, p.final_norm, S.n_l > 0);
    else
        norm_decompose<1>(c, nullptr, p.final_norm, S.n_l > 0);
    CST(1);
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    if (S.n_l > 0) {
        signal_operand(c, PH_LM);
        CST(2);
        wait_acc(c, PH_LM, tok_count & 1);
        CST(3);
        if (c.ok) {
            const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
            for (uint32_t i = warp >> 2; i < S.n_l; i += kCW / 4) {
                const float s = acc_row(c.tbase, 8 * i);
                const uint32_t row = S.l_tile[i] * 128 + 32 * (warp & 3) + lane;
                if (row < p.vocab) {
                    p.logits[row] = s;
                    const uint32_t gi = p.v0 + row;  // vocab index (shard offset under TP)
                    if (s > bv || (s == bv && gi < bi)) bv = s, bi = gi;  // llama_run:283-292
                }
            }
        }
    }
    // CTA argmax: larger value wins, ties to the lower index
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t *ri = reinterpret_cast<uint32_t *>(c.red + 256);
    if (lane == 0) c.red[128 + warp] = bv, ri[warp] = bi;
    csync();
    if (threadIdx.x == 0) {
        float v = c.red[128];
        uint32_t ix = ri[0];
        for (int w = 1; w < kCW; ++w)
            if (c.red[128 + w] > v || (c.red[128 + w] == v && ri[w] < ix)) v = c.red[128 + w], ix = ri[w];
        for (uint32_t r = 0; r < p.tp_size; ++r) {  // every rank reduces the same candidate list
            p.cvr[r][p.tp_rank * gridDim.x + blockIdx.x] = v;
            p.cir[r][p.tp_rank * gridDim.x + blockIdx.x] = ix;
        }
    }
}

// ---------------------------------------------------------------- MMA warp (one lane)

struct BOperand {
    uint32_t addr, sfb, atoms, zero;
    bool k32;
};

__device__ BOperand operand_of(int ph, const Params &p, const Sched &S, uint8_t *smem, const Smem &L) {
    BOperand b;
    b.zero = smem_u32(smem + L.bh + 4 * 128);
    b.k32 = false;
    if (ph == PH_O) {
        b.addr = smem_u32(smem + L.bo), b.sfb = smem_u32(smem + L.sfbo);
        b.atoms = (S.nh * p.hd / 32 + 3) / 4;
    } else if (ph == PH_DOWN) {
        b.addr = smem_u32(smem + L.bh), b.sfb = smem_u32(smem + L.sfbh);
        b.k32 = (S.U % 64) != 0;
        b.atoms = b.k32 ? (S.U / 32 + 1) / 2 : (S.U / 32 + 3) / 4;
    } else {
        b.addr = smem_u32(smem + L.bx), b.sfb = smem_u32(smem + L.sfbx);
        b.atoms = p.dim / 128;
    }
    return b;
}

// Byte-ring placement, computed identically by the producer and the MMA lane:
// chunks are laid end to end and a chunk that would cross the end starts at 0.
struct RingPlace {
    uint64_t wrap = 0;  // virtual position of the current pass's ring start
    uint32_t off = 0;
    __device__ __forceinline__ uint32_t place(uint32_t bytes, uint32_t R, uint64_t &vstart) {
        if (off + bytes > R) {
            wrap += R;
            off = 0;
        }
        vstart = wrap + off;
        const uint32_t at = off;
        off += bytes;
        return at;
    }
};

// Issues the MMAs of one list of chunk ops; returns false on abort.
__device__ bool run_ops(const Params &p, const Sched &S, const ChunkOp *ops, uint32_t n_ops, uint32_t count,
                        uint8_t *smem, const Smem &L, const Bars &B, uint32_t tbase, uint32_t &seq, RingPlace &rp,
                        uint32_t tsb) {
    int cur = -1;
    BOperand bo{};
    uint8_t *ring = smem + L.ring;
    for (uint32_t i = 0; i < n_ops; ++i) {
        const ChunkOp op = ops[i];
        if (op.phase != cur) {
            if (cur >= 0) tc::commit(&B.accr[cur]);
            cur = op.phase;
            if (!wait_bar(&B.bready[cur], count & 1, p, B.abort)) return false;
            tstamp(tsb + 19 + (cur == PH_LM ? 0 : cur));
            tc::fence_after_sync();
            bo = operand_of(cur, p, S, smem, L);
            // only the atoms this CTA's blocks read (a QKV unit's k-range needs a few)
            for (uint32_t r = 0; r < 4; r += 2) {
                const uint32_t a0 = S.batoms[cur][r], a1 = a0 + S.batoms[cur][r + 1];
                for (uint32_t a = a0; a < a1; ++a)
                    tc::utccp_scale_atom(tbase + p.sfb_col0 + 4 * a, tc::smem_desc(bo.sfb + 128 * a, 128, 128, 0));
            }
        }
        const uint32_t slot = seq % kMaxSlots;
        uint64_t vstart;
        const uint32_t at = rp.place(op.bytes, p.ring_bytes, vstart);
        if (!wait_bar(&B.full[slot], (seq / kMaxSlots) & 1, p, B.abort)) return false;
        mstamp(2 * seq);
        tc::fence_after_sync();
        const uint32_t base = smem_u32(ring + at);
        const uint32_t bbytes = (op.kmode ? 128u : 256u) * op.rows8;
        const uint32_t atoms = base + op.nblk * bbytes, sfa = tbase + p.sfa_col0 + (seq % p.n_inflight) * 16;
        for (uint32_t a = 0; a < (op.nblk + 1u) / 2; ++a)
            tc::utccp_scale_atom(sfa + 4 * a, tc::smem_desc(atoms + kAtom * a, 128, 128, 0));
        // descriptors advance by adding to their 16-byte-unit address fields
        uint64_t adesc = op.kmode ? tc::smem_desc(base, 128, 128, 0) : tc::smem_desc(base, 128, 256, 0);
        const uint64_t astep = bbytes >> 4;
        uint64_t bdesc0, bstep;
        if (bo.k32) {  // 32-k block: the MMA's second k half reads the zero column (LBO shrinks as start grows)
            bdesc0 = tc::smem_desc(bo.addr, bo.zero - bo.addr, 128, 0);
            bstep = 8u - ((uint64_t)8u << 16);
        } else {
            bdesc0 = tc::smem_desc(bo.addr, 128, 128, 0);
            bstep = 16u;
        }
        const uint32_t idesc = tc::idesc_mxf4(8), sfb0 = tbase + p.sfb_col0;
        uint32_t acc = tbase + 8u * op.acc0, jj = 0, bk = op.bk0;
        for (uint32_t j = 0; j < op.nblk; ++j) {
            const uint64_t bdesc = bdesc0 + bstep * bk;
            const uint32_t tsfb = (sfb0 + 4u * (bk >> 1)) | ((2u * (bk & 1u)) << 30);
            const uint32_t tsfa = (sfa + 4u * (j >> 1)) | ((2u * (j & 1u)) << 30);
            tc::mma_mxf4(acc, adesc, bdesc, idesc, tsfa, tsfb, (jj != 0) || (j == 0 && op.cont));
            adesc += astep;
            if (++jj == op.bpa) {
                jj = 0;
                acc += 8;
                bk = op.bk0;
            } else {
                ++bk;
            }
        }
        tc::commit(&B.empty[slot]);
        mstamp(2 * seq + 1);
        seq += 1;
    }
    if (cur >= 0) tc::commit(&B.accr[cur]);
    return true;
}

__device__ void producer(const Params &p, const Sched &S, const Bars &B, uint8_t *ring) {
    const int lane = threadIdx.x & 31;
    const uint8_t *stream = p.arena + S.stream_off;
    const uint64_t pol = policy_evict_first();
    const uint32_t pos0 = p.state[1];
    const uint32_t n_eff = pos0 < p.max_seq ? min(p.n_tokens, p.max_seq - pos0) : 0u;
    const uint32_t R = p.ring_bytes;
    RingPlace rp;
    uint64_t vst[kMaxSlots];  // virtual start of the chunks in flight (by seq % kMaxSlots)
    uint32_t seq = 0, oldest = 0;
    bool abort = false;
    for (uint32_t tok = 0; tok < n_eff && !abort; ++tok) {
        size_t off = 0;
        for (uint32_t l = 0; l <= p.n_layers && !abort; ++l) {
            const ChunkOp *ops = l < p.n_layers ? S.ops : S.lm_ops;
            const uint32_t n = l < p.n_layers ? S.n_ops : S.n_lm_ops;
            for (uint32_t i = 0; i < n; ++i, ++seq) {
                const uint32_t bytes = ops[i].bytes;
                uint64_t vstart;
                const uint32_t at = rp.place(bytes, R, vstart);
                // the chunk's bytes must be free: retire older chunks (in order) until no chunk in
                // flight starts within R of this chunk's end, and at most n_inflight are in flight
                while (oldest < seq && (seq - oldest >= p.n_inflight || vst[oldest % kMaxSlots] + R < vstart + bytes)) {
                    bool got = false;
                    if (lane == 0) got = wait_bar(&B.empty[oldest % kMaxSlots], (oldest / kMaxSlots) & 1, p, B.abort);
                    got = __shfl_sync(0xffffffffu, got, 0);
                    if (!got) {
                        abort = true;
                        break;
                    }
                    ++oldest;
                }
                if (abort) break;
                vst[seq % kMaxSlots] = vstart;
                if (lane == 0) {
                    const uint32_t slot = seq % kMaxSlots;
                    mbar_arrive_expect_tx(&B.full[slot], bytes);
                    bulk_g2s_hint(ring + at, stream + off, bytes, &B.full[slot], pol);
                }
                __syncwarp();
                off += bytes;
            }
        }
    }
    // never leave with copies in flight: the last use of each barrier
    const uint32_t issued = seq;
    if (lane == 0)
        for (uint32_t c = issued > (uint32_t)kMaxSlots ? issued - kMaxSlots : 0; c < issued; ++c)
            for (uint32_t it = 0; it < kSpinLimit && !mbar_try_wait(&B.full[c % kMaxSlots], (c / kMaxSlots) & 1); ++it) {
            }
}

__global__ void __launch_bounds__(kThreads, 1) decode_tc_kernel(Params p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw;
    const Smem L = smem_layout(p);
    const Bars B = bars_of(smem, L);
    const uint32_t warp = threadIdx.x >> 5;
    {  // stage the schedule; zero the operand buffers (unused atom bytes, the zero column)
        const uint32_t *src = reinterpret_cast<const uint32_t *>(&p.sched[blockIdx.x]);
        uint32_t *dst = reinterpret_cast<uint32_t *>(smem + L.sched);
        for (uint32_t i = threadIdx.x; i < sizeof(Sched) / 4; i += blockDim.x) dst[i] = src[i];
        for (uint32_t i = L.bx + threadIdx.x * 4; i < L.qs; i += blockDim.x * 4)
            *reinterpret_cast<uint32_t *>(smem + i) = 0u;
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMaxSlots; ++i) {
            mbar_init(&B.full[i], 1);
            mbar_init(&B.empty[i], 1);
        }
        for (int i = 0; i < PH_N; ++i) {
            mbar_init(&B.bready[i], 1);
            mbar_init(&B.accr[i], 1);
        }
        mbar_init(B.fin, 1);
        *B.abort = 0;
        reinterpret_cast<volatile uint32_t *>(smem + L.flag)[0] = 1;
        reinterpret_cast<volatile uint32_t *>(smem + L.flag)[1] = 0;
        fence_mbar_init();
    }
    if (warp == kCW) {
        tc::tmem_alloc(B.tmem, p.tmem_cols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = *B.tmem;
    const Sched &S = *reinterpret_cast<const Sched *>(smem + L.sched);
    const uint32_t pos0 = p.state[1];
    const uint32_t n_eff = pos0 < p.max_seq ? min(p.n_tokens, p.max_seq - pos0) : 0u;

    if (warp == kCW + 1) {
        producer(p, S, B, smem + L.ring);
    } else if (warp == kCW) {
        if ((threadIdx.x & 31) == 0) {
            uint32_t seq = 0;
            RingPlace rp;
            bool ok = true;
            for (uint32_t tok = 0; tok < n_eff && ok; ++tok) {
                for (uint32_t l = 0; l < p.n_layers && ok; ++l)
                    ok = run_ops(p, S, S.ops, S.n_ops, tok * p.n_layers + l, smem, L, B, tbase, seq, rp,
                                 (tok * (p.n_layers + 1) + l) * kTsPerLayer);
                if (ok)
                    ok = run_ops(p, S, S.lm_ops, S.n_lm_ops, tok, smem, L, B, tbase, seq, rp,
                                 (tok * (p.n_layers + 1) + p.n_layers) * kTsPerLayer);
            }
            // no MMA or scale copy may still be running when TMEM is freed
            tc::commit(B.fin);
            for (uint32_t it = 0; it < kSpinLimit && !mbar_try_wait(B.fin, 0); ++it) {
            }
        }
        __syncwarp();
    } else {
        Ctx c;
        c.p = &p, c.S = &S, c.smem = smem, c.L = L, c.B = B, c.tbase = tbase;
        c.red = reinterpret_cast<float *>(smem + L.red);
        c.nbar = 0, c.ok = true;
        c.epoch0 = p.tp_size > 1 ? *p.epoch : 0u;
        c.xn = p.tp_size > 1 ? *p.xepoch : 0u;
        uint32_t tok = p.state[0], pos = pos0;
        const uint32_t n_prompt = p.state[3], cap = p.state[4];
        for (uint32_t it = 0; it < n_eff && c.ok; ++it) {
            for (uint32_t l = 0; l < p.n_layers; ++l) {
                const uint32_t lc = it * p.n_layers + l;
                c.tsb = (it * (p.n_layers + 1) + l) * kTsPerLayer;
                CST(0);
                const bool split = p.attn_slices && pos + 1 > kSplitMinSeq;  // same decision in every CTA
                phase_qkv(c, l, tok, lc, split ? (int)pos : -1);
                if (!grid_barrier(c)) break;
                CST(5);
                if (split) {
                    phase_attn_units(c, l, pos);
                    if (!grid_barrier(c)) break;
                    phase_attn_combine_o(c, lc);
                } else {
                    phase_attn_o(c, l, pos, lc);
                }
                if (!grid_barrier(c)) break;
                if (p.tp_size > 1 && (!tp_exchange(c, 0, c.xn) || !grid_barrier(c))) break;
                CST(11);
                phase_ffn(c, l, lc);
                if (!grid_barrier(c)) break;
                if (p.tp_size > 1 && (!tp_exchange(c, 1, c.xn) || !grid_barrier(c))) break;
                c.xn += 1;
                CST(18);
            }
            if (!c.ok) break;
            c.tsb = (it * (p.n_layers + 1) + p.n_layers) * kTsPerLayer;
            CST(0);
            phase_lm(c, it);
            if (!grid_barrier(c, true)) break;  // every rank's argmax candidates are in place
            CST(5);
            // every CTA reduces the candidates itself (same order -> same token)
            float *rv = c.red;
            uint32_t *ri = reinterpret_cast<uint32_t *>(c.red + 1);
            if (threadIdx.x < 32) {
                const int lane = threadIdx.x;
                float bv = -INFINITY;
                uint32_t bi = 0xFFFFFFFFu;
                for (uint32_t i = lane; i < gridDim.x * p.tp_size; i += 32) {
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
                if (lane == 0) rv[0] = bv, ri[0] = bi;
            }
            csync();
            const uint32_t next = ri[0];
            csync();
            if (blockIdx.x == 0 && threadIdx.x == 0) {
                p.state[2] = next;
                if (pos + 1 >= n_prompt && pos + 1 - n_prompt < cap) p.out[pos + 1 - n_prompt] = next;
                p.state[0] = (pos + 1 < n_prompt) ? p.prompt[pos + 1] : next;
                p.state[1] = pos + 1;
            }
            tok = (pos + 1 < n_prompt) ? p.prompt[pos + 1] : next;
            pos += 1;
        }
        if (!c.ok && threadIdx.x == 0) {
            *B.abort = 1;
            atomicExch(&p.bar[1], 1u);
        }
        // every rank ran the same barrier sequence: record it for the next launch
        if (p.tp_size > 1 && c.ok && blockIdx.x == 0 && threadIdx.x == 0) {
            *p.epoch = c.epoch0 + c.nbar;
            *p.xepoch = c.xn;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == kCW) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, p.tmem_cols);
    }
}

}  // namespace ptc
}  // namespace fp4x

// ---------------------------------------------------------------- host side
namespace fp4x {
namespace ptc {

// One packing job: nblk MMA blocks of one 128-row tile (rows mapped from the
// engine's storage order) and their scale bytes, placed at chunk block j0.
struct PackJob {
    const uint8_t *w, *s;
    uint32_t K;        // source row length (values)
    uint32_t rowmode;  // 0: row = lrow + off; 1: logical q|k|v -> engine QKV rows; 2: [gate f0.. | up f0..]
    uint32_t off, hd, qd, kvd, f0, U;
    uint32_t lrow0, nrows;
    uint32_t kb0;      // first 32-value block
    uint32_t nblk, kmode, rows8, j0;
    uint64_t blk_dst, atom_dst;
};

// Engine storage row of logical row r (see the row maps of the engine's initialiser).
__device__ __forceinline__ uint32_t engine_row(const PackJob &J, uint32_t r) {
    if (J.rowmode == 1) {
        if (r < J.qd + J.kvd) {
            const uint32_t base = r < J.qd ? 0u : J.qd, rr = r < J.qd ? r : r - J.qd;
            const uint32_t half = J.hd / 2, head = rr / J.hd, j = rr % J.hd, jj = j < half ? j : j - half;
            return base + (head * (half / 8) + jj / 8) * 16 + (j < half ? 0u : 8u) + jj % 8;
        }
        return r;  // V rows are stored in order after Q and K
    }
    if (J.rowmode == 2) {
        const bool up = r >= J.U;
        const uint32_t f = J.f0 + (up ? r - J.U : r);
        return (f / 8) * 16 + (up ? 8u : 0u) + f % 8;
    }
    return r + J.off;
}

__global__ void pack_kernel(const PackJob *jobs, uint8_t *arena) {
    const PackJob J = jobs[blockIdx.x];
    const uint32_t ncol = J.kmode ? 1u : 2u, bbytes = J.rows8 * ncol * 128u, nkb = J.K / 32;
    for (uint32_t b = 0; b < J.nblk; ++b) {
        const uint32_t jb = J.j0 + b;
        uint8_t *dst = arena + J.blk_dst + (size_t)jb * bbytes;
        for (uint32_t pc = threadIdx.x; pc < J.rows8 * 8 * ncol; pc += blockDim.x) {
            const uint32_t r = pc / ncol, col = pc % ncol, kb = J.kb0 + b * ncol + col;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r < J.nrows && kb < nkb)
                v = *reinterpret_cast<const uint4 *>(J.w + (size_t)engine_row(J, J.lrow0 + r) * (J.K / 2) + kb * 16);
            *reinterpret_cast<uint4 *>(dst + (r / 8) * (ncol * 128) + col * 128 + (r % 8) * 16) = v;
        }
        uint8_t *atom = arena + J.atom_dst + (size_t)(jb / 2) * kAtom;
        for (uint32_t r = threadIdx.x; r < 128; r += blockDim.x) {
            uint8_t s0 = 0, s1 = 0;
            const uint32_t kb = J.kb0 + b * ncol;
            if (r < J.nrows && kb < nkb) {
                const size_t rs = (size_t)engine_row(J, J.lrow0 + r) * nkb;
                s0 = J.s[rs + kb];
                s1 = (J.kmode || kb + 1 >= nkb) ? s0 : J.s[rs + kb + 1];
            }
            const uint32_t o = 16 * (r % 32) + 4 * (r / 32) + 2 * (jb % 2);
            atom[o] = s0;
            atom[o + 1] = s1;
        }
    }
}

struct Engine {
    Params p;
    int grid = 0;
    size_t smem = 0;
    uint32_t launches = 0;  // launches so far (the FFN split tags)
    uint64_t arena_bytes = 0;
    std::vector<void *> allocs;
};

static int fail(const char *what, cudaError_t e) {
    set_error("tensor-core decode: %s: %s", what, cudaGetErrorString(e));
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
        set_error("tensor-core decode: cudaMalloc(%zu): %s", count * sizeof(T), cudaGetErrorString(err));
        return FP4X_ENOMEM;
    }
    e->allocs.push_back(q);
    *p = static_cast<T *>(q);
    return FP4X_OK;
}

// Tensor-parallel placement of the kernel's shared buffers (all inside the ranks'
// exchange areas): this rank, the rank count, its first vocab row, and per rank the
// X / Y / candidate / flag buffers mapped into this process.
struct TpIn {
    uint32_t rank = 0, size = 1, v0 = 0;
    float *xr[kMaxTp] = {}, *yr[kMaxTp] = {}, *cvr[kMaxTp] = {};
    uint32_t *cir[kMaxTp] = {}, *flagr[kMaxTp] = {};
    uint32_t *epoch = nullptr;
    // row-parallel exchange: every rank's receive slots, this rank's partials
    uint64_t *ro[kMaxTp] = {}, *rd[kMaxTp] = {};
    float *po = nullptr, *pd = nullptr;
    uint32_t *xepoch = nullptr;
};

#define PTC_UNSUPPORTED(...)            \
    do {                                \
        set_error(__VA_ARGS__);         \
        return FP4X_EUNSUPPORTED;       \
    } while (0)

// Builds the schedule, packs every weight into the per-CTA chunk streams and
// sizes shared and tensor memory.  FP4X_EUNSUPPORTED when the shape does not
// fit the kernel's static limits (the caller keeps another path).
int build(const persist::BuildIn &in, cudaStream_t st, Engine **out, const TpIn *tpin = nullptr) {
    const fp4x_llama_config &c = in.cfg;
    const uint32_t hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
    int dev = 0, G = 0, coop = 0, max_smem = 0, cc_major = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&G, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    if (!coop || G <= 0) PTC_UNSUPPORTED("tensor-core decode: cooperative launch unavailable");
    if (tpin && (tpin->size > (uint32_t)kMaxTp || G > 256))
        PTC_UNSUPPORTED("tensor-core decode: %u ranks x %d SMs above the exchange limits", tpin->size, G);
    if (cc_major != 10) PTC_UNSUPPORTED("tensor-core decode: needs an sm_100 GPU");
    if (c.dim % 128 || c.ffn % 32 || (hd != 64 && hd != 128) || c.n_heads % c.n_kv_heads || c.dim > 8192)
        PTC_UNSUPPORTED("tensor-core decode: unsupported shape");
    const uint32_t rows_qkv = qd + 2 * kvd, kb64 = c.dim / 64, otile = c.dim / 128;
    // FFN slices: 32-index units, contiguous per CTA.  When every unit has a CTA of
    // its own (ffn / 32 <= CTAs: the 8B shape at TP >= 4, small models), pairs of
    // CTAs share 64-index units instead, each taking half of gate/up's K and half of
    // down's output tiles: the same CTAs hold FFN work, but each one's gate/up MMA
    // chain is K/128 instead of K/64 steps and its down chain half as long; the pair
    // adds its partial gate/up sums (exchanged through global memory) before SwiGLU.
    const uint32_t nunits = c.ffn / 32;
    std::vector<Sched> S(G);
    for (auto &s : S) memset(&s, 0, sizeof(Sched));
    const bool pairs = c.ffn % 64 == 0 && nunits <= (uint32_t)G && kb64 % 2 == 0 && otile % 2 == 0;
    const uint32_t n64 = c.ffn / 64;
    uint32_t minU = ~0u;
    if (pairs) {
        for (uint32_t q = 0; q < 2 * n64; ++q) {
            Sched &s = S[(uint64_t)q * G / (2 * n64)];
            s.f0 = 64 * (q / 2), s.U = 64, s.ks = 2, s.kh = q % 2;
        }
    }
    for (int g = 0; g < G; ++g) {
        if (!pairs) {
            const uint32_t u0 = (uint32_t)((uint64_t)nunits * g / G), u1 = (uint32_t)((uint64_t)nunits * (g + 1) / G);
            S[g].f0 = 32 * u0, S[g].U = 32 * (u1 - u0), S[g].ks = 1, S[g].kh = 0;
        } else if (S[g].U == 0) {
            S[g].ks = 1;
        }
        if (S[g].U > 128) PTC_UNSUPPORTED("tensor-core decode: FFN slice of %u > 128 indices per CTA", S[g].U);
        minU = std::min(minU, S[g].U);
    }
    std::vector<int> light, order;  // CTAs with the smallest FFN slice take QKV/O first
    for (int g = 0; g < G; ++g)
        if (S[g].U == minU) light.push_back(g);
    order = light;
    for (int g = 0; g < G; ++g)
        if (S[g].U != minU) order.push_back(g);
    const uint32_t NL = (uint32_t)light.size();
    // QKV: flattened (tile, 64-k block) sequence split evenly over the light CTAs
    const uint32_t qtiles = (rows_qkv + 127) / 128, qtotal = qtiles * kb64;
    std::vector<std::vector<std::array<uint32_t, 3>>> qunits(G);  // (tile, b0, b1)
    for (uint32_t k = 0; k < NL; ++k) {
        const int g = light[k];
        uint32_t i0 = (uint32_t)((uint64_t)qtotal * k / NL), i1 = (uint32_t)((uint64_t)qtotal * (k + 1) / NL);
        while (i0 < i1) {
            const uint32_t t = i0 / kb64, b0 = i0 % kb64, b1 = std::min(kb64, b0 + (i1 - i0));
            if (S[g].n_a >= (uint32_t)kMaxAUnits) PTC_UNSUPPORTED("tensor-core decode: too many QKV units per CTA");
            S[g].a_tile[S[g].n_a++] = t;
            qunits[g].push_back({t, b0, b1});
            i0 += b1 - b0;
        }
    }
    // O: (head, 128-row tile) pairs, head-major, over the light CTAs.  When every
    // head can have the same number of CTAs (cph), each CTA takes pairs of one head
    // only, so every CTA with O work attends exactly one head (phase B balanced);
    // otherwise the pairs are split evenly.
    const uint32_t npairs = c.n_heads * otile, cph = NL / c.n_heads;
    const bool by_head = cph >= 1 && (otile + cph - 1) / cph <= (uint32_t)kMaxPairs;
    for (uint32_t k = 0; k < NL; ++k) {
        Sched &s = S[light[k]];
        uint32_t p0 = (uint32_t)((uint64_t)npairs * k / NL), p1 = (uint32_t)((uint64_t)npairs * (k + 1) / NL);
        if (by_head) {
            const uint32_t h = k / cph, j = k % cph;
            p0 = p1 = 0;
            if (h < c.n_heads) p0 = h * otile + otile * j / cph, p1 = h * otile + otile * (j + 1) / cph;
        }
        if (p1 - p0 > (uint32_t)kMaxPairs) PTC_UNSUPPORTED("tensor-core decode: too many O pairs per CTA");
        for (uint32_t q = p0; q < p1; ++q) {
            s.pair_head[s.n_pairs] = q / otile;
            s.pair_tile[s.n_pairs++] = q % otile;
        }
        if (s.n_pairs) {
            s.h0 = s.pair_head[0];
            s.nh = s.pair_head[s.n_pairs - 1] - s.h0 + 1;
            if (s.nh > (uint32_t)kMaxHeads) PTC_UNSUPPORTED("tensor-core decode: a CTA spans too many heads");
        }
    }
    // lm_head tiles: round robin, light CTAs first
    const uint32_t ltiles = (c.vocab + 127) / 128;
    for (uint32_t i = 0; i < ltiles; ++i) {
        Sched &s = S[order[i % G]];
        if (s.n_l >= (uint32_t)kMaxLm) PTC_UNSUPPORTED("tensor-core decode: too many lm_head tiles per CTA");
        s.l_tile[s.n_l++] = i;
    }
    // chunk programs + packing jobs
    std::vector<PackJob> jobs;
    uint64_t off = 0;
    uint32_t slot_bytes = 0;
    // blocks per chunk: as many as fit kSlotTarget (at most kMaxBlkPerChunk)
    auto per_chunk = [](uint32_t kmode, uint32_t rows8) {
        const uint32_t bb = rows8 * (kmode ? 128u : 256u);
        uint32_t nb = kMaxBlkPerChunk;
        while (nb > 1 && nb * bb + (nb + 1) / 2 * kAtom > kSlotTarget) --nb;
        return nb;
    };
    auto chunk = [&](Sched &s, bool lm, uint8_t ph, uint32_t nblk, uint8_t kmode, uint32_t bpa, uint32_t bk0,
                     uint32_t acc0, bool cont, uint32_t rows8, bool record) -> std::pair<uint64_t, uint64_t> {
        const uint32_t bytes = nblk * rows8 * (kmode ? 128u : 256u) + (nblk + 1) / 2 * kAtom;
        if (record) {
            ChunkOp op = {};
            op.bytes = bytes, op.phase = ph, op.nblk = (uint8_t)nblk, op.kmode = kmode;
            op.bpa = (uint8_t)std::min<uint32_t>(bpa, 255), op.bk0 = (uint16_t)bk0, op.acc0 = (uint8_t)acc0;
            op.cont = cont, op.rows8 = (uint8_t)rows8;
            if (lm) s.lm_ops[s.n_lm_ops++] = op;
            else s.ops[s.n_ops++] = op;
        }
        slot_bytes = std::max(slot_bytes, bytes);
        const uint64_t blk = off, atoms = off + (uint64_t)nblk * rows8 * (kmode ? 128u : 256u);
        off += bytes;
        return {blk, atoms};
    };
    auto job = [&](const persist::Tensor &t, uint32_t rowmode, uint32_t f0, uint32_t U, uint32_t lrow0,
                   uint32_t nrows, uint32_t kb0, uint32_t nblk, uint32_t kmode, uint32_t rows8, uint32_t j0,
                   std::pair<uint64_t, uint64_t> dst) {
        PackJob j = {};
        j.w = t.w, j.s = t.s, j.K = t.k, j.rowmode = rowmode, j.off = 0, j.hd = hd, j.qd = qd, j.kvd = kvd;
        j.f0 = f0, j.U = U, j.lrow0 = lrow0, j.nrows = nrows, j.kb0 = kb0, j.nblk = nblk, j.kmode = kmode;
        j.rows8 = rows8, j.j0 = j0, j.blk_dst = dst.first, j.atom_dst = dst.second;
        jobs.push_back(j);
    };
    for (int g = 0; g < G; ++g) {
        Sched &s = S[g];
        s.stream_off = off;
        for (uint32_t l = 0; l < c.n_layers; ++l) {
            const bool rec = (l == 0);
            const uint64_t l0 = off;
            for (uint32_t u = 0; u < s.n_a; ++u) {  // A: QKV units
                const auto [t, b0, b1] = qunits[g][u];
                const uint32_t nrows = std::min(128u, rows_qkv - t * 128), r8 = (nrows + 7) / 8;
                const uint32_t pc = per_chunk(0, r8);
                for (uint32_t b = b0; b < b1; b += pc) {
                    const uint32_t nb = std::min<uint32_t>(pc, b1 - b);
                    auto d = chunk(s, false, PH_QKV, nb, 0, 255, b, u, b != b0, r8, rec);
                    job(in.qkv[l], 1, 0, 0, t * 128, nrows, 2 * b, nb, 0, r8, 0, d);
                }
            }
            {  // B: O pairs, one head per chunk
                const uint32_t bpa = hd / 64, per = std::max(1u, per_chunk(0, 16) / bpa);
                uint32_t i = 0;
                while (i < s.n_pairs) {
                    const uint32_t head = s.pair_head[i];
                    uint32_t j = i;
                    while (j < s.n_pairs && j - i < per && s.pair_head[j] == head) ++j;
                    auto d = chunk(s, false, PH_O, (j - i) * bpa, 0, bpa, (head - s.h0) * bpa, i, false, 16, rec);
                    for (uint32_t q = i; q < j; ++q)
                        job(in.o[l], 0, 0, 0, s.pair_tile[q] * 128, 128, head * hd / 32, bpa, 0, 16, (q - i) * bpa, d);
                    i = j;
                }
            }
            if (s.U) {  // C: gate/up tiles over the concatenation [gate | up], then down
                const uint32_t ngu = (2 * s.U + 127) / 128;
                const uint32_t kb0 = kb64 * s.kh / s.ks, kb1 = kb64 * (s.kh + 1) / s.ks;  // this CTA's K part
                for (uint32_t q = 0; q < ngu; ++q) {
                    const uint32_t nrows = std::min(128u, 2 * s.U - 128 * q), r8 = (nrows + 7) / 8;
                    const uint32_t pc = per_chunk(0, r8);
                    for (uint32_t b = kb0; b < kb1; b += pc) {
                        const uint32_t nb = std::min<uint32_t>(pc, kb1 - b);
                        auto d = chunk(s, false, PH_GU, nb, 0, 255, b, q, b != kb0, r8, rec);
                        job(in.gu[l], 2, s.f0, s.U, 128 * q, nrows, 2 * b, nb, 0, r8, 0, d);
                    }
                }
                const uint8_t km = (s.U % 64) ? 1 : 0;
                const uint32_t bpa = km ? s.U / 32 : s.U / 64, per = std::max(1u, per_chunk(km, 16) / bpa);
                const uint32_t ta = otile * s.kh / s.ks, tb = otile * (s.kh + 1) / s.ks;  // down tiles
                for (uint32_t t0 = ta; t0 < tb; t0 += per) {
                    const uint32_t nt = std::min(per, tb - t0);
                    auto d = chunk(s, false, PH_DOWN, nt * bpa, km, bpa, 0, t0, false, 16, rec);
                    for (uint32_t t = t0; t < t0 + nt; ++t)
                        job(in.down[l], 0, 0, 0, t * 128, 128, s.f0 / 32, bpa, km, 16, (t - t0) * bpa, d);
                }
            }
            if (rec) s.layer_bytes = off - l0;
        }
        const uint64_t m0 = off;
        for (uint32_t i = 0; i < s.n_l; ++i) {
            const uint32_t t = s.l_tile[i], nrows = std::min(128u, c.vocab - t * 128), r8 = (nrows + 7) / 8;
            const uint32_t pc = per_chunk(0, r8);
            for (uint32_t b = 0; b < kb64; b += pc) {
                const uint32_t nb = std::min<uint32_t>(pc, kb64 - b);
                auto d = chunk(s, true, PH_LM, nb, 0, 255, b, i, b != 0, r8, true);
                job(in.lm, 0, 0, 0, t * 128, nrows, 2 * b, nb, 0, r8, 0, d);
            }
        }
        s.lm_bytes = off - m0;
        if (s.n_ops > (uint32_t)kMaxOps || s.n_lm_ops > (uint32_t)kMaxLmOps)
            PTC_UNSUPPORTED("tensor-core decode: too many chunks per CTA");
        // B scale atoms per phase (atom a covers k blocks 2a, 2a + 1 of the operand) as
        // at most two runs; more than two runs are copied as their hull
        uint64_t used[PH_N] = {};
        for (int lmp = 0; lmp < 2; ++lmp) {
            const ChunkOp *ops = lmp ? s.lm_ops : s.ops;
            const uint32_t n = lmp ? s.n_lm_ops : s.n_ops;
            for (uint32_t i = 0; i < n; ++i) {
                const ChunkOp &op = ops[i];
                const uint32_t klast = op.bk0 + std::min<uint32_t>(op.nblk, op.bpa) - 1;
                if ((klast >> 1) >= 64) PTC_UNSUPPORTED("tensor-core decode: operand wider than 64 scale atoms");
                for (uint32_t a = op.bk0 >> 1; a <= (klast >> 1); ++a) used[op.phase] |= 1ull << a;
            }
        }
        for (int ph = 0; ph < PH_N; ++ph) {
            std::vector<std::pair<uint32_t, uint32_t>> runs;  // (start, count)
            for (uint32_t a = 0; a < 64; ++a)
                if ((used[ph] >> a) & 1u) {
                    if (!runs.empty() && runs.back().first + runs.back().second == a) ++runs.back().second;
                    else runs.push_back({a, 1});
                }
            if (runs.size() > 2) runs = {{runs.front().first, runs.back().first + runs.back().second - runs.front().first}};
            for (size_t r = 0; r < runs.size(); ++r)
                s.batoms[ph][2 * r] = (uint8_t)runs[r].first, s.batoms[ph][2 * r + 1] = (uint8_t)runs[r].second;
        }
    }
    // shared and tensor memory
    Params P = {};
    P.n_layers = c.n_layers, P.dim = c.dim, P.ffn = c.ffn, P.n_heads = c.n_heads, P.n_kv = c.n_kv_heads;
    P.hd = hd, P.vocab = c.vocab, P.max_seq = c.max_seq, P.eps = c.eps, P.qd = qd, P.kvd = kvd;
    P.ring_bytes = 0;
    const uint32_t base = smem_layout(P).total;
    const uint32_t room = max_smem > (int)base + 1024 ? (uint32_t)max_smem - base - 1024 : 0;  // ring alignment
    P.ring_bytes = room / 1024 * 1024;
    if (P.ring_bytes < 3 * slot_bytes) PTC_UNSUPPORTED("tensor-core decode: shared memory too small for the weight ring");
    uint32_t nacc = otile;
    for (auto &s : S) nacc = std::max({nacc, s.n_a, s.n_pairs, (2 * s.U + 127) / 128, s.n_l});
    const uint32_t sfb_atoms = std::max({c.dim / 128, (kMaxHeads * hd / 32 + 3) / 4, 2u});
    P.acc_cols = 8 * nacc;
    P.sfb_col0 = P.acc_cols;
    P.sfa_col0 = P.sfb_col0 + 4 * sfb_atoms;
    if (P.sfa_col0 + 16 * 4 > 512) PTC_UNSUPPORTED("tensor-core decode: tensor memory too small");
    P.n_inflight = std::min<uint32_t>(kMaxSlots, (512 - P.sfa_col0) / 16);  // 16 scale columns per chunk
    const uint32_t cols = P.sfa_col0 + 16 * P.n_inflight;
    P.tmem_cols = 32;
    while (P.tmem_cols < cols) P.tmem_cols *= 2;
    if (P.tmem_cols > 512) PTC_UNSUPPORTED("tensor-core decode: %u tensor-memory columns needed", cols);

    Engine *e = new Engine();
    int rc = FP4X_OK;
    uint8_t *arena = nullptr;
    uint32_t *bar = nullptr, *cidx = nullptr;
    Sched *dsched = nullptr;
    PackJob *djobs = nullptr;
    float *X = nullptr, *Y = nullptr, *qkv = nullptr, *cval = nullptr;
    rc = dalloc(e, &arena, off);
    if (!rc) rc = dalloc(e, &dsched, (size_t)G);
    if (!rc) rc = dalloc(e, &bar, 4);
    uint64_t *ffx = nullptr;
    if (!rc && pairs) rc = dalloc(e, &ffx, (size_t)n64 * 2 * 128);
    if (tpin) {  // X, Y and the candidates live in the exchange area
        X = tpin->xr[tpin->rank], Y = tpin->yr[tpin->rank];
    } else {
        if (!rc) rc = dalloc(e, &X, c.dim);
        if (!rc) rc = dalloc(e, &Y, c.dim);
    }
    if (!rc) rc = dalloc(e, &qkv, rows_qkv);
    const uint32_t group = c.n_heads / c.n_kv_heads;
    const uint32_t slices = (group == 2 || group == 4 || group == 8) ? (uint32_t)G / c.n_kv_heads : 0u;
    float *apart = nullptr;
    if (!rc && slices) rc = dalloc(e, &apart, (size_t)c.n_heads * slices * (hd + 2));
    if (tpin) {
        cval = tpin->cvr[tpin->rank], cidx = tpin->cir[tpin->rank];
    } else {
        if (!rc) rc = dalloc(e, &cval, (size_t)G);
        if (!rc) rc = dalloc(e, &cidx, (size_t)G);
    }
    if (!rc) rc = dalloc(e, &djobs, jobs.size());
    if (rc) {
        destroy(e);
        return rc;
    }
    cudaError_t err = cudaMemsetAsync(arena, 0, off, st);
    if (err == cudaSuccess)
        err = cudaMemcpyAsync(dsched, S.data(), S.size() * sizeof(Sched), cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess)
        err = cudaMemcpyAsync(djobs, jobs.data(), jobs.size() * sizeof(PackJob), cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(Y, 0, c.dim * 4, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(qkv, 0, rows_qkv * 4, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(bar, 0, 16, st);
    if (err == cudaSuccess && ffx) err = cudaMemsetAsync(ffx, 0, (size_t)n64 * 2 * 128 * 8, st);  // tag 0: never valid
    for (size_t j0 = 0; j0 < jobs.size() && err == cudaSuccess; j0 += 65535) {
        const unsigned nj = (unsigned)std::min<size_t>(65535, jobs.size() - j0);
        pack_kernel<<<nj, 256, 0, st>>>(djobs + j0, arena);
        err = cudaGetLastError();
    }
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);  // the host job table goes away
    if (err != cudaSuccess) {
        destroy(e);
        return fail("build", err);
    }
    cudaFree(djobs);
    e->allocs.pop_back();
    P.arena = arena, P.sched = dsched;
    P.attn_norm = in.attn_norm, P.ffn_norm = in.ffn_norm, P.final_norm = in.final_norm;
    P.embed = in.embed, P.cos_t = in.cos_t, P.sin_t = in.sin_t, P.kc = in.kc, P.vc = in.vc;
    P.X = X, P.Y = Y, P.qkv = qkv, P.logits = in.logits, P.cand_val = cval, P.cand_idx = cidx;
    P.attn_part = apart, P.attn_slices = slices;
    P.ffx = ffx, P.launch_seq = 0;
    P.tp_rank = 0, P.tp_size = 1, P.v0 = 0, P.epoch = nullptr;
    P.xr[0] = X, P.yr[0] = Y, P.cvr[0] = cval, P.cir[0] = cidx;
    if (tpin) {
        P.tp_rank = tpin->rank, P.tp_size = tpin->size, P.v0 = tpin->v0, P.epoch = tpin->epoch;
        for (uint32_t r = 0; r < tpin->size; ++r) {
            P.xr[r] = tpin->xr[r], P.yr[r] = tpin->yr[r], P.cvr[r] = tpin->cvr[r], P.cir[r] = tpin->cir[r];
            P.flagr[r] = tpin->flagr[r];
            P.tro[r] = tpin->ro[r], P.trd[r] = tpin->rd[r];
        }
        P.tpo = tpin->po, P.tpd = tpin->pd, P.xepoch = tpin->xepoch;
    }
    P.state = in.state, P.prompt = in.prompt, P.out = in.out, P.bar = bar, P.n_tokens = 0;
    e->p = P;
    e->grid = G;
    e->smem = smem_layout(P).total;
    e->arena_bytes = off;
    err = cudaFuncSetAttribute(decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)e->smem);
    int per_sm = 0;
    if (err == cudaSuccess)
        err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_tc_kernel, kThreads, e->smem);
    if (err != cudaSuccess || per_sm < 1) {
        cudaFuncAttributes fa = {};
        cudaFuncGetAttributes(&fa, decode_tc_kernel);
        const size_t smem = e->smem;
        destroy(e);
        if (err != cudaSuccess) return fail("occupancy", err);
        PTC_UNSUPPORTED("tensor-core decode: kernel does not fit one CTA per SM (%d threads, %d regs, %zu B shared)",
                        kThreads, fa.numRegs, smem);
    }
    *out = e;
    return FP4X_OK;
}

#ifdef FP4X_PHASE_TIMING
extern "C" FP4X_API int fp4x_tc_timestamps(unsigned long long *out, uint32_t n) {
    n = std::min<uint32_t>(n, 2 * kTcStamps);
    return cudaMemcpyFromSymbol(out, g_tc_ts, n * sizeof(unsigned long long)) == cudaSuccess ? 0 : 2;
}
extern "C" FP4X_API int fp4x_tc_mma_timestamps(unsigned long long *out, uint32_t n) {
    n = std::min<uint32_t>(n, 2 * kMts);
    return cudaMemcpyFromSymbol(out, g_tc_mts, n * sizeof(unsigned long long)) == cudaSuccess ? 0 : 2;
}
#endif

int launch(Engine *e, cudaStream_t st, uint32_t n_tokens) {
    if (n_tokens == 0) return FP4X_OK;
    cudaError_t err = cudaMemsetAsync(e->p.bar, 0, 16, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(e->p.qkv, 0, (e->p.qd + 2 * e->p.kvd) * 4, st);
    if (err != cudaSuccess) return fail("reset", err);
    Params p = e->p;
    p.n_tokens = n_tokens;
    p.launch_seq = e->launches++ % 4095u + 1u;  // 1..4095: 12 bits above the FFN split tags' barrier count
    void *args[] = {&p};
    err = cudaLaunchCooperativeKernel((const void *)decode_tc_kernel, dim3(e->grid), dim3(kThreads), args, e->smem, st);
    if (err != cudaSuccess) return fail("cooperative launch", err);
    return FP4X_OK;
}

}  // namespace ptc
}  // namespace fp4x
