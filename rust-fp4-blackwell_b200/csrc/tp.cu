// tp.cu -- tensor parallelism for the decode graph: the
// exchange area every rank shares over NVLink, the row-parallel allreduce that
// follows the O and down projections (llama_run/src/main.rs:522-530 with the
// contraction split across ranks), and the vocab-parallel argmax.
//
// One process per GPU.  Each rank cudaMallocs an exchange area and exports it with
// CUDA IPC; after the host has passed every rank's handle to every rank
// (llama_model_tp_connect), rank r maps the others' areas and its kernels write
// straight into them with peer stores:
//   area = slots[2][kMaxRanks][dim] f32 | flags[2][kMaxRanks] u32 |
//          argv[2][kMaxRanks] f32 | argi[2][kMaxRanks] u32 | aflags[2][kMaxRanks] u32
// Exchange number n (a per-rank device counter; every rank runs the same sequence)
// uses phase n & 1 and epoch n / 2 + 1: rank r stores its vector into slot
// [phase][r] of every area, fences at system scope, raises flag [phase][r] to the
// epoch everywhere, waits (bounded) until all flags of its own area reach the epoch,
// and sums the slots in rank order, so every rank gets the same bits.  Two phases
// suffice: rank r reaches exchange n+2 only after every rank finished n+1, hence
// after every rank finished reading the phase of n.  No multicast object and no
// library collective is involved.
#include "common.cuh"

#include <algorithm>
#include <cstring>

namespace fp4x {
namespace tp {

constexpr uint32_t kMaxRanks = 8;
constexpr uint32_t kThreads = 1024;

struct Peers {
    uint8_t *area[kMaxRanks];
};

constexpr uint32_t kMaxCtas = 256;  // argmax candidates per rank (persistent kernel)

// Exchange area of one rank.  The graph path uses slots/flags/arg*; the tensor-core
// persistent kernel keeps its residual X, FFN delta Y, argmax candidates and
// barrier flags here so that every rank can add into / write them with peer stores.
struct Layout {
    size_t slots, flags, argv, argi, aflags, px, py, pcv, pci, pflag, pro, prd, ppo, ppd, total;
};

__host__ __device__ inline Layout layout(uint32_t dim) {
    Layout L;
    L.slots = 0;
    L.flags = (size_t)2 * kMaxRanks * dim * 4;
    L.argv = L.flags + 2 * kMaxRanks * 4;
    L.argi = L.argv + 2 * kMaxRanks * 4;
    L.aflags = L.argi + 2 * kMaxRanks * 4;
    L.px = (L.aflags + 2 * kMaxRanks * 4 + 255) / 256 * 256;
    L.py = L.px + (size_t)dim * 4;
    L.pcv = L.py + (size_t)dim * 4;
    L.pci = L.pcv + (size_t)kMaxRanks * kMaxCtas * 4;
    L.pflag = L.pci + (size_t)kMaxRanks * kMaxCtas * 4;  // one 128-byte line per source rank
    // tensor-core kernel's row-parallel exchange: receive slots [2 parities][source
    // rank][dim] of tagged 64-bit words for the O and down partials, and this rank's
    // own partial accumulators
    L.pro = (L.pflag + (size_t)kMaxRanks * 128 + 255) / 256 * 256;
    L.prd = L.pro + (size_t)2 * kMaxRanks * dim * 8;
    L.ppo = L.prd + (size_t)2 * kMaxRanks * dim * 8;
    L.ppd = L.ppo + (size_t)dim * 4;
    L.total = (L.ppd + (size_t)dim * 4 + 255) / 256 * 256;
    return L;
}

struct Exchange {
    uint32_t rank = 0, size = 1, dim = 0;
    uint8_t *local = nullptr;  // this rank's area (exported)
    Peers peers = {};          // every rank's area in this process (peers[rank] = local)
    uint32_t *count = nullptr; // completed exchanges (device); [1] = persistent-kernel barrier epoch
    bool connected = false;
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Threads [0, size) wait until flag[src] >= epoch (bounded); returns false on timeout.
__device__ bool wait_flags(const uint32_t *flags, uint32_t size, uint32_t epoch) {
    __shared__ uint32_t ok;
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    if (threadIdx.x < size) {
        const uint32_t lim = flag_wait_limit(kSpinLimit);
        uint32_t i = 0;
        while (ld_acquire_sys(flags + threadIdx.x) < epoch) {
            if (++i > lim) {
                raise_device_error(DEVERR_FLAG_TIMEOUT);
                ok = 0;
                break;
            }
            __nanosleep(100);
        }
    }
    __syncthreads();
    return ok != 0;
}

// x[i] += sum over ranks of part[i] (rank order), with the residual folded in.
__global__ void __launch_bounds__(kThreads) allreduce_add_kernel(Peers peers, const float *__restrict__ part,
                                                                 float *__restrict__ x, uint32_t dim,
                                                                 uint32_t *count, uint32_t rank, uint32_t size) {
    pdl_launch_dependents();
    pdl_wait();
    const Layout L = layout(dim);
    const uint32_t n = *count, phase = n & 1u, epoch = n / 2 + 1;
    for (uint32_t i = threadIdx.x * 4; i < dim; i += kThreads * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(part + i);
        for (uint32_t p = 0; p < size; ++p)
            *reinterpret_cast<float4 *>(peers.area[p] + L.slots + ((size_t)(phase * kMaxRanks + rank) * dim + i) * 4) =
                v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (uint32_t p = 0; p < size; ++p)
            st_release_sys(reinterpret_cast<uint32_t *>(peers.area[p] + L.flags) + phase * kMaxRanks + rank, epoch);
    }
    const uint8_t *mine = peers.area[rank];
    const bool ok = wait_flags(reinterpret_cast<const uint32_t *>(mine + L.flags) + phase * kMaxRanks, size, epoch);
    if (ok)
        for (uint32_t i = threadIdx.x * 4; i < dim; i += kThreads * 4) {
            float4 acc = *reinterpret_cast<const float4 *>(x + i);
            for (uint32_t s = 0; s < size; ++s) {
                const float4 v = __ldcg(reinterpret_cast<const float4 *>(
                    mine + L.slots + ((size_t)(phase * kMaxRanks + s) * dim + i) * 4));
                acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
            }
            *reinterpret_cast<float4 *>(x + i) = acc;
        }
    __syncthreads();
    if (threadIdx.x == 0) *count = n + 1;
}

__device__ __forceinline__ void argmax_merge(float &bv, uint32_t &bi, float ov, uint32_t oi) {
    if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
    }
}

// Argmax over this rank's vocab slice [v0, v0 + n), exchange of (value, index)
// with every rank, global argmax (larger value, ties to the lower index,
// llama_run/src/main.rs:263-315), then the loop-state advance of
// llama_run/src/main.rs:550-566 (every rank computes the same next token).
__global__ void __launch_bounds__(kThreads) argmax_advance_kernel(Peers peers, uint32_t dim, uint32_t n, uint32_t v0,
                                                                  const float *__restrict__ logits, uint32_t *count,
                                                                  uint32_t rank, uint32_t size,
                                                                  uint32_t *__restrict__ state,
                                                                  const uint32_t *__restrict__ prompt,
                                                                  uint32_t *__restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float mv[32];
    __shared__ uint32_t mi[32];
    const Layout L = layout(dim);
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) argmax_merge(bv, bi, logits[i], v0 + i);
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) mv[warp] = bv, mi[warp] = bi;
    __syncthreads();
    const uint32_t c = *count, phase = c & 1u, epoch = c / 2 + 1;
    if (threadIdx.x == 0) {
        float gv = -INFINITY;
        uint32_t gi = 0xFFFFFFFFu;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) argmax_merge(gv, gi, mv[w], mi[w]);
        for (uint32_t p = 0; p < size; ++p) {
            reinterpret_cast<float *>(peers.area[p] + L.argv)[phase * kMaxRanks + rank] = gv;
            reinterpret_cast<uint32_t *>(peers.area[p] + L.argi)[phase * kMaxRanks + rank] = gi;
        }
        __threadfence_system();
        for (uint32_t p = 0; p < size; ++p)
            st_release_sys(reinterpret_cast<uint32_t *>(peers.area[p] + L.aflags) + phase * kMaxRanks + rank, epoch);
    }
    const uint8_t *mine = peers.area[rank];
    const bool ok = wait_flags(reinterpret_cast<const uint32_t *>(mine + L.aflags) + phase * kMaxRanks, size, epoch);
    if (threadIdx.x == 0) {
        float gv = -INFINITY;
        uint32_t gi = 0;
        if (ok)
            for (uint32_t s = 0; s < size; ++s)
                argmax_merge(gv, gi, __ldcg(reinterpret_cast<const float *>(mine + L.argv) + phase * kMaxRanks + s),
                             __ldcg(reinterpret_cast<const uint32_t *>(mine + L.argi) + phase * kMaxRanks + s));
        const uint32_t pos = state[1], n_prompt = state[3], cap = state[4];
        state[2] = gi;
        if (pos + 1 >= n_prompt && pos + 1 - n_prompt < cap) out[pos + 1 - n_prompt] = gi;
        state[0] = (pos + 1 < n_prompt) ? prompt[pos + 1] : gi;
        state[1] = pos + 1;
        *count = c + 1;
    }
}

// ---------------------------------------------------------------- batched engine
// A batch exchange area of one rank (the batched engine's row-parallel outputs
// [rows][dim] and per-row argmax candidates):
//   slots[2][kMaxRanks][n_max] f32 | flags[2][kMaxRanks][kRowChunks] u32 |
//   argv[2][kMaxRanks][kMaxRows] f32 | argi[...] u32 | aflags[...] u32
// Counters (device, this rank): [0] allreduces done, [1] argmax exchanges done,
// [2]/[3] CTAs finished in the current allreduce / argmax.  Same phase/epoch
// protocol as the single-vector exchange; every CTA owns one chunk of the vector
// (allreduce) or one row (argmax) and waits only for the other ranks' copies of
// it.  A kernel of exchange n + 1 runs only after this rank's kernel of exchange
// n completed (stream order), so a rank that has seen exchange n + 1 flags of a
// peer knows the peer has finished reading the slots of exchange n.
constexpr uint32_t kRowChunks = 128;
constexpr uint32_t kMaxRows = 256;

struct RowLayout {
    size_t slots, flags, argv, argi, aflags, total;
};

__host__ __device__ inline RowLayout row_layout(size_t n_max) {
    RowLayout L;
    L.slots = 0;
    L.flags = 2 * kMaxRanks * n_max * 4;
    L.argv = L.flags + 2 * kMaxRanks * kRowChunks * 4;
    L.argi = L.argv + 2 * kMaxRanks * kMaxRows * 4;
    L.aflags = L.argi + 2 * kMaxRanks * kMaxRows * 4;
    L.total = (L.aflags + 2 * kMaxRanks * kMaxRows * 4 + 255) / 256 * 256;
    return L;
}

struct RowExchange {
    uint32_t rank = 0, size = 1;
    size_t n_max = 0;
    uint8_t *local = nullptr;
    Peers peers = {};
    uint32_t *count = nullptr;
    bool connected = false;
};

// The CTA that finishes last advances exchange counter `which` (and clears the
// CTA count `which + 2`).
__device__ __forceinline__ void finish_exchange(uint32_t *count, uint32_t which, uint32_t n) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&count[which + 2], 1u) == gridDim.x - 1) {
            count[which + 2] = 0;
            count[which] = n + 1;
        }
    }
}

// x[i] += sum over ranks of part[i] (rank order) for i < n; CTA c owns chunk c.
__global__ void __launch_bounds__(512) rows_allreduce_kernel(Peers peers, const float *__restrict__ part,
                                                             float *__restrict__ x, size_t n, size_t n_max,
                                                             uint32_t *count, uint32_t rank, uint32_t size) {
    const RowLayout L = row_layout(n_max);
    const uint32_t e = count[0], phase = e & 1u, epoch = e / 2 + 1, c = blockIdx.x;
    const size_t per = ((n + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
    const size_t i0 = (size_t)c * per, i1 = i0 + per < n ? i0 + per : n;
    for (size_t i = i0 + threadIdx.x * 4; i < i1; i += blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(part + i);
        for (uint32_t p = 0; p < size; ++p)
            *reinterpret_cast<float4 *>(peers.area[p] + L.slots + ((size_t)(phase * kMaxRanks + rank) * n_max + i) * 4) =
                v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (uint32_t p = 0; p < size; ++p)
            st_release_sys(reinterpret_cast<uint32_t *>(peers.area[p] + L.flags) + (phase * kMaxRanks + rank) * kRowChunks + c,
                           epoch);
    }
    const uint8_t *mine = peers.area[rank];
    __shared__ uint32_t ok;
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    if (threadIdx.x < size) {
        const uint32_t *f = reinterpret_cast<const uint32_t *>(mine + L.flags) + (phase * kMaxRanks + threadIdx.x) * kRowChunks + c;
        const uint32_t lim = flag_wait_limit(kSpinLimit);
        for (uint32_t it = 0; ld_acquire_sys(f) < epoch; ++it) {
            if (it > lim) {
                raise_device_error(DEVERR_FLAG_TIMEOUT);
                ok = 0;
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    if (ok)
        for (size_t i = i0 + threadIdx.x * 4; i < i1; i += blockDim.x * 4) {
            float4 acc = *reinterpret_cast<const float4 *>(x + i);
            for (uint32_t r = 0; r < size; ++r) {
                const float4 v = __ldcg(reinterpret_cast<const float4 *>(
                    mine + L.slots + ((size_t)(phase * kMaxRanks + r) * n_max + i) * 4));
                acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
            }
            *reinterpret_cast<float4 *>(x + i) = acc;
        }
    finish_exchange(count, 0, e);
}

// Per logits row r of this rank's vocab slice [v0, v0 + vocab): local argmax,
// exchange of (value, index) with every rank, global argmax (ties to the lower
// index, llama_run/src/main.rs:263-315).  Decode (seq == ~0u): row r is
// sequence r: ids[r][pos + 1] = next, dec_tok[r] = next, dec_pos[r] += 1.
// Prefill: the single row belongs to sequence `seq` with next position next_pos.
__global__ void __launch_bounds__(1024) rows_argmax_kernel(Peers peers, size_t n_max, uint32_t vocab, uint32_t v0,
                                                           const float *__restrict__ logits, uint32_t *count,
                                                           uint32_t rank, uint32_t size, uint32_t *dec_tok,
                                                           uint32_t *dec_pos, uint32_t *ids, uint32_t max_seq,
                                                           uint32_t seq, uint32_t next_pos) {
    __shared__ float mv[32];
    __shared__ uint32_t mi[32];
    __shared__ uint32_t ok;
    const RowLayout L = row_layout(n_max);
    const uint32_t e = count[1], phase = e & 1u, epoch = e / 2 + 1, r = blockIdx.x;
    const float *lg = logits + (size_t)r * vocab;
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) argmax_merge(bv, bi, lg[i], v0 + i);
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) mv[warp] = bv, mi[warp] = bi;
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    const size_t slot = (size_t)(phase * kMaxRanks + rank) * kMaxRows + r;
    if (threadIdx.x == 0) {
        float gv = -INFINITY;
        uint32_t gi = 0xFFFFFFFFu;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) argmax_merge(gv, gi, mv[w], mi[w]);
        for (uint32_t p = 0; p < size; ++p) {
            reinterpret_cast<float *>(peers.area[p] + L.argv)[slot] = gv;
            reinterpret_cast<uint32_t *>(peers.area[p] + L.argi)[slot] = gi;
        }
        __threadfence_system();
        for (uint32_t p = 0; p < size; ++p) st_release_sys(reinterpret_cast<uint32_t *>(peers.area[p] + L.aflags) + slot, epoch);
    }
    const uint8_t *mine = peers.area[rank];
    if (threadIdx.x < size) {
        const uint32_t *f =
            reinterpret_cast<const uint32_t *>(mine + L.aflags) + (size_t)(phase * kMaxRanks + threadIdx.x) * kMaxRows + r;
        const uint32_t lim = flag_wait_limit(kSpinLimit);
        for (uint32_t it = 0; ld_acquire_sys(f) < epoch; ++it) {
            if (it > lim) {
                raise_device_error(DEVERR_FLAG_TIMEOUT);
                ok = 0;
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && ok) {
        float gv = -INFINITY;
        uint32_t gi = 0;
        for (uint32_t s = 0; s < size; ++s) {
            const size_t o = (size_t)(phase * kMaxRanks + s) * kMaxRows + r;
            argmax_merge(gv, gi, __ldcg(reinterpret_cast<const float *>(mine + L.argv) + o),
                         __ldcg(reinterpret_cast<const uint32_t *>(mine + L.argi) + o));
        }
        const uint32_t sq = seq == ~0u ? r : seq;
        const uint32_t np = seq == ~0u ? dec_pos[sq] + 1 : next_pos;
        if (np < max_seq) {
            ids[(size_t)sq * max_seq + np] = gi;
            dec_tok[sq] = gi;
            dec_pos[sq] = np;
        }
    }
    finish_exchange(count, 1, e);
}

// ---------------------------------------------------------------- host

int create(Exchange **out, uint32_t rank, uint32_t size, uint32_t dim) {
    FP4X_REQUIRE(size >= 2 && size <= kMaxRanks && rank < size, "tensor parallel: rank %u of %u (2..%u ranks)", rank,
                 size, kMaxRanks);
    FP4X_REQUIRE(dim % 4 == 0, "tensor parallel: dim %u %% 4 != 0", dim);
    Exchange *x = new Exchange();
    x->rank = rank, x->size = size, x->dim = dim;
    const size_t bytes = layout(dim).total;
    cudaError_t e = cudaMalloc(&x->local, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&x->count, 16);
    if (e == cudaSuccess) e = cudaMemset(x->local, 0, bytes);
    if (e == cudaSuccess) e = cudaMemset(x->count, 0, 16);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any peer can see the handle
    if (e != cudaSuccess) {
        if (x->local) cudaFree(x->local);
        if (x->count) cudaFree(x->count);
        delete x;
        set_error("tensor parallel: exchange area: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    x->peers.area[rank] = x->local;
    *out = x;
    return FP4X_OK;
}

void destroy(Exchange *x) {
    if (!x) return;
    for (uint32_t p = 0; p < x->size; ++p)
        if (p != x->rank && x->peers.area[p]) cudaIpcCloseMemHandle(x->peers.area[p]);
    if (x->local) cudaFree(x->local);
    if (x->count) cudaFree(x->count);
    delete x;
}

int export_handle(Exchange *x, void *handle64) {
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, x->local);
    if (e != cudaSuccess) {
        set_error("tensor parallel: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(handle64, &h, sizeof(h));
    return FP4X_OK;
}

int connect(Exchange *x, const void *handles) {
    FP4X_REQUIRE(!x->connected, "tensor parallel: already connected");
    for (uint32_t p = 0; p < x->size; ++p) {
        if (p == x->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t *>(handles) + 64 * p, 64);
        void *ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            set_error("tensor parallel: cudaIpcOpenMemHandle(rank %u): %s", p, cudaGetErrorString(e));
            return FP4X_ECUDA;
        }
        x->peers.area[p] = static_cast<uint8_t *>(ptr);
    }
    x->connected = true;
    return FP4X_OK;
}

// Where the tensor-core persistent kernel finds every rank's X, Y, argmax
// candidates and barrier flags (inside the exchange areas), and its epoch word.
void ptc_buffers(const Exchange *x, ptc::TpIn &t) {
    const Layout L = layout(x->dim);
    t.rank = x->rank, t.size = x->size;
    for (uint32_t r = 0; r < x->size; ++r) {
        uint8_t *base = x->peers.area[r];
        t.xr[r] = reinterpret_cast<float *>(base + L.px);
        t.yr[r] = reinterpret_cast<float *>(base + L.py);
        t.cvr[r] = reinterpret_cast<float *>(base + L.pcv);
        t.cir[r] = reinterpret_cast<uint32_t *>(base + L.pci);
        t.flagr[r] = reinterpret_cast<uint32_t *>(base + L.pflag);
        t.ro[r] = reinterpret_cast<uint64_t *>(base + L.pro);
        t.rd[r] = reinterpret_cast<uint64_t *>(base + L.prd);
    }
    t.po = reinterpret_cast<float *>(x->local + L.ppo);
    t.pd = reinterpret_cast<float *>(x->local + L.ppd);
    t.epoch = x->count + 1;
    t.xepoch = x->count + 2;
}

static int launch_cfg(cudaStream_t st, bool pdl, cudaLaunchConfig_t &cfg, cudaLaunchAttribute *attr) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return FP4X_OK;
}

int allreduce_add(cudaStream_t st, Exchange *x, const float *part, float *y, bool pdl) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[1];
    launch_cfg(st, pdl, cfg, attr);
    const cudaError_t e =
        cudaLaunchKernelEx(&cfg, allreduce_add_kernel, x->peers, part, y, x->dim, x->count, x->rank, x->size);
    if (e != cudaSuccess) {
        set_error("tensor parallel allreduce: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    return FP4X_OK;
}

int argmax_advance(cudaStream_t st, Exchange *x, uint32_t n, uint32_t v0, const float *logits, uint32_t *state,
                   const uint32_t *prompt, uint32_t *out, bool pdl) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[1];
    launch_cfg(st, pdl, cfg, attr);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, argmax_advance_kernel, x->peers, x->dim, n, v0, logits, x->count,
                                             x->rank, x->size, state, prompt, out);
    if (e != cudaSuccess) {
        set_error("tensor parallel argmax: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    return FP4X_OK;
}

int row_create(RowExchange **out, uint32_t rank, uint32_t size, size_t n_max) {
    FP4X_REQUIRE(size >= 2 && size <= kMaxRanks && rank < size, "tensor parallel: rank %u of %u (2..%u ranks)", rank,
                 size, kMaxRanks);
    RowExchange *x = new RowExchange();
    x->rank = rank, x->size = size, x->n_max = (n_max + 3) / 4 * 4;
    const size_t bytes = row_layout(x->n_max).total;
    cudaError_t e = cudaMalloc(&x->local, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&x->count, 16);
    if (e == cudaSuccess) e = cudaMemset(x->local, 0, bytes);
    if (e == cudaSuccess) e = cudaMemset(x->count, 0, 16);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (x->local) cudaFree(x->local);
        if (x->count) cudaFree(x->count);
        delete x;
        set_error("tensor parallel: batch exchange area: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    x->peers.area[rank] = x->local;
    *out = x;
    return FP4X_OK;
}

void row_destroy(RowExchange *x) {
    if (!x) return;
    for (uint32_t p = 0; p < x->size; ++p)
        if (p != x->rank && x->peers.area[p]) cudaIpcCloseMemHandle(x->peers.area[p]);
    if (x->local) cudaFree(x->local);
    if (x->count) cudaFree(x->count);
    delete x;
}

int row_export_handle(RowExchange *x, void *handle64) {
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, x->local);
    if (e != cudaSuccess) {
        set_error("tensor parallel: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    memcpy(handle64, &h, sizeof(h));
    return FP4X_OK;
}

int row_connect(RowExchange *x, const void *handles) {
    FP4X_REQUIRE(!x->connected, "tensor parallel: batch exchange already connected");
    for (uint32_t p = 0; p < x->size; ++p) {
        if (p == x->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t *>(handles) + 64 * p, 64);
        void *ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            set_error("tensor parallel: cudaIpcOpenMemHandle(rank %u): %s", p, cudaGetErrorString(e));
            return FP4X_ECUDA;
        }
        x->peers.area[p] = static_cast<uint8_t *>(ptr);
    }
    x->connected = true;
    return FP4X_OK;
}

int rows_allreduce_add(cudaStream_t st, RowExchange *x, const float *part, float *y, size_t n) {
    FP4X_REQUIRE(n <= x->n_max && n % 4 == 0, "tensor parallel: allreduce of %zu values (at most %zu)", n, x->n_max);
    const uint32_t ctas = (uint32_t)std::min<size_t>(kRowChunks, std::max<size_t>(1, (n + 2047) / 2048));
    rows_allreduce_kernel<<<ctas, 512, 0, st>>>(x->peers, part, y, n, x->n_max, x->count, x->rank, x->size);
    return check_launch("tensor parallel batch allreduce");
}

int rows_argmax(cudaStream_t st, RowExchange *x, uint32_t rows, uint32_t vocab, uint32_t v0, const float *logits,
                uint32_t *dec_tok, uint32_t *dec_pos, uint32_t *ids, uint32_t max_seq, uint32_t seq,
                uint32_t next_pos) {
    FP4X_REQUIRE(rows >= 1 && rows <= kMaxRows, "tensor parallel: %u argmax rows", rows);
    rows_argmax_kernel<<<rows, 1024, 0, st>>>(x->peers, x->n_max, vocab, v0, logits, x->count, x->rank, x->size,
                                              dec_tok, dec_pos, ids, max_seq, seq, next_pos);
    return check_launch("tensor parallel batch argmax");
}

}  // namespace tp
}  // namespace fp4x
