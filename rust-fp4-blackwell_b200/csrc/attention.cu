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
    const uint32_t seq = p.pos_ptr ? min(*p.pos_ptr + 1, p.max_seq) : p.seq;
    const uint32_t t_begin = split * p.split_len, t_end = min(seq, t_begin + p.split_len);
    if (t_begin >= seq) return;  // slice past the current position (whole CTA, before any barrier)

    const QT *q = reinterpret_cast<const QT *>(p.q) + ((size_t)b * p.n_heads + h0) * HD;
    for (uint32_t i = tid; i < H * HD; i += kThreads) qs[i / HD][i % HD] = to_f32(q[i]) * p.scale;
    __syncthreads();

    const size_t row_stride = (size_t)p.n_kv * HD;
    const KT *kbase = reinterpret_cast<const KT *>(p.kc) + (size_t)b * p.max_seq * row_stride + (size_t)kvh * HD;
    const KT *vbase = reinterpret_cast<const KT *>(p.vc) + (size_t)b * p.max_seq * row_stride + (size_t)kvh * HD;

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

// grid = (n_heads, batch), block = HD: merge the slices of one (b, head).
template <int HD, typename OT>
__global__ void attn_combine_kernel(Params p) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const size_t bh = (size_t)b * p.n_heads + h;
    const float *rec = p.ws + bh * p.splits * (HD + 2);
    const uint32_t seq = p.pos_ptr ? min(*p.pos_ptr + 1, p.max_seq) : p.seq;
    const uint32_t used = (seq + p.split_len - 1) / p.split_len;
    float M = -INFINITY;
    for (uint32_t s = 0; s < used; ++s) M = fmaxf(M, rec[s * (HD + 2)]);
    float L = 0.0f, O = 0.0f;
    for (uint32_t s = 0; s < used; ++s) {
        const float *r = rec + s * (HD + 2);
        const float f = __expf(r[0] - M);
        L += r[1] * f;
        O += r[2 + d] * f;
    }
    store_out(reinterpret_cast<OT *>(p.out) + bh * HD + d, O / L);
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

// Slices so that batch * head-groups * slices covers the SMs ~4x, each slice >= 128 tokens.
uint32_t choose_splits(uint32_t batch, uint32_t groups, uint32_t seq) {
    const uint32_t ctas = batch * groups;
    const uint32_t target = (uint32_t)num_sms() * 4;
    uint32_t s = std::max<uint32_t>(1, (target + ctas - 1) / ctas);
    s = std::min<uint32_t>(s, std::max<uint32_t>(1, seq / 128));
    return std::min<uint32_t>(s, 256);
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
        splits = choose_splits(batch, n_heads / hpc, seq);
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
#define FP4X_ATTN_CASE(HD_, HPC_)                                                                       \
    if (hd == HD_ && hpc == HPC_) {                                                                   \
        attn_split_kernel<HD_, HPC_, QT, KT, OT><<<grid, kThreads, 0, stream>>>(p);                   \
        if (p.splits > 1) attn_combine_kernel<HD_, OT><<<dim3(n_heads, batch), HD_, 0, stream>>>(p); \
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
    cudaError_t e = cudaLaunchKernelEx(&cfg, attn_split_kernel<HD, HPC, float, uint16_t, float>, p);
    if (e == cudaSuccess && p.splits > 1) {
        cudaLaunchConfig_t c2 = cfg;
        c2.gridDim = dim3(p.n_heads, p.batch);
        c2.blockDim = dim3(HD);
        e = cudaLaunchKernelEx(&c2, attn_combine_kernel<HD, float>, p);
    }
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
    return attn::workspace_bytes(batch, n_heads, head_dim, attn::choose_splits(batch, n_heads / hpc, seq));
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
// host-side stand-in, so its device address is looked up once per device with
// cudaGetSymbolAddress (on the first call made with that device current; make
// that first call before any stream capture) and cached.
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

constexpr int kNoAllocMaxDevices = 64;
static float *g_noalloc_ptr[kNoAllocMaxDevices] = {};
static std::mutex g_noalloc_mu;

static int noalloc_scratch(float **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_error("llama_attn_decode_bf16_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    FP4X_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, "llama_attn_decode_bf16_noalloc: device %d out of range",
                 dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            set_error("llama_attn_decode_bf16_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
            return FP4X_ECUDA;
        }
        g_noalloc_ptr[dev] = static_cast<float *>(p);
    }
    *out = g_noalloc_ptr[dev];
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
