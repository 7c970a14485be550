// engine.cu -- the Llama decode engine: model handle, random-init weights,
// one captured CUDA graph per token, device-resident token loop.
//
// Replaces the drivers of the reference: forward(tok, pos) -> u32 of
// examples/llama_run/src/main.rs:492-536 with its generation loop :544-587, and
// decode_step of examples/llama_decode/src/main.rs:428-477.  The reference
// issues 22 x 17 + 3 = 377 launches per token from the host, uploads the
// embedding row (H2D, :509-510) and reads the argmax back (D2H, :535) every
// token.  Here one token is one CUDA graph of fused kernels per layer:
//   1. RMSNorm + QKV GEMV + RoPE + bf16 KV append   (layer 0 also gathers the
//      embedding row of the device-resident token)
//   2. split-KV GQA attention (+ combine)
//   3. O GEMV + residual add
//   4. RMSNorm + gate/up GEMV + SwiGLU
//   5. down GEMV + residual add
// then RMSNorm + lm_head GEMV and one argmax kernel that also advances the
// device-resident (token, position) pair, so a whole generation is graph
// replays with no host round trip.  Kernels are chained with programmatic
// dependent launch: each GEMV starts streaming its weights while its
// predecessor finishes.
#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

namespace fp4x {
namespace quant {
int init_mxfp4_rowmap(cudaStream_t stream, uint64_t seed, float sigma, uint32_t n, uint32_t k, uint8_t *packed,
                      uint8_t *scales, int mode, uint32_t off, uint32_t hd, uint32_t row0 = 0, uint32_t k_global = 0,
                      uint32_t col0 = 0);
}
}  // namespace fp4x

// Tensor ids of the synthetic initialiser (shared with the oracle): the tensor
// seed is hash64(model seed, id).
enum { T_EMBED = 0, T_LMHEAD = 1, T_LAYER0 = 16 };
enum { M_Q = 0, M_K, M_V, M_O, M_GATE, M_UP, M_DOWN, M_COUNT };

struct QMat {
    uint8_t *w = nullptr;
    uint8_t *s = nullptr;
    uint32_t n = 0, k = 0;
};

struct LayerW {
    QMat qkv, o, gu, down;
    float *attn_norm = nullptr, *ffn_norm = nullptr;
    uint16_t *kc = nullptr, *vc = nullptr;
};

struct fp4x_llama_model {
    fp4x_llama_config cfg;  // the whole model
    fp4x_llama_config lc;   // this rank's shard: n_heads, n_kv_heads, ffn, vocab per rank (== cfg without TP)
    uint32_t v0 = 0;        // first vocab row of this rank's lm_head shard
    float *part = nullptr;  // row-parallel partial outputs [dim] (tensor parallel)
    fp4x::tp::Exchange *xc = nullptr;
    int device = 0;
    std::vector<void *> allocs;
    std::vector<LayerW> layers;
    QMat lm_head;
    uint16_t *embed = nullptr;
    float *final_norm = nullptr;
    float *cos_t = nullptr, *sin_t = nullptr;
    // activations
    float *x = nullptr, *q = nullptr, *att = nullptr, *s = nullptr, *logits = nullptr, *ws = nullptr;
    uint32_t *state = nullptr;  // [0] tok, [1] pos, [2] next, [3] n_prompt, [4] out capacity
    uint32_t *prompt = nullptr, *out = nullptr;
    uint32_t attn_split_len = 64, attn_splits = 1;
    cudaStream_t cap_stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    bool pdl = true;
    // contiguous [n_layers][...] blocks shared by both decode paths
    float *norms = nullptr;        // attn norms [L][dim] then ffn norms [L][dim]
    uint16_t *kv = nullptr;        // K [L][max_seq][kvd] then V [L][max_seq][kvd]
    fp4x::persist::Engine *pe = nullptr;  // persistent decode kernel (null: unsupported shape)
    fp4x::ptc::Engine *pt = nullptr;      // tensor-core persistent decode kernel (null: unsupported)
    fp4x_llama_batch *pf = nullptr;        // prompt prefill through the batched engine (created on first use)
    int path = 0;                  // 0: CUDA graph of fused kernels, 1: persistent kernel (CUDA-core
                                   // MXFP4 decode), 2: persistent kernel on tcgen05 MMAs
    int64_t hpos = -1;             // host view of the device-resident position (-1: unknown)
    char persist_why[256] = "";    // why the persistent kernel is unavailable, if it is
    char tc_why[256] = "";         // why the tensor-core kernel is unavailable, if it is
};

namespace fp4x {
namespace batch {
void destroy(fp4x_llama_batch *b);                                                        // batch.cu
int model_prefill(fp4x_llama_model *m, cudaStream_t st, const uint32_t *prompt, uint32_t n);  // batch.cu
}  // namespace batch
namespace engine {

__device__ __forceinline__ void argmax_merge(float &bv, uint32_t &bi, float ov, uint32_t oi) {
    if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
    }
}

// argmax (llama_run/src/main.rs:263-315: ties to the lowest index) + advance of
// the device-resident loop state (llama_run/src/main.rs:550-566).
__global__ void __launch_bounds__(1024) argmax_advance_kernel(uint32_t n, const float *__restrict__ logits,
                                                              uint32_t *__restrict__ state,
                                                              const uint32_t *__restrict__ prompt,
                                                              uint32_t *__restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
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
        const uint32_t pos = state[1], n_prompt = state[3], cap = state[4];
        state[2] = gi;
        if (pos + 1 >= n_prompt && pos + 1 - n_prompt < cap) out[pos + 1 - n_prompt] = gi;
        state[0] = (pos + 1 < n_prompt) ? prompt[pos + 1] : gi;
        state[1] = pos + 1;
    }
}

__global__ void fill_f32_kernel(float *p, float v, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        p[i] = v;
}

int cuda_fail(const char *what, cudaError_t e) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return FP4X_ECUDA;
}

#define FP4X_CUDA(call)                                 \
    do {                                                \
        cudaError_t e_ = (call);                        \
        if (e_ != cudaSuccess) return cuda_fail(#call, e_); \
    } while (0)
#define FP4X_TRY(call)          \
    do {                        \
        int s_ = (call);        \
        if (s_) return s_;      \
    } while (0)

template <typename T>
int alloc(fp4x_llama_model *m, T **p, size_t count) {
    void *q = nullptr;
    cudaError_t e = cudaMalloc(&q, count * sizeof(T) + 16);
    if (e != cudaSuccess) {
        set_error("llama_model_create: cudaMalloc(%zu): %s", count * sizeof(T), cudaGetErrorString(e));
        return FP4X_ENOMEM;
    }
    m->allocs.push_back(q);
    *p = static_cast<T *>(q);
    return FP4X_OK;
}

int alloc_q(fp4x_llama_model *m, QMat &q, uint32_t n, uint32_t k) {
    q.n = n, q.k = k;
    FP4X_TRY(alloc(m, &q.w, (size_t)n * k / 2));
    FP4X_TRY(alloc(m, &q.s, (size_t)n * k / 32));
    return FP4X_OK;
}

int validate_config(const fp4x_llama_config &c) {
    FP4X_REQUIRE(c.n_layers >= 1 && c.vocab >= 1 && c.max_seq >= 1, "llama config: empty model");
    FP4X_REQUIRE(c.head_dim == 64 || c.head_dim == 128, "llama config: head_dim %u not in {64, 128}", c.head_dim);
    FP4X_REQUIRE(c.n_kv_heads >= 1 && c.n_heads % c.n_kv_heads == 0, "llama config: n_heads %% n_kv_heads != 0");
    FP4X_REQUIRE(c.dim % 32 == 0 && c.ffn % 32 == 0, "llama config: dim and ffn must be multiples of 32");
    FP4X_REQUIRE(c.dim <= gemv::kMaxK && c.ffn <= gemv::kMaxK && c.n_heads * c.head_dim <= gemv::kMaxK,
                 "llama config: contraction length above %u", gemv::kMaxK);
    if (c.tp_size > 1) {
        const uint32_t T = c.tp_size;
        FP4X_REQUIRE(c.tp_rank < T && T <= 8, "llama config: tp_rank %u of tp_size %u (at most 8)", c.tp_rank, T);
        FP4X_REQUIRE(c.n_kv_heads % T == 0, "llama config: %u KV heads do not split over %u ranks", c.n_kv_heads, T);
        FP4X_REQUIRE(c.ffn % (32 * T) == 0, "llama config: ffn %u does not split over %u ranks in 32-blocks", c.ffn, T);
    }
    return FP4X_OK;
}

// One token of the model on `st` (captured into the graph).
int enqueue_token(fp4x_llama_model *m, cudaStream_t st) {
    const fp4x_llama_config &c = m->lc;
    const bool tp = m->xc != nullptr;
    const uint32_t hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
    const bool pdl = m->pdl;
    uint32_t *tok = m->state, *pos = m->state + 1;
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        LayerW &L = m->layers[l];
        gemv::Args a = {};
        // 1. [embed] + RMSNorm + QKV + RoPE + KV append
        a.n = L.qkv.n, a.k = c.dim, a.w = L.qkv.w, a.scales = L.qkv.s, a.x = m->x;
        a.norm_w = L.attn_norm, a.eps = c.eps;
        a.embed = m->embed, a.tok = tok, a.x_out = m->x;
        a.q_tiles = qd / 16, a.k_tiles = kvd / 16, a.n_kv = c.n_kv_heads, a.head_dim = hd;
        a.cos_t = m->cos_t, a.sin_t = m->sin_t, a.pos = pos, a.q_out = m->q, a.kc = L.kc, a.vc = L.vc;
        a.max_seq = c.max_seq;
        FP4X_TRY(gemv::launch_fused(st, l == 0 ? gemv::PRO_EMBED_RMSNORM : gemv::PRO_RMSNORM, gemv::EPI_QKV_ROPE,
                                    a, pdl));
        // 2. attention over positions 0..pos
        {
            attn::Params p;
            p.batch = 1, p.n_heads = c.n_heads, p.n_kv = c.n_kv_heads, p.seq = 1, p.max_seq = c.max_seq;
            p.splits = m->attn_splits, p.split_len = m->attn_split_len;
            p.scale = 1.0f / sqrtf((float)hd);
            p.q = m->q, p.kc = L.kc, p.vc = L.vc, p.out = m->att, p.ws = m->ws, p.pos_ptr = pos;
            FP4X_TRY(attn::launch_engine(st, p, hd, pdl));
        }
        // 3. O + residual
        a = gemv::Args{};
        a.n = c.dim, a.k = qd, a.w = L.o.w, a.scales = L.o.s, a.x = m->att, a.y = tp ? m->part : m->x;
        FP4X_TRY(gemv::launch_fused(st, gemv::PRO_NONE, tp ? gemv::EPI_STORE : gemv::EPI_RESIDUAL, a, pdl));
        if (tp) FP4X_TRY(tp::allreduce_add(st, m->xc, m->part, m->x, pdl));  // row-parallel O
        // 4. RMSNorm + gate/up + SwiGLU
        a = gemv::Args{};
        a.n = 2 * c.ffn, a.k = c.dim, a.w = L.gu.w, a.scales = L.gu.s, a.x = m->x, a.y = m->s;
        a.norm_w = L.ffn_norm, a.eps = c.eps;
        FP4X_TRY(gemv::launch_fused(st, gemv::PRO_RMSNORM, gemv::EPI_SWIGLU, a, pdl));
        // 5. down + residual
        a = gemv::Args{};
        a.n = c.dim, a.k = c.ffn, a.w = L.down.w, a.scales = L.down.s, a.x = m->s, a.y = tp ? m->part : m->x;
        FP4X_TRY(gemv::launch_fused(st, gemv::PRO_NONE, tp ? gemv::EPI_STORE : gemv::EPI_RESIDUAL, a, pdl));
        if (tp) FP4X_TRY(tp::allreduce_add(st, m->xc, m->part, m->x, pdl));  // row-parallel down
    }
    gemv::Args a = {};
    a.n = c.vocab, a.k = c.dim, a.w = m->lm_head.w, a.scales = m->lm_head.s, a.x = m->x, a.y = m->logits;
    a.norm_w = m->final_norm, a.eps = c.eps;
    FP4X_TRY(gemv::launch_fused(st, gemv::PRO_RMSNORM, gemv::EPI_STORE, a, pdl));
    if (tp) return tp::argmax_advance(st, m->xc, c.vocab, m->v0, m->logits, m->state, m->prompt, m->out, pdl);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1024);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    FP4X_CUDA(cudaLaunchKernelEx(&cfg, argmax_advance_kernel, c.vocab, (const float *)m->logits, m->state,
                                 (const uint32_t *)m->prompt, m->out));
    return FP4X_OK;
}

int build_graph(fp4x_llama_model *m) {
    if (m->exec) return FP4X_OK;
    cudaStream_t st = m->cap_stream;
    FP4X_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_token(m, st);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail("cudaStreamEndCapture", e);
    m->graph = g;
    FP4X_CUDA(cudaGraphInstantiate(&m->exec, g, 0));
    return FP4X_OK;
}

int init_weights(fp4x_llama_model *m, cudaStream_t st) {
    // shard of rank r (the whole model without TP): q rows of heads [r*H_l, ...), k/v
    // rows of KV heads [r*KV_l, ...), O columns of those q heads, gate/up rows and
    // down columns [r*ffn_l, ...), lm_head rows [v0, v0 + vocab_l)
    const fp4x_llama_config &c = m->lc, &g = m->cfg;
    const uint32_t hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd, r = g.tp_size > 1 ? g.tp_rank : 0;
    const uint32_t gqd = g.n_heads * hd;
    auto tseed = [&](uint32_t id) { return hash64(c.seed, id); };
    const float sig = 0.02f;
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        LayerW &L = m->layers[l];
        const uint32_t base = T_LAYER0 + 8 * l;
        // QKV: q and k rope-paired, v natural, concatenated
        FP4X_TRY(quant::init_mxfp4_rowmap(st, tseed(base + M_Q), sig, qd, c.dim, L.qkv.w, L.qkv.s, 1, 0, hd, r * qd));
        FP4X_TRY(quant::init_mxfp4_rowmap(st, tseed(base + M_K), sig, kvd, c.dim, L.qkv.w, L.qkv.s, 1, qd, hd, r * kvd));
        FP4X_TRY(quant::init_mxfp4_rowmap(st, tseed(base + M_V), sig, kvd, c.dim, L.qkv.w, L.qkv.s, 0, qd + kvd, hd,
                                          r * kvd));
        FP4X_TRY(quant::init_mxfp4_rowmap(st, tseed(base + M_O), sig, c.dim, qd, L.o.w, L.o.s, 0, 0, hd, 0, gqd,
                                          r * qd));
        FP4X_TRY(quant::init_mxfp4_rowmap(st, tseed(base + M_GATE), sig, c.ffn, c.dim, L.gu.w, L.gu.s, 2, 0, hd,
                                          r * c.ffn));
        FP4X_TRY(quant::init_mxfp4_rowmap(st, tseed(base + M_UP), sig, c.ffn, c.dim, L.gu.w, L.gu.s, 2, 8, hd,
                                          r * c.ffn));
        FP4X_TRY(quant::init_mxfp4_rowmap(st, tseed(base + M_DOWN), sig, c.dim, c.ffn, L.down.w, L.down.s, 0, 0, hd, 0,
                                          g.ffn, r * c.ffn));
        fill_f32_kernel<<<8, 256, 0, st>>>(L.attn_norm, 1.0f, c.dim);
        fill_f32_kernel<<<8, 256, 0, st>>>(L.ffn_norm, 1.0f, c.dim);
        FP4X_CUDA(cudaMemsetAsync(L.kc, 0, (size_t)c.max_seq * kvd * 2, st));
        FP4X_CUDA(cudaMemsetAsync(L.vc, 0, (size_t)c.max_seq * kvd * 2, st));
    }
    FP4X_TRY(quant::init_mxfp4_rowmap(st, tseed(T_LMHEAD), sig, c.vocab, c.dim, m->lm_head.w, m->lm_head.s, 0, 0, hd,
                                      m->v0));
    FP4X_TRY(fp4x_fill_normal_bf16((fp4x_stream_t)st, tseed(T_EMBED), 0, sig, m->embed, (size_t)g.vocab * c.dim));
    fill_f32_kernel<<<8, 256, 0, st>>>(m->final_norm, 1.0f, c.dim);
    FP4X_TRY(llama_rope_tables((fp4x_stream_t)st, c.max_seq, hd, (double)c.rope_theta, m->cos_t, m->sin_t));
    return check_launch("init_weights");
}

// The persistent decode kernels over this model's (shard's) weights; a path the
// shape does not fit is left out with its reason.  Under tensor parallelism only
// the tensor-core kernel is built, with its shared buffers in the exchange areas.
int build_persistent(fp4x_llama_model *m, const ptc::TpIn *tpin) {
    const fp4x_llama_config &c = m->lc;
    const uint32_t kvd = c.n_kv_heads * c.head_dim;
    int rc = FP4X_OK;
    persist::BuildIn in;
    in.cfg = c;
    for (auto &L : m->layers) {
        in.qkv.push_back({L.qkv.w, L.qkv.s, L.qkv.n, L.qkv.k});
        in.o.push_back({L.o.w, L.o.s, L.o.n, L.o.k});
        in.gu.push_back({L.gu.w, L.gu.s, L.gu.n, L.gu.k});
        in.down.push_back({L.down.w, L.down.s, L.down.n, L.down.k});
    }
    in.lm = {m->lm_head.w, m->lm_head.s, m->lm_head.n, m->lm_head.k};
    in.attn_norm = m->norms, in.ffn_norm = m->norms + (size_t)c.n_layers * c.dim, in.final_norm = m->final_norm;
    in.embed = m->embed, in.cos_t = m->cos_t, in.sin_t = m->sin_t;
    in.kc = m->kv, in.vc = m->kv + (size_t)c.n_layers * c.max_seq * kvd;
    in.q = m->q, in.logits = m->logits, in.state = m->state, in.prompt = m->prompt, in.out = m->out;
    if (!tpin) {
        const int prc = persist::build(in, m->cap_stream, &m->pe);
        if (prc == FP4X_OK) {
            m->path = 1;
        } else if (prc == FP4X_EUNSUPPORTED) {
            m->pe = nullptr;  // graph path only
            snprintf(m->persist_why, sizeof(m->persist_why), "%s", fp4x_last_error());
        } else {
            rc = prc;
        }
    } else {
        snprintf(m->persist_why, sizeof(m->persist_why), "not built under tensor parallelism");
    }
    if (!rc) {
        const int trc = ptc::build(in, m->cap_stream, &m->pt, tpin);
        if (trc == FP4X_OK) {
            m->path = 2;
        } else if (trc == FP4X_EUNSUPPORTED) {
            m->pt = nullptr;
            snprintf(m->tc_why, sizeof(m->tc_why), "%s", fp4x_last_error());
        } else {
            rc = trc;
        }
    }
    // Under tensor parallelism the tensor-core kernel is the default too (its grid
    // barriers stay on one GPU; ranks meet only in the row-parallel exchanges after
    // the O and down projections and at the argmax); the graph path (per-layer
    // kernels + the peer-memory allreduce kernel) remains selectable.
    const char *env = getenv("FP4X_DECODE_PATH");
    if (env && strcmp(env, "graph") == 0) m->path = 0;
    if (env && strcmp(env, "persistent") == 0 && m->pe) m->path = 1;
    if (env && strcmp(env, "tensor") == 0 && m->pt) m->path = 2;
    return rc;
}

int load_safetensors(fp4x_llama_model *m, cudaStream_t st, const char *path);  // loader.cu

// weights_path: a safetensors checkpoint to load instead of the seeded init.
int create(const fp4x_llama_config *cfg, fp4x_llama_model **out, const char *weights_path = nullptr) {
    FP4X_REQUIRE(cfg && out, "llama_model_create: null pointer");
    FP4X_TRY(validate_config(*cfg));
    fp4x_llama_model *m = new (std::nothrow) fp4x_llama_model();
    if (!m) return FP4X_ENOMEM;
    m->cfg = *cfg;
    m->lc = *cfg;
    if (cfg->tp_size > 1) {  // this rank's shard sizes
        const uint32_t T = cfg->tp_size, per = (cfg->vocab + T * 16 - 1) / (T * 16) * 16;
        m->lc.n_heads = cfg->n_heads / T, m->lc.n_kv_heads = cfg->n_kv_heads / T, m->lc.ffn = cfg->ffn / T;
        m->v0 = std::min(cfg->vocab, cfg->tp_rank * per);
        m->lc.vocab = std::min(cfg->vocab, m->v0 + per) - m->v0;
    }
    cudaGetDevice(&m->device);
    const fp4x_llama_config &c = m->lc;
    const uint32_t hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
    int rc = FP4X_OK;
    auto fail = [&](int r) {
        llama_model_destroy(m);
        return r;
    };
    m->layers.resize(c.n_layers);
    rc = alloc(m, &m->norms, (size_t)2 * c.n_layers * c.dim);
    if (!rc) rc = alloc(m, &m->kv, (size_t)2 * c.n_layers * c.max_seq * kvd);
    for (uint32_t l = 0; l < c.n_layers && !rc; ++l) {
        LayerW &L = m->layers[l];
        rc = alloc_q(m, L.qkv, qd + 2 * kvd, c.dim);
        if (!rc) rc = alloc_q(m, L.o, c.dim, qd);
        if (!rc) rc = alloc_q(m, L.gu, 2 * c.ffn, c.dim);
        if (!rc) rc = alloc_q(m, L.down, c.dim, c.ffn);
        L.attn_norm = m->norms + (size_t)l * c.dim;
        L.ffn_norm = m->norms + (size_t)(c.n_layers + l) * c.dim;
        L.kc = m->kv + (size_t)l * c.max_seq * kvd;
        L.vc = m->kv + (size_t)(c.n_layers + l) * c.max_seq * kvd;
    }
    if (!rc) rc = alloc_q(m, m->lm_head, std::max(1u, c.vocab), c.dim);
    if (!rc) rc = alloc(m, &m->embed, (size_t)m->cfg.vocab * c.dim);
    if (!rc) rc = alloc(m, &m->part, c.dim);
    if (!rc && m->cfg.tp_size > 1) rc = tp::create(&m->xc, m->cfg.tp_rank, m->cfg.tp_size, c.dim);
    if (!rc) rc = alloc(m, &m->final_norm, c.dim);
    if (!rc) rc = alloc(m, &m->cos_t, (size_t)c.max_seq * hd / 2);
    if (!rc) rc = alloc(m, &m->sin_t, (size_t)c.max_seq * hd / 2);
    if (!rc) rc = alloc(m, &m->x, c.dim);
    if (!rc) rc = alloc(m, &m->q, qd);
    if (!rc) rc = alloc(m, &m->att, qd);
    if (!rc) rc = alloc(m, &m->s, c.ffn);
    if (!rc) rc = alloc(m, &m->logits, c.vocab);
    m->attn_split_len = 64;
    m->attn_splits = (c.max_seq + m->attn_split_len - 1) / m->attn_split_len;
    if (!rc) rc = alloc(m, &m->ws, (size_t)c.n_heads * m->attn_splits * (hd + 2));
    if (!rc) rc = alloc(m, &m->state, 8);
    if (!rc) rc = alloc(m, &m->prompt, c.max_seq);
    if (!rc) rc = alloc(m, &m->out, c.max_seq);
    if (rc) return fail(rc);
    if (cudaStreamCreateWithFlags(&m->cap_stream, cudaStreamNonBlocking) != cudaSuccess)
        return fail(cuda_fail("cudaStreamCreate", cudaGetLastError()));
    rc = weights_path ? load_safetensors(m, m->cap_stream, weights_path) : init_weights(m, m->cap_stream);
    if (!rc) {
        const uint32_t st[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (cudaMemcpyAsync(m->state, st, sizeof(st), cudaMemcpyHostToDevice, m->cap_stream) != cudaSuccess ||
            cudaStreamSynchronize(m->cap_stream) != cudaSuccess)
            rc = cuda_fail("llama_model_create: init", cudaGetLastError());
    }
    if (!rc && m->xc) {  // tensor parallel: graph path only, built by llama_model_tp_connect
        *out = m;
        return FP4X_OK;
    }
    if (!rc) rc = build_graph(m);
    if (!rc) rc = build_persistent(m, nullptr);
    if (rc) return fail(rc);
    *out = m;
    return FP4X_OK;
}

// Run n tokens of the device-resident loop on the selected path.
int run_tokens(fp4x_llama_model *m, cudaStream_t st, uint32_t n) {
    FP4X_REQUIRE(m->hpos >= 0, "decode: no position set (call llama_forward or llama_generate first)");
    FP4X_REQUIRE((uint64_t)m->hpos + n <= m->cfg.max_seq, "decode: position %lld + %u tokens exceeds max_seq %u",
                 (long long)m->hpos, n, m->cfg.max_seq);
    if (m->path == 2) {
        FP4X_TRY(ptc::launch(m->pt, st, n));
    } else if (m->path == 1) {
        FP4X_TRY(persist::launch(m->pe, st, n));
    } else {
        for (uint32_t i = 0; i < n; ++i) FP4X_CUDA(cudaGraphLaunch(m->exec, st));
    }
    m->hpos += n;
    return FP4X_OK;
}

int set_state(fp4x_llama_model *m, cudaStream_t st, uint32_t tok, uint32_t pos, uint32_t n_prompt, uint32_t cap) {
    // pageable source: the copy is staged before the call returns
    const uint32_t v[5] = {tok, pos, 0, n_prompt, cap};
    FP4X_CUDA(cudaMemcpyAsync(m->state, v, sizeof(v), cudaMemcpyHostToDevice, st));
    m->hpos = pos;
    return FP4X_OK;
}

}  // namespace engine
}  // namespace fp4x

using namespace fp4x;
using namespace fp4x::engine;

extern "C" int llama_model_create(const fp4x_llama_config *cfg, fp4x_llama_model **out) {
    return engine::create(cfg, out);
}

extern "C" int llama_model_destroy(fp4x_llama_model *m) {
    if (!m) return FP4X_OK;
    cudaSetDevice(m->device);
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    if (m->cap_stream) {
        cudaStreamSynchronize(m->cap_stream);
        cudaStreamDestroy(m->cap_stream);
    }
    batch::destroy(m->pf);
    persist::destroy(m->pe);
    ptc::destroy(m->pt);
    tp::destroy(m->xc);
    for (void *p : m->allocs) cudaFree(p);
    delete m;
    return FP4X_OK;
}

extern "C" int llama_model_reset(fp4x_llama_model *m, fp4x_stream_t stream) {
    FP4X_REQUIRE(m, "llama_model_reset: null model");
    const uint32_t kvd = m->lc.n_kv_heads * m->lc.head_dim;
    FP4X_CUDA(cudaMemsetAsync(m->kv, 0, (size_t)2 * m->lc.n_layers * m->lc.max_seq * kvd * 2,
                              (cudaStream_t)stream));
    return FP4X_OK;
}

extern "C" int llama_decode_step(fp4x_llama_model *m, fp4x_stream_t stream) {
    FP4X_REQUIRE(m && m->exec, "llama_decode_step: null model");
    return run_tokens(m, (cudaStream_t)stream, 1);
}

extern "C" int llama_decode_steps(fp4x_llama_model *m, fp4x_stream_t stream, uint32_t n) {
    FP4X_REQUIRE(m && m->exec, "llama_decode_steps: null model");
    return run_tokens(m, (cudaStream_t)stream, n);
}

extern "C" int llama_model_set_path(fp4x_llama_model *m, int path) {
    FP4X_REQUIRE(m && path >= 0 && path <= 2, "llama_model_set_path: bad argument");
    if (path == 1 && !m->pe) {
        set_error("llama_model_set_path: the persistent kernel is unavailable: %s", m->persist_why);
        return FP4X_EUNSUPPORTED;
    }
    if (path == 2 && !m->pt) {
        set_error("llama_model_set_path: the tensor-core kernel is unavailable: %s", m->tc_why);
        return FP4X_EUNSUPPORTED;
    }
    m->path = path;
    return FP4X_OK;
}

extern "C" int llama_model_get_path(const fp4x_llama_model *m) { return m ? m->path : -1; }

extern "C" int llama_forward(fp4x_llama_model *m, fp4x_stream_t stream, uint32_t token, uint32_t pos,
                             uint32_t *next_host, float *logits_host) {
    FP4X_REQUIRE(m && m->exec, "llama_forward: null model");
    FP4X_REQUIRE(token < m->cfg.vocab, "llama_forward: token %u >= vocab", token);
    FP4X_REQUIRE(pos < m->cfg.max_seq, "llama_forward: pos %u >= max_seq %u", pos, m->cfg.max_seq);
    cudaStream_t st = (cudaStream_t)stream;
    FP4X_TRY(set_state(m, st, token, pos, 0, 0));
    FP4X_TRY(run_tokens(m, st, 1));
    if (next_host) FP4X_CUDA(cudaMemcpyAsync(next_host, m->state + 2, 4, cudaMemcpyDeviceToHost, st));
    if (logits_host)
        FP4X_CUDA(cudaMemcpyAsync(logits_host, m->logits, (size_t)m->lc.vocab * 4, cudaMemcpyDeviceToHost, st));
    FP4X_CUDA(cudaStreamSynchronize(st));
    return FP4X_OK;
}

extern "C" int llama_generate(fp4x_llama_model *m, fp4x_stream_t stream, const uint32_t *prompt, uint32_t n_prompt,
                              uint32_t n_gen, uint32_t *out_ids, float *prefill_ms, float *decode_ms) {
    FP4X_REQUIRE(m && m->exec && prompt && out_ids, "llama_generate: null pointer");
    FP4X_REQUIRE(n_prompt >= 1 && n_gen >= 1, "llama_generate: need n_prompt >= 1 and n_gen >= 1");
    FP4X_REQUIRE(n_prompt + n_gen - 1 <= m->cfg.max_seq, "llama_generate: %u + %u - 1 positions exceed max_seq %u",
                 n_prompt, n_gen, m->cfg.max_seq);
    for (uint32_t i = 0; i < n_prompt; ++i)
        FP4X_REQUIRE(prompt[i] < m->cfg.vocab, "llama_generate: prompt id %u >= vocab", prompt[i]);
    cudaStream_t st = (cudaStream_t)stream;
    FP4X_CUDA(cudaMemcpyAsync(m->prompt, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, st));
    FP4X_TRY(set_state(m, st, prompt[0], 0, n_prompt, n_gen));
    cudaEvent_t e0, e1, e2;
    FP4X_CUDA(cudaEventCreate(&e0));
    FP4X_CUDA(cudaEventCreate(&e1));
    FP4X_CUDA(cudaEventCreate(&e2));
    FP4X_CUDA(cudaEventRecord(e0, st));
    // prefill: the prompt in multi-token passes of the batched engine (written into
    // this model's KV cache), or -- under tensor parallelism, or FP4X_PREFILL=serial --
    // the one-token decode path over the prompt as llama_run:550-556; either way the
    // last prompt position yields the first generated token
    const char *pfe = getenv("FP4X_PREFILL");
    if (!m->xc && !(pfe && strcmp(pfe, "serial") == 0)) {
        FP4X_TRY(batch::model_prefill(m, st, prompt, n_prompt));
        m->hpos = n_prompt;
    } else {
        FP4X_TRY(run_tokens(m, st, n_prompt));
    }
    FP4X_CUDA(cudaEventRecord(e1, st));
    FP4X_TRY(run_tokens(m, st, n_gen - 1));
    FP4X_CUDA(cudaEventRecord(e2, st));
    FP4X_CUDA(cudaMemcpyAsync(out_ids, m->out, (size_t)n_gen * 4, cudaMemcpyDeviceToHost, st));
    FP4X_CUDA(cudaStreamSynchronize(st));
    float a = 0, b = 0;
    cudaEventElapsedTime(&a, e0, e1);
    cudaEventElapsedTime(&b, e1, e2);
    if (prefill_ms) *prefill_ms = a;
    if (decode_ms) *decode_ms = b;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaEventDestroy(e2);
    return FP4X_OK;
}

extern "C" int llama_model_export_tensor(fp4x_llama_model *m, uint32_t tensor_id, uint8_t *packed_host,
                                         uint8_t *scales_host, uint32_t *n_out, uint32_t *k_out) {
    FP4X_REQUIRE(m, "llama_model_export_tensor: null model");
    const fp4x_llama_config &c = m->lc;  // this rank's shard under tensor parallelism
    const uint32_t hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
    const QMat *src = nullptr;
    uint32_t n = 0, k = 0, mode = 0, off = 0;
    if (tensor_id == T_LMHEAD) {
        src = &m->lm_head, n = c.vocab, k = c.dim;
    } else if (tensor_id >= T_LAYER0) {
        const uint32_t l = (tensor_id - T_LAYER0) / 8, w = (tensor_id - T_LAYER0) % 8;
        FP4X_REQUIRE(l < c.n_layers && w < M_COUNT, "llama_model_export_tensor: bad tensor id %u", tensor_id);
        const LayerW &L = m->layers[l];
        switch (w) {
        case M_Q: src = &L.qkv, n = qd, k = c.dim, mode = 1, off = 0; break;
        case M_K: src = &L.qkv, n = kvd, k = c.dim, mode = 1, off = qd; break;
        case M_V: src = &L.qkv, n = kvd, k = c.dim, mode = 0, off = qd + kvd; break;
        case M_O: src = &L.o, n = c.dim, k = qd; break;
        case M_GATE: src = &L.gu, n = c.ffn, k = c.dim, mode = 2, off = 0; break;
        case M_UP: src = &L.gu, n = c.ffn, k = c.dim, mode = 2, off = 8; break;
        default: src = &L.down, n = c.dim, k = c.ffn; break;
        }
    } else {
        FP4X_REQUIRE(false, "llama_model_export_tensor: tensor %u is not an MXFP4 matrix", tensor_id);
    }
    if (n_out) *n_out = n;
    if (k_out) *k_out = k;
    if (!packed_host || !scales_host) return FP4X_OK;
    for (uint32_t r = 0; r < n; ++r) {
        uint32_t d;
        if (mode == 1) {
            const uint32_t half = hd / 2, head = r / hd, j = r % hd, jj = j < half ? j : j - half;
            d = off + (head * (half / 8) + jj / 8) * 16 + (j < half ? 0u : 8u) + jj % 8;
        } else if (mode == 2) {
            d = (r / 8) * 16 + (r % 8) + off;
        } else {
            d = r + off;
        }
        FP4X_CUDA(cudaMemcpy(packed_host + (size_t)r * k / 2, src->w + (size_t)d * k / 2, k / 2, cudaMemcpyDeviceToHost));
        FP4X_CUDA(cudaMemcpy(scales_host + (size_t)r * k / 32, src->s + (size_t)d * k / 32, k / 32,
                             cudaMemcpyDeviceToHost));
    }
    return FP4X_OK;
}

extern "C" int llama_model_embedding(fp4x_llama_model *m, uint16_t *embed_host) {
    FP4X_REQUIRE(m && embed_host, "llama_model_embedding: null pointer");
    FP4X_CUDA(cudaMemcpy(embed_host, m->embed, (size_t)m->cfg.vocab * m->cfg.dim * 2, cudaMemcpyDeviceToHost));
    return FP4X_OK;
}

extern "C" uint32_t llama_model_kernels_per_token(const fp4x_llama_model *m) {
    if (!m || !m->graph) return 0;
    size_t n = 0;
    if (cudaGraphGetNodes(m->graph, nullptr, &n) != cudaSuccess) return 0;
    return (uint32_t)n;
}

extern "C" size_t llama_model_weight_bytes(const fp4x_llama_model *m) {
    if (!m) return 0;
    size_t b = (size_t)m->lm_head.n * m->lm_head.k * 17 / 32;
    for (const auto &L : m->layers)
        b += ((size_t)L.qkv.n * L.qkv.k + (size_t)L.o.n * L.o.k + (size_t)L.gu.n * L.gu.k +
              (size_t)L.down.n * L.down.k) * 17 / 32;
    return b;
}

// ---------------------------------------------------------------- tensor parallel

extern "C" int llama_model_tp_handle(fp4x_llama_model *m, void *handle_out) {
    FP4X_REQUIRE(m && handle_out, "llama_model_tp_handle: null pointer");
    FP4X_REQUIRE(m->xc, "llama_model_tp_handle: the model was not created with tp_size > 1");
    cudaSetDevice(m->device);
    return tp::export_handle(m->xc, handle_out);
}

extern "C" int llama_model_tp_connect(fp4x_llama_model *m, const void *handles) {
    FP4X_REQUIRE(m && handles, "llama_model_tp_connect: null pointer");
    FP4X_REQUIRE(m->xc, "llama_model_tp_connect: the model was not created with tp_size > 1");
    cudaSetDevice(m->device);
    FP4X_TRY(tp::connect(m->xc, handles));
    FP4X_TRY(build_graph(m));
    ptc::TpIn t;
    tp::ptc_buffers(m->xc, t);
    t.v0 = m->v0;
    return build_persistent(m, &t);
}

extern "C" int llama_model_shard(const fp4x_llama_model *m, uint32_t *v0, uint32_t *vocab_local) {
    FP4X_REQUIRE(m, "llama_model_shard: null model");
    if (v0) *v0 = m->v0;
    if (vocab_local) *vocab_local = m->lc.vocab;
    return FP4X_OK;
}
