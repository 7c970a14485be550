// batch.cu -- batched decode and prefill of the Llama model on the tcgen05
// fp4_mma GEMM (BASELINE config 4 at batch 64, config 3's batched decode as a
// whole model, and batched prompt prefill).
//
// The reference decodes one sequence one token at a time and prefills a prompt
// token by token through the same forward (examples/llama_run/src/main.rs:492-587).
// Here one step runs R "rows" through the model at once.  A row is
// (token, position, cache): in a decode step row r is sequence r at its own
// position; in a prefill pass the rows are consecutive prompt tokens of one
// sequence, sharing its cache, each attending causally up to its own position.
// Per layer:
//   1. RMSNorm + 8-term MXFP4 decomposition of every row (layer 0 gathers the
//      bf16 embedding rows of the row tokens first);
//   2. QKV: fp4_mma over the R x 8 term rows, the epilogue adding the 8 term
//      columns of each row and red.add-ing into an f32 QKV buffer;
//   3. RoPE of q and k (rope-paired storage rows), bf16 K/V append at each row's
//      (cache, position); the QKV buffer is cleared for the next layer;
//   4. split-KV flash-decode attention, per-row sequence length and cache;
//   5. decomposition of the attention rows -> O projection red.add into the
//      f32 residual rows;
//   6. RMSNorm + decomposition -> gate/up (rows interleaved by 8) red.add into an
//      f32 buffer;
//   7. SwiGLU + decomposition (clearing the gate/up buffer) -> down projection
//      red.add into the residual;
// then final RMSNorm -> lm_head -> per-row argmax, which advances each decoded
// sequence (token history, next token, position) on the device.  A decode step
// is one captured CUDA graph.
//
// Activations enter the tensor cores as the same 8-term MXFP4 sums as in the
// batch-1 tensor-core kernel (each term's scale 3 binades below the previous
// one, the sum within ~1.6e-7 of the block maximum), so every linear is an exact
// E2M1 x E2M1 product with fp32 accumulation.
#include "attention.cuh"
#include "common.cuh"

#include <algorithm>
#include <vector>

struct fp4x_llama_batch {
    fp4x_llama_model *m = nullptr;
    uint32_t rows = 0;     // rows per pass (prefill tokens per pass; decode rows = seqs)
    uint32_t seqs = 0;     // sequences, each with its own KV cache (== rows for llama_batch_create)
    uint32_t max_seq = 0;  // positions per sequence cache
    bool own_kv = true;    // false: the caches are the model's (its one-sequence prefill batch)
    std::vector<void *> allocs;
    uint16_t *kv = nullptr;  // K [L][seqs][max_seq][kvd], then V
    float *x = nullptr;      // residual rows [rows][dim]
    float *qkv = nullptr;    // [rows][qd + 2 kvd] (storage row order), kept zero between uses
    float *q = nullptr;      // roped q rows [rows][qd]
    float *att = nullptr;    // attention rows [rows][qd]
    float *gu = nullptr;     // gate/up rows [rows][2 ffn] (interleaved by 8), kept zero between uses
    float *logits = nullptr; // [rows][vocab]
    float *attn_ws = nullptr;
    size_t attn_ws_bytes = 0;
    uint32_t terms = 8;      // MXFP4 terms per activation row (8, or 4 on request)
    uint8_t *act = nullptr;    // term rows [terms rows][kmax / 2]
    uint8_t *act_s = nullptr;  // their E8M0 scales, as the atom image of the GEMM they feed
    float *mma_part = nullptr;  // split-K partials
    size_t mma_part_bytes = 0;
    // weight scales as the GEMM's 512-byte atom images (per layer: qkv, o, gu, down; then lm_head)
    std::vector<uint8_t *> wimg;
    uint32_t *dec_tok = nullptr, *dec_pos = nullptr;            // per sequence: next token, its position
    uint32_t *pf_tok = nullptr, *pf_pos = nullptr, *pf_cache = nullptr;  // prefill rows
    uint32_t *prompt = nullptr;  // staging for prefill tokens [max_seq]
    uint32_t *ids = nullptr;     // token history [rows][max_seq]
    std::vector<uint32_t> len;   // host: positions written per sequence
    cudaStream_t cap_stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint32_t last_rows = 0;  // logits rows of the last pass
    // tensor parallelism: row-parallel O / down outputs [rows][dim] before the
    // cross-rank allreduce, and the batch exchange area shared with the peers
    float *part = nullptr;
    fp4x::tp::RowExchange *rx = nullptr;
};

namespace fp4x {
namespace batch {

using engine::cuda_fail;

constexpr uint32_t kMaxTerms = 8;
constexpr int kThreads = 256;

enum Src : int { SRC_EMBED = 0, SRC_NORM = 1, SRC_PLAIN = 2, SRC_SWIGLU = 3 };

__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();  // red is reused by consecutive calls
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    return t;
}

// 8 source values [8i, 8i + 8) of row r.
template <int SRC>
__device__ __forceinline__ void load8(float (&x)[8], uint32_t i, uint32_t r, uint32_t K, const float *src,
                                      const uint16_t *erow) {
    if (SRC == SRC_EMBED) {
        const uint4 q = *reinterpret_cast<const uint4 *>(erow + 8 * i);
        const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            x[2 * j] = __uint_as_float(u[j] << 16);
            x[2 * j + 1] = __uint_as_float(u[j] & 0xFFFF0000u);
        }
    } else if (SRC == SRC_SWIGLU) {
        // storage rows 16j..16j+7 = gate 8j..8j+7, 16j+8.. = up; 8 values = one group
        const float *g = src + (size_t)r * 2 * K + 16 * i;
        const float4 g0 = __ldcg(reinterpret_cast<const float4 *>(g)), g1 = __ldcg(reinterpret_cast<const float4 *>(g + 4));
        const float4 u0 = __ldcg(reinterpret_cast<const float4 *>(g + 8)), u1 = __ldcg(reinterpret_cast<const float4 *>(g + 12));
        const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float uv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = gv[j] / (1.0f + expf(-gv[j])) * uv[j];  // llama_run:248-250
    } else {
        const float *p = src + (size_t)r * K + 8 * i;
        const float4 a0 = __ldcg(reinterpret_cast<const float4 *>(p)), a1 = __ldcg(reinterpret_cast<const float4 *>(p + 4));
        x[0] = a0.x, x[1] = a0.y, x[2] = a0.z, x[3] = a0.w, x[4] = a1.x, x[5] = a1.y, x[6] = a1.z, x[7] = a1.w;
    }
}

// Row r of the source -> (RMSNorm) -> term rows T r .. T r + T - 1 of act (packed E2M1,
// low nibble = lower k) + act_s (E8M0 per 32).  Thread = one 8-value word; the 4
// words of a 32-block sit in adjacent lanes; CTA (r, c) covers words
// [c * kThreads, (c + 1) * kThreads) of the row (the RMSNorm sum of squares is
// taken over the whole row by every CTA of it).  SRC_EMBED also writes the
// gathered row to x_out; SRC_SWIGLU clears the gate/up values it consumed.
template <int SRC>
__global__ void __launch_bounds__(kThreads) rows_decompose_kernel(uint32_t K, const float *src, float *x_out,
                                                                  const uint16_t *embed, const uint32_t *tok,
                                                                  const float *norm_w, float eps, uint8_t *act,
                                                                  uint8_t *act_s, uint32_t row0, uint32_t terms,
                                                                  uint32_t img_nt) {
    __shared__ float red[kThreads / 32];
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t r = blockIdx.x, rs = row0 + r;  // output row, source row
    const uint32_t nw = K / 8, i = blockIdx.y * kThreads + threadIdx.x;
    const uint16_t *erow = SRC == SRC_EMBED ? embed + (size_t)tok[rs] * K : nullptr;
    float rms = 1.0f;
    if (SRC == SRC_EMBED || SRC == SRC_NORM) {
        float ss = 0.0f;
        for (uint32_t j = threadIdx.x; j < nw; j += kThreads) {
            float x[8];
            load8<SRC>(x, j, rs, K, src, erow);
#pragma unroll
            for (int e = 0; e < 8; ++e) ss += x[e] * x[e];
        }
        const float total = block_sum(ss, red);
        rms = 1.0f / sqrtf(total / (float)K + eps);  // llama_run:79-116
    }
    const bool valid = i < nw;  // whole 32-blocks are valid together (nw % 4 == 0)
    float x[8];
    if (valid) {
        load8<SRC>(x, i, rs, K, src, erow);
        if (SRC == SRC_EMBED) {
            *reinterpret_cast<float4 *>(x_out + (size_t)rs * K + 8 * i) = make_float4(x[0], x[1], x[2], x[3]);
            *reinterpret_cast<float4 *>(x_out + (size_t)rs * K + 8 * i + 4) = make_float4(x[4], x[5], x[6], x[7]);
        }
        if (SRC == SRC_SWIGLU) {
            float4 *g = reinterpret_cast<float4 *>(const_cast<float *>(src) + (size_t)rs * 2 * K + 16 * i);
#pragma unroll
            for (int e = 0; e < 4; ++e) g[e] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        if (SRC == SRC_EMBED || SRC == SRC_NORM) {
            const float4 w0 = __ldg(reinterpret_cast<const float4 *>(norm_w + 8 * i));
            const float4 w1 = __ldg(reinterpret_cast<const float4 *>(norm_w + 8 * i + 4));
            const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = x[e] * rms * wv[e];
        }
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = 0.0f;
    }
    uint32_t words[8];
    const int e1 = ptc::term_words8(x, words);  // every lane of the warp takes part
    if (!valid) return;
    const size_t row_bytes = K / 2;
#pragma unroll
    for (uint32_t t = 0; t < kMaxTerms; ++t) {
        if (t >= terms) break;
        const size_t tr = (size_t)r * terms + t;
        *reinterpret_cast<uint32_t *>(act + tr * row_bytes + 4 * i) = words[t];
        if ((i & 3) == 0)
            act_s[mma::scale_image_offset((uint32_t)tr, i / 4, K, img_nt)] = (uint8_t)(ptc::term_exp(e1, (int)t) + 127);
    }
}

// RoPE of the q and k storage rows (rope-paired 16-row tiles: rows 0..7 = dims
// j..j+7, rows 8..15 = dims j+half..), q to q_out in head-major order, k and v
// to the bf16 cache of the row at its position; every value read is cleared for
// the next layer's sums.  CTA (r, c): items c, c + gridDim.y, ... of row r
// (item = a rope pair of q/k rows or one v row).
__global__ void __launch_bounds__(kThreads) rows_rope_append_kernel(uint32_t qd, uint32_t kvd, uint32_t hd,
                                                                    float *qkv, float *q_out, uint16_t *kc,
                                                                    uint16_t *vc, const uint32_t *pos,
                                                                    const uint32_t *cache, uint32_t max_seq,
                                                                    const float *cos_t, const float *sin_t) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t r = blockIdx.x, half = hd / 2, n = qd + 2 * kvd, pairs = (qd + kvd) / 2;
    const uint32_t p = pos[r];
    const size_t c = cache ? cache[r] : r;
    float *row = qkv + (size_t)r * n;
    const bool in_cache = p < max_seq;
    uint16_t *kdst = kc + (c * max_seq + (in_cache ? p : 0)) * kvd, *vdst = vc + (c * max_seq + (in_cache ? p : 0)) * kvd;
    for (uint32_t it = blockIdx.y * kThreads + threadIdx.x; it < pairs + kvd; it += gridDim.y * kThreads) {
        if (it < pairs) {
            const uint32_t tile = it / 8, w = it % 8;
            const uint32_t s0 = tile * 16 + w;  // partner at s0 + 8
            const bool is_q = s0 < qd;
            const uint32_t lr = is_q ? s0 : s0 - qd;
            const uint32_t head = lr / hd, j = ((lr % hd) / 16) * 8 + w;
            const float x0 = __ldcg(row + s0), x1 = __ldcg(row + s0 + 8);
            row[s0] = 0.0f, row[s0 + 8] = 0.0f;
            if (!in_cache) continue;
            const float cs = cos_t[(size_t)p * half + j], sn = sin_t[(size_t)p * half + j];
            const float o0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));  // llama_run:135-136
            const float o1 = __fadd_rn(__fmul_rn(x1, cs), __fmul_rn(x0, sn));
            if (is_q) {
                q_out[(size_t)r * qd + head * hd + j] = o0;
                q_out[(size_t)r * qd + head * hd + j + half] = o1;
            } else {
                kdst[head * hd + j] = f32_to_bf16_bits(o0);
                kdst[head * hd + j + half] = f32_to_bf16_bits(o1);
            }
        } else {
            const uint32_t v = it - pairs;
            const float x = __ldcg(row + qd + kvd + v);
            row[qd + kvd + v] = 0.0f;
            if (in_cache) vdst[v] = f32_to_bf16_bits(x);
        }
    }
}

__device__ __forceinline__ void argmax_merge(float &bv, uint32_t &bi, float ov, uint32_t oi) {
    if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
    }
}

// Per logits row: argmax (ties -> lowest index, llama_run:263-315).  Decode
// (seq == ~0u): row r is sequence r: history ids[r][pos + 1] = next, next token,
// position + 1.  Prefill: the single row belongs to sequence `seq`, whose next
// position is `next_pos`.
__global__ void __launch_bounds__(1024) rows_argmax_kernel(uint32_t vocab, const float *logits, uint32_t *dec_tok,
                                                           uint32_t *dec_pos, uint32_t *ids, uint32_t max_seq,
                                                           uint32_t seq, uint32_t next_pos) {
    __shared__ float mv[32];
    __shared__ uint32_t mi[32];
    const uint32_t r = blockIdx.x;
    const float *lg = logits + (size_t)r * vocab;
    float bv = -INFINITY;
    uint32_t bi = 0;
    for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) {
        const float v = lg[i];
        if (v > bv) bv = v, bi = i;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) mv[warp] = bv, mi[warp] = bi;
    __syncthreads();
    if (threadIdx.x != 0) return;
    float gv = -INFINITY;
    uint32_t gi = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) argmax_merge(gv, gi, mv[w], mi[w]);
    const uint32_t s = seq == ~0u ? r : seq;
    const uint32_t np = seq == ~0u ? dec_pos[s] + 1 : next_pos;
    if (np < max_seq) {
        ids[(size_t)s * max_seq + np] = gi;
        dec_tok[s] = gi;
        dec_pos[s] = np;
    }
}

// Prefill rows: tokens prompt[0, n) of sequence `seq` at positions pos0 + i.
__global__ void prefill_rows_kernel(uint32_t n, uint32_t seq, uint32_t pos0, const uint32_t *prompt, uint32_t *tok,
                                    uint32_t *pos, uint32_t *cache, uint32_t *ids, uint32_t max_seq) {
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        tok[i] = prompt[i];
        pos[i] = pos0 + i;
        cache[i] = seq;
        ids[(size_t)seq * max_seq + pos0 + i] = prompt[i];
    }
}

template <typename T>
int alloc(fp4x_llama_batch *b, T **p, size_t count) {
    void *q = nullptr;
    cudaError_t e = cudaMalloc(&q, count * sizeof(T) + 16);
    if (e != cudaSuccess) {
        set_error("llama_batch_create: cudaMalloc(%zu): %s", count * sizeof(T), cudaGetErrorString(e));
        return FP4X_ENOMEM;
    }
    b->allocs.push_back(q);
    *p = static_cast<T *>(q);
    return FP4X_OK;
}

// Term rows = terms x R; out[R][n] = (or +=) the sums.  img: w's scale atom image.
int linear(fp4x_llama_batch *b, cudaStream_t st, uint32_t R, const QMat &w, const uint8_t *img, float *out,
           bool accumulate) {
    const uint32_t m = R * b->terms;
    const mma::Plan p = mma::plan(m, w.n, w.k);
    if (mma::partials_bytes(p, m, w.n, b->terms) > b->mma_part_bytes) {
        set_error("llama_batch: GEMM workspace too small");
        return FP4X_EINVAL;
    }
    return mma::launch(st, m, w.n, w.k, b->act, b->act_s, w.w, w.s, out, accumulate ? mma::OUT_ADD_F32 : mma::OUT_F32,
                       p, b->terms, b->mma_part, false, 1.0f, b->act_s, img);
}

// Largest split-K scratch a pass of up to `rows` rows needs over the model's linears.
size_t mma_ws_need(const fp4x_llama_model *m, uint32_t rows, uint32_t terms) {
    size_t part = 0;
    auto upd = [&](const QMat &w) {
        for (uint32_t r = 1; r <= rows; ++r) {
            const mma::Plan p = mma::plan(r * terms, w.n, w.k);
            part = std::max(part, mma::partials_bytes(p, r * terms, w.n, terms));
        }
    };
    const LayerW &L = m->layers[0];
    upd(L.qkv), upd(L.o), upd(L.gu), upd(L.down), upd(m->lm_head);
    return part;
}

// Token-tile rows of the GEMM fed by R rows of terms (the plan's tile width).
inline uint32_t act_tile_rows(uint32_t m) { return mma::token_tile(m); }

template <int SRC>
int decompose(fp4x_llama_batch *b, cudaStream_t st, uint32_t R, uint32_t K, const float *src, float *x_out,
              const uint32_t *tok, const float *norm_w, uint32_t row0 = 0) {
    const uint32_t chunks = (K / 8 + kThreads - 1) / kThreads;
    const cudaError_t e = launch_pdl(rows_decompose_kernel<SRC>, dim3(R, chunks), dim3(kThreads), 0, st, K, src, x_out,
                                     (const uint16_t *)b->m->embed, tok, norm_w, b->m->lc.eps, b->act, b->act_s, row0,
                                     b->terms, act_tile_rows(R * b->terms));
    if (e != cudaSuccess) {
        set_error("llama_batch: decompose: %s", cudaGetErrorString(e));
        return FP4X_ECUDA;
    }
    return check_launch("llama_batch: decompose");
}

// Slices of the attention: about 4 CTAs per SM over R rows, slices >= 128 positions.
void attn_geometry(const fp4x_llama_model *m, uint32_t R, uint32_t max_seq, uint32_t &splits, uint32_t &split_len) {
    const fp4x_llama_config &c = m->lc;
    const uint32_t hpc = attn::heads_per_cta(c.n_heads / c.n_kv_heads, true);
    const uint32_t ctas = R * (c.n_heads / hpc), target = 4u * (uint32_t)num_sms();
    uint32_t s = std::max(1u, (target + ctas - 1) / ctas);
    s = std::min(s, std::max(1u, (max_seq + 127) / 128));
    split_len = (max_seq + s - 1) / s;
    split_len = (split_len + 63) / 64 * 64;
    splits = (max_seq + split_len - 1) / split_len;
}

// One pass of R rows (tokens tok, positions pos, caches cache: null = row index)
// through the model; logits of rows [lm0, R) into b->logits.
int forward(fp4x_llama_batch *b, cudaStream_t st, uint32_t R, const uint32_t *tok, const uint32_t *pos,
            const uint32_t *cache, uint32_t lm0) {
    fp4x_llama_model *m = b->m;
    const fp4x_llama_config &c = m->lc;
    const uint32_t hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
    const size_t layer_kv = (size_t)b->seqs * b->max_seq * kvd;
    uint16_t *kbase = b->kv, *vbase = b->kv + (size_t)c.n_layers * layer_kv;
    attn::Params ap{};
    ap.batch = R, ap.n_heads = c.n_heads, ap.n_kv = c.n_kv_heads, ap.seq = 1, ap.max_seq = b->max_seq;
    attn_geometry(m, R, b->max_seq, ap.splits, ap.split_len);
    if (attn::workspace_bytes(R, c.n_heads, hd, ap.splits) > b->attn_ws_bytes) {
        set_error("llama_batch: attention workspace too small");
        return FP4X_EINVAL;
    }
    ap.scale = 1.0f / sqrtf((float)hd);
    ap.q = b->q, ap.out = b->att, ap.ws = b->attn_ws, ap.pos_ptr = nullptr, ap.row_pos = pos, ap.row_cache = cache;
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        LayerW &L = m->layers[l];
        uint16_t *kc = kbase + l * layer_kv, *vc = vbase + l * layer_kv;
        if (l == 0)
            FP4X_TRY(decompose<SRC_EMBED>(b, st, R, c.dim, nullptr, b->x, tok, L.attn_norm));
        else
            FP4X_TRY(decompose<SRC_NORM>(b, st, R, c.dim, b->x, nullptr, nullptr, L.attn_norm));
        const uint8_t *const *wi = b->wimg.data() + 4 * l;
        FP4X_TRY(linear(b, st, R, L.qkv, wi[0], b->qkv, false));
        if (launch_pdl(rows_rope_append_kernel, dim3(R, (qd + 3 * kvd + 2 * kThreads - 1) / (2 * kThreads)),
                       dim3(kThreads), 0, st, qd, kvd, hd, b->qkv, b->q, kc, vc, pos, cache, b->max_seq,
                       (const float *)m->cos_t, (const float *)m->sin_t) != cudaSuccess) {
            set_error("llama_batch: rope launch failed");
            return FP4X_ECUDA;
        }
        FP4X_TRY(check_launch("llama_batch: rope"));
        ap.kc = kc, ap.vc = vc;
        FP4X_TRY(attn::launch_engine(st, ap, hd, true));
        FP4X_TRY(decompose<SRC_PLAIN>(b, st, R, qd, b->att, nullptr, nullptr, nullptr));
        if (b->rx) {  // row-parallel O: local partial, then the cross-rank sum into the residual
            FP4X_TRY(linear(b, st, R, L.o, wi[1], b->part, false));
            FP4X_TRY(tp::rows_allreduce_add(st, b->rx, b->part, b->x, (size_t)R * c.dim));
        } else {
            FP4X_TRY(linear(b, st, R, L.o, wi[1], b->x, true));
        }
        FP4X_TRY(decompose<SRC_NORM>(b, st, R, c.dim, b->x, nullptr, nullptr, L.ffn_norm));
        FP4X_TRY(linear(b, st, R, L.gu, wi[2], b->gu, false));
        FP4X_TRY(decompose<SRC_SWIGLU>(b, st, R, c.ffn, b->gu, nullptr, nullptr, nullptr));
        if (b->rx) {  // row-parallel down
            FP4X_TRY(linear(b, st, R, L.down, wi[3], b->part, false));
            FP4X_TRY(tp::rows_allreduce_add(st, b->rx, b->part, b->x, (size_t)R * c.dim));
        } else {
            FP4X_TRY(linear(b, st, R, L.down, wi[3], b->x, true));
        }
    }
    const uint32_t RL = R - lm0;
    if (RL == 0) return FP4X_OK;  // no logits wanted (a prompt chunk before the last)
    FP4X_TRY(decompose<SRC_NORM>(b, st, RL, c.dim, b->x, nullptr, nullptr, m->final_norm, lm0));
    FP4X_TRY(linear(b, st, RL, m->lm_head, b->wimg[4 * c.n_layers], b->logits, false));
    b->last_rows = RL;
    return FP4X_OK;
}

// Per-row argmax of the last pass's logits (across ranks under tensor parallelism).
int argmax(fp4x_llama_batch *b, cudaStream_t st, uint32_t rows, uint32_t seq, uint32_t next_pos) {
    fp4x_llama_model *m = b->m;
    if (b->rx)
        return tp::rows_argmax(st, b->rx, rows, m->lc.vocab, m->v0, b->logits, b->dec_tok, b->dec_pos, b->ids,
                               b->max_seq, seq, next_pos);
    rows_argmax_kernel<<<rows, 1024, 0, st>>>(m->lc.vocab, b->logits, b->dec_tok, b->dec_pos, b->ids, b->max_seq, seq,
                                              next_pos);
    return check_launch("llama_batch: argmax");
}

int build_graph(fp4x_llama_batch *b) {
    if (b->exec) return FP4X_OK;
    cudaStream_t st = b->cap_stream;
    FP4X_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    int rc = forward(b, st, b->rows, b->dec_tok, b->dec_pos, nullptr, 0);
    if (!rc) rc = argmax(b, st, b->rows, ~0u, 0);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail("cudaStreamEndCapture", e);
    b->graph = g;
    FP4X_CUDA(cudaGraphInstantiate(&b->exec, g, 0));
    return FP4X_OK;
}

void destroy(fp4x_llama_batch *b) {
    if (!b) return;
    tp::row_destroy(b->rx);
    if (b->exec) cudaGraphExecDestroy(b->exec);
    if (b->graph) cudaGraphDestroy(b->graph);
    if (b->cap_stream) cudaStreamDestroy(b->cap_stream);
    for (void *p : b->allocs) cudaFree(p);
    delete b;
}

}  // namespace batch
}  // namespace fp4x

using namespace fp4x;

namespace fp4x {
namespace batch {
// rows per pass, seqs caches (kv: the caches, or null to allocate them).
int create(fp4x_llama_model *m, uint32_t rows, uint32_t seqs, uint16_t *kv, fp4x_llama_batch **out) {
    FP4X_REQUIRE(m && out, "llama_batch_create: null pointer");
    FP4X_REQUIRE(rows >= 1 && rows <= 256 && seqs >= 1 && seqs <= rows, "llama_batch_create: rows %u not in [1, 256]",
                 rows);
    const fp4x_llama_config &c = m->lc;
    FP4X_REQUIRE(c.dim % 64 == 0 && c.ffn % 64 == 0 && (c.n_heads * c.head_dim) % 64 == 0,
                 "llama_batch_create: dim, ffn and n_heads * head_dim must be multiples of 64");
    *out = nullptr;
    fp4x_llama_batch *b = new (std::nothrow) fp4x_llama_batch();
    if (!b) return FP4X_ENOMEM;
    b->m = m, b->rows = rows, b->seqs = seqs, b->max_seq = c.max_seq, b->own_kv = kv == nullptr;
    if (const char *e = getenv("FP4X_BATCH_TERMS")) b->terms = atoi(e) == 4 ? 4 : 8;
    b->len.assign(seqs, 0);
    const uint32_t hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
    const uint32_t kmax = std::max(std::max(c.dim, c.ffn), qd);
    uint32_t splits = 1, split_len = 0;
    batch::attn_geometry(m, rows, c.max_seq, splits, split_len);
    for (uint32_t r = 1; r <= rows; ++r) {  // the largest workspace any pass of <= rows rows needs
        uint32_t s2, l2;
        batch::attn_geometry(m, r, c.max_seq, s2, l2);
        b->attn_ws_bytes = std::max(b->attn_ws_bytes, attn::workspace_bytes(r, c.n_heads, hd, s2));
    }
    int rc = FP4X_OK;
    if (kv) {
        b->kv = kv;
    } else {
        rc = batch::alloc(b, &b->kv, (size_t)2 * c.n_layers * seqs * c.max_seq * kvd);
        if (!rc) rc = cudaMemset(b->kv, 0, (size_t)2 * c.n_layers * seqs * c.max_seq * kvd * 2) == cudaSuccess
                          ? FP4X_OK
                          : batch::cuda_fail("llama_batch_create: clear KV", cudaGetLastError());
    }
    if (!rc) rc = batch::alloc(b, &b->x, (size_t)rows * c.dim);
    if (!rc) rc = batch::alloc(b, &b->qkv, (size_t)rows * (qd + 2 * kvd));
    if (!rc) rc = batch::alloc(b, &b->q, (size_t)rows * qd);
    if (!rc) rc = batch::alloc(b, &b->att, (size_t)rows * qd);
    if (!rc) rc = batch::alloc(b, &b->gu, (size_t)rows * 2 * c.ffn);
    if (!rc) rc = batch::alloc(b, &b->logits, (size_t)rows * c.vocab);
    if (!rc) rc = batch::alloc(b, &b->attn_ws, std::max<size_t>(16, b->attn_ws_bytes / 4));
    if (!rc) rc = batch::alloc(b, &b->act, (size_t)rows * b->terms * kmax / 2);
    size_t act_img = 0;  // the largest activation scale image any pass of <= rows rows writes
    for (uint32_t r = 1; r <= rows; ++r)
        act_img = std::max(act_img, mma::scale_image_bytes(r * b->terms, kmax, batch::act_tile_rows(r * b->terms)));
    if (!rc) rc = batch::alloc(b, &b->act_s, act_img);
    if (!rc && cudaMemset(b->act_s, 0, act_img) != cudaSuccess)  // only finite E8M0 bytes are ever written
        rc = batch::cuda_fail("llama_batch_create: clear", cudaGetLastError());
    auto image = [&](const QMat &w) {
        uint8_t *img = nullptr;
        const size_t bytes = mma::scale_image_bytes(w.n, w.k, 128);
        int e = batch::alloc(b, &img, bytes);
        if (!e && cudaMemset(img, 0, bytes) != cudaSuccess)  // blocks past k in a partial last stage stay 0
            e = batch::cuda_fail("llama_batch_create: clear", cudaGetLastError());
        if (!e) {
            mma::scale_image_kernel<<<(unsigned)std::min<size_t>((bytes + 255) / 256, 8192), 256>>>(w.s, w.n, w.k, 128,
                                                                                                   img);
            e = check_launch("llama_batch_create: scale image");
        }
        b->wimg.push_back(img);
        return e;
    };
    for (uint32_t l = 0; l < c.n_layers && !rc; ++l) {
        const LayerW &L = m->layers[l];
        rc = image(L.qkv);
        if (!rc) rc = image(L.o);
        if (!rc) rc = image(L.gu);
        if (!rc) rc = image(L.down);
    }
    if (!rc) rc = image(m->lm_head);
    b->mma_part_bytes = batch::mma_ws_need(m, rows, b->terms);
    if (!rc) rc = batch::alloc(b, &b->mma_part, std::max<size_t>(4, b->mma_part_bytes / 4));
    if (!rc) rc = batch::alloc(b, &b->dec_tok, seqs);
    if (!rc) rc = batch::alloc(b, &b->dec_pos, seqs);
    if (!rc) rc = batch::alloc(b, &b->pf_tok, rows);
    if (!rc) rc = batch::alloc(b, &b->pf_pos, rows);
    if (!rc) rc = batch::alloc(b, &b->pf_cache, rows);
    if (!rc) rc = batch::alloc(b, &b->prompt, c.max_seq);
    if (!rc) rc = batch::alloc(b, &b->ids, (size_t)seqs * c.max_seq);
    if (!rc && m->cfg.tp_size > 1) {
        rc = batch::alloc(b, &b->part, (size_t)rows * c.dim);
        if (!rc) rc = tp::row_create(&b->rx, m->cfg.tp_rank, m->cfg.tp_size, (size_t)rows * c.dim);
    }
    if (!rc && (cudaMemset(b->qkv, 0, (size_t)rows * (qd + 2 * kvd) * 4) != cudaSuccess ||
                cudaMemset(b->gu, 0, (size_t)rows * 2 * c.ffn * 4) != cudaSuccess ||
                cudaMemset(b->dec_tok, 0, seqs * 4) != cudaSuccess || cudaMemset(b->dec_pos, 0, seqs * 4) != cudaSuccess ||
                cudaMemset(b->ids, 0, (size_t)seqs * c.max_seq * 4) != cudaSuccess))
        rc = batch::cuda_fail("llama_batch_create: clear", cudaGetLastError());
    if (!rc && cudaStreamCreateWithFlags(&b->cap_stream, cudaStreamNonBlocking) != cudaSuccess)
        rc = batch::cuda_fail("llama_batch_create: stream", cudaGetLastError());
    if (!rc && cudaDeviceSynchronize() != cudaSuccess) rc = batch::cuda_fail("llama_batch_create", cudaGetLastError());
    if (rc) {
        batch::destroy(b);
        return rc;
    }
    *out = b;
    return FP4X_OK;
}

}  // namespace batch
}  // namespace fp4x

extern "C" int llama_batch_create(fp4x_llama_model *m, uint32_t rows, fp4x_llama_batch **out) {
    return batch::create(m, rows, rows, nullptr, out);
}

extern "C" int llama_batch_destroy(fp4x_llama_batch *b) {
    batch::destroy(b);
    return FP4X_OK;
}

extern "C" int llama_batch_prefill(fp4x_llama_batch *b, fp4x_stream_t stream, uint32_t seq, const uint32_t *tokens,
                                   uint32_t n) {
    FP4X_REQUIRE(b && tokens, "llama_batch_prefill: null pointer");
    FP4X_REQUIRE(!b->rx || b->rx->connected, "llama_batch_prefill: tensor-parallel batch not connected");
    FP4X_REQUIRE(seq < b->seqs, "llama_batch_prefill: sequence %u of %u", seq, b->seqs);
    FP4X_REQUIRE(n >= 1 && b->len[seq] + n < b->max_seq, "llama_batch_prefill: %u tokens after %u exceed max_seq %u",
                 n, b->len[seq], b->max_seq);
    const uint32_t vocab = b->m->cfg.vocab;
    for (uint32_t i = 0; i < n; ++i)
        FP4X_REQUIRE(tokens[i] < vocab, "llama_batch_prefill: token %u out of vocab %u", tokens[i], vocab);
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaMemcpyAsync(b->prompt, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return batch::cuda_fail("llama_batch_prefill: upload", cudaGetLastError());
    for (uint32_t i0 = 0; i0 < n; i0 += b->rows) {
        const uint32_t R = std::min(b->rows, n - i0), pos0 = b->len[seq] + i0;
        batch::prefill_rows_kernel<<<1, 256, 0, st>>>(R, seq, pos0, b->prompt + i0, b->pf_tok, b->pf_pos, b->pf_cache,
                                                       b->ids, b->max_seq);
        FP4X_TRY(check_launch("llama_batch_prefill: rows"));
        const bool last = i0 + R == n;
        FP4X_TRY(batch::forward(b, st, R, b->pf_tok, b->pf_pos, b->pf_cache, last ? R - 1 : R));
        if (last) {
            FP4X_TRY(batch::argmax(b, st, 1, seq, pos0 + R));
        }
    }
    b->len[seq] += n;  // K/V of the prompt cached; the next token sits at position len
    return FP4X_OK;
}

extern "C" int llama_batch_set_length(fp4x_llama_batch *b, fp4x_stream_t stream, uint32_t seq, uint32_t len,
                                      uint32_t next_token) {
    FP4X_REQUIRE(b, "llama_batch_set_length: null pointer");
    FP4X_REQUIRE(seq < b->seqs && len < b->max_seq && next_token < b->m->cfg.vocab,
                 "llama_batch_set_length: sequence %u, length %u, token %u out of range", seq, len, next_token);
    cudaStream_t st = (cudaStream_t)stream;
    const uint32_t v[2] = {next_token, len};
    if (cudaMemcpyAsync(b->dec_tok + seq, &v[0], 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(b->dec_pos + seq, &v[1], 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(b->ids + (size_t)seq * b->max_seq + len, &v[0], 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return batch::cuda_fail("llama_batch_set_length", cudaGetLastError());
    b->len[seq] = len;
    return FP4X_OK;
}

extern "C" int llama_batch_decode(fp4x_llama_batch *b, fp4x_stream_t stream, uint32_t n_steps) {
    FP4X_REQUIRE(b, "llama_batch_decode: null pointer");
    FP4X_REQUIRE(!b->rx || b->rx->connected, "llama_batch_decode: tensor-parallel batch not connected");
    FP4X_REQUIRE(b->seqs == b->rows, "llama_batch_decode: a prefill-only batch");
    for (uint32_t s = 0; s < b->seqs; ++s)
        FP4X_REQUIRE(b->len[s] + n_steps < b->max_seq, "llama_batch_decode: sequence %u at %u + %u steps exceeds %u", s,
                     b->len[s], n_steps, b->max_seq);
    FP4X_TRY(batch::build_graph(b));
    cudaStream_t st = (cudaStream_t)stream;
    for (uint32_t i = 0; i < n_steps; ++i)
        if (cudaGraphLaunch(b->exec, st) != cudaSuccess) return batch::cuda_fail("llama_batch_decode", cudaGetLastError());
    for (uint32_t s = 0; s < b->seqs; ++s) b->len[s] += n_steps;
    b->last_rows = b->rows;
    return FP4X_OK;
}

extern "C" int llama_batch_tokens(fp4x_llama_batch *b, uint32_t seq, uint32_t *out, uint32_t n, uint32_t *len_out) {
    FP4X_REQUIRE(b && seq < (b ? b->seqs : 0), "llama_batch_tokens: bad sequence");
    const uint32_t len = b->len[seq] + 1;  // positions 0..len-1 hold tokens (the last one not yet consumed)
    if (len_out) *len_out = len;
    if (!out || n == 0) return FP4X_OK;
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(out, b->ids + (size_t)seq * b->max_seq, (size_t)std::min(n, len) * 4, cudaMemcpyDeviceToHost) !=
            cudaSuccess)
        return batch::cuda_fail("llama_batch_tokens", cudaGetLastError());
    return FP4X_OK;
}

extern "C" int llama_batch_logits(fp4x_llama_batch *b, float *out, uint32_t *rows_out) {
    FP4X_REQUIRE(b, "llama_batch_logits: null pointer");
    if (rows_out) *rows_out = b->last_rows;
    if (!out) return FP4X_OK;
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(out, b->logits, (size_t)b->last_rows * b->m->lc.vocab * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return batch::cuda_fail("llama_batch_logits", cudaGetLastError());
    return FP4X_OK;
}

extern "C" size_t llama_batch_kv_bytes(const fp4x_llama_batch *b) {
    if (!b) return 0;
    const fp4x_llama_config &c = b->m->lc;
    return (size_t)2 * c.n_layers * b->seqs * b->max_seq * c.n_kv_heads * c.head_dim * 2;
}

extern "C" int llama_batch_tp_handle(fp4x_llama_batch *b, void *handle_out) {
    FP4X_REQUIRE(b && handle_out, "llama_batch_tp_handle: null pointer");
    FP4X_REQUIRE(b->rx, "llama_batch_tp_handle: the model is not tensor parallel");
    return tp::row_export_handle(b->rx, handle_out);
}

extern "C" int llama_batch_tp_connect(fp4x_llama_batch *b, const void *handles) {
    FP4X_REQUIRE(b && handles, "llama_batch_tp_connect: null pointer");
    FP4X_REQUIRE(b->rx, "llama_batch_tp_connect: the model is not tensor parallel");
    return tp::row_connect(b->rx, handles);
}

namespace fp4x {
namespace batch {

// Hand-over from a batched prompt prefill to the model's device-resident loop:
// the first generated token is the next input at position n_prompt.
__global__ void finish_prefill_kernel(const uint32_t *first, uint32_t *state, uint32_t *out, uint32_t n_prompt) {
    const uint32_t g = first[0];
    state[0] = g, state[1] = n_prompt, state[2] = g;
    out[0] = g;
}

// Prompt prefill of the model (batch 1) through the batched engine: passes of up to
// 64 prompt tokens, K/V written into the model's own cache (a one-sequence batch
// cache has its [layer][max_seq][kvd] layout).  Replaces the token-at-a-time
// prefill of llama_run/src/main.rs:550-556.
int model_prefill(fp4x_llama_model *m, cudaStream_t st, const uint32_t *prompt, uint32_t n) {
    if (!m->pf) FP4X_TRY(create(m, std::min(64u, m->cfg.max_seq), 1, m->kv, &m->pf));
    m->pf->len[0] = 0;
    FP4X_TRY(llama_batch_prefill(m->pf, (fp4x_stream_t)st, 0, prompt, n));
    finish_prefill_kernel<<<1, 1, 0, st>>>(m->pf->dec_tok, m->state, m->out, n);
    return check_launch("llama_generate: prefill hand-over");
}

}  // namespace batch
}  // namespace fp4x
