/*
 * oracle.h -- CPU restatement of the reference's MXFP4 Llama decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path is
 * compared against; it is never linked into, loaded by, or called from the
 * product library.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it.
 *
 * Every function restates a CPU loop (or, where the reference has no CPU loop,
 * a device kernel body) of botBehavior/rust-fp4-blackwell; the citation on each
 * declaration is path:line inside that project.  Build flags: -O2
 * -ffp-contract=off (Rust never contracts a*b+c into an FMA; GCC would).
 * OpenMP is used only across independent rows / heads, keeping the per-row
 * accumulation order, so 1-thread and N-thread results are bit-identical.
 */
#ifndef FP4X_ORACLE_H
#define FP4X_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ RNG */

/* Marsaglia xorshift32 (13,17,5), the generator of every reference test:
 * examples/fp4_gemv/src/main.rs:101-107, llama_decode/src/main.rs:300-305. */
uint32_t orc_xorshift32(uint32_t *state);
void orc_xorshift32_fill(uint32_t seed, uint32_t *out, size_t n);

/* Synthetic-input generator (this framework's, not the reference's; shared
 * bit-for-bit with the device initialiser): the i-th splitmix64 output for
 * state `seed`, and a seeded N(0, sigma) draw built from it with the
 * Irwin-Hall(12) construction in exact integer arithmetic. */
uint64_t orc_hash64(uint64_t seed, uint64_t i);
float orc_normal(uint64_t seed, uint64_t i, float sigma);
void orc_fill_normal(uint64_t seed, uint64_t offset, float sigma, float *out, size_t n);
void orc_fill_normal_bf16(uint64_t seed, uint64_t offset, float sigma, uint16_t *out, size_t n);
void orc_fill_uniform_ids(uint64_t seed, uint32_t vocab, uint32_t *out, size_t n);

/* ------------------------------------------------------------- formats */

/* E2M1 decode, llama_run/src/main.rs:21-32 (identical in fp4_gemv/src/main.rs:20-30). */
float orc_e2m1_decode(uint32_t code);
/* bf16 <-> f32: widen as llama_run/src/main.rs:425; narrow with round-to-nearest-even. */
float orc_bf16_to_f32(uint16_t h);
uint16_t orc_f32_to_bf16(float f);
/* IEEE half -> f32, llama_run/src/main.rs:591-614. */
float orc_f16_to_f32(uint16_t h);
/* E8M0 scale byte for a block with max magnitude `amax`: 2^(floor(log2 amax) - 2),
 * exponent taken from the float's bits (BASELINE config 0 rule).  amax == 0 gives
 * 127 (scale 1.0), mirroring the reference's 1.0 fallback (llama_run:345). */
uint8_t orc_e8m0_from_amax(float amax);
float orc_e8m0_to_f32(uint8_t e);
/* Nearest-E2M1 code of v (already divided by its scale): strict '<' scan over the
 * ascending level table, so ties go to the smaller magnitude; v < 0 sets the sign
 * bit even when the magnitude rounds to 0 (llama_run/src/main.rs:347-363). */
uint32_t orc_e2m1_nearest(float v);

/* Reference quantiser, llama_run/src/main.rs:334-376: f32 scale = amax/6 per
 * (row, 32-block), 8 codes per u32 word, low nibble = lowest k. */
void orc_quant_ref(const float *w, size_t outd, size_t ind, uint32_t *packed, float *scales);
/* MXFP4 quantiser (config 0): E8M0 scale bytes, two codes per byte, low nibble first. */
void orc_quant_mxfp4(const float *w, size_t outd, size_t ind, uint8_t *packed, uint8_t *scales);
void orc_dequant_mxfp4(const uint8_t *packed, const uint8_t *scales, size_t n, size_t k, float *out);

/* ----------------------------------------------------------------- ops */

/* fp4_gemv CPU reference, examples/fp4_gemv/src/main.rs:135-142, reference storage
 * (u32 words, f32 scales, f32 x).  Order: acc += (fp4 * scale) * x[k]. */
void orc_gemv_ref(uint32_t n, uint32_t k, const uint32_t *w, const float *scales,
                  const float *x, float *y, int threads);
/* Same loop on native MXFP4 storage (u8 nibble pairs, E8M0 bytes) with bf16 x. */
void orc_gemv_mxfp4_bf16x(uint32_t n, uint32_t k, const uint8_t *w, const uint8_t *scales,
                          const uint16_t *x, float *y, int threads);
/* Same loop on native MXFP4 storage with f32 x (the engine's activations). */
void orc_gemv_mxfp4(uint32_t n, uint32_t k, const uint8_t *w, const uint8_t *scales,
                    const float *x, float *y, int threads);

/* RMSNorm, examples/llama_rmsnorm/src/main.rs:75-77. */
void orc_rmsnorm(uint32_t dim, float eps, const float *x, const float *weight, float *y);
/* RoPE cos/sin table [n_pos][head_dim/2] in f64 cast to f32, llama_run/src/main.rs:462-473. */
void orc_rope_tables(uint32_t n_pos, uint32_t head_dim, double theta, float *cos_t, float *sin_t);
/* In-place rotate-half RoPE, llama_rope/src/main.rs:74-84 (cos/sin at cos_base). */
void orc_rope(uint32_t num_heads, uint32_t head_dim, uint32_t cos_base,
              const float *cos_t, const float *sin_t, float *q);
/* KV append, llama_run/src/main.rs:140-146: dst[off + i] = src[i]. */
void orc_copy_into(uint32_t n, uint32_t off, const float *src, float *dst);
/* Single-query GQA attention, llama_attn_decode/src/main.rs:150-179.
 * Cache layout [seq][n_kv][head_dim], f32; out [n_heads][head_dim]. */
void orc_attn_decode(uint32_t n_heads, uint32_t n_kv, uint32_t head_dim, uint32_t seq,
                     const float *q, const float *kc, const float *vc, float *out, int threads);
/* Batched bf16 variant of the same loop (config 2 layout): q [B][n_heads][hd],
 * kc/vc [B][max_seq][n_kv][hd] bf16, out [B][n_heads][hd] bf16 (RNE of the f32 result). */
void orc_attn_decode_bf16(uint32_t batch, uint32_t n_heads, uint32_t n_kv, uint32_t head_dim,
                          uint32_t seq, uint32_t max_seq, const uint16_t *q, const uint16_t *kc,
                          const uint16_t *vc, uint16_t *out, int threads);
/* SwiGLU, llama_run/src/main.rs:244-252: out = g / (1 + exp(-g)) * u. */
void orc_swiglu(uint32_t n, const float *gate, const float *up, float *out);
/* Residual, llama_run/src/main.rs:254-261: x += y. */
void orc_residual(uint32_t n, const float *y, float *x);
/* Argmax with ties to the lowest index, llama_run/src/main.rs:263-315. */
uint32_t orc_argmax(uint32_t n, const float *logits);

/* Block-scaled FP4 x FP4 contraction (the fp4_mma semantics, trackb/fp4_scale_test.cu:112):
 * D[m][n] = sum_k (A[m][k] * SA[m][k/32]) * W[n][k] * SW[n][k/32], f32 accumulation in k
 * order.  A: [M][K/2] packed + [M][K/32] E8M0; W: [N][K/2] + [N][K/32]; D f32 [M][N]. */
void orc_mma_mxf4(uint32_t m, uint32_t n, uint32_t k, const uint8_t *a, const uint8_t *sa,
                  const uint8_t *w, const uint8_t *sw, float *d, int threads);

/* --------------------------------------------------------------- model */

typedef struct {
    uint32_t n_layers, dim, ffn, n_heads, n_kv_heads, head_dim, vocab, max_seq;
    float rope_theta, eps;
    uint64_t seed;
} orc_config;

/* NVFP4: E2M1 with an unsigned-E4M3 scale per 16 values and a per-tensor f32 g. */
float orc_ue4m3_to_f32(uint8_t b);
uint8_t orc_f32_to_ue4m3(float s);
void orc_quant_nvfp4(const float *w, size_t n, size_t k, uint8_t *packed, uint8_t *scales, float g);
void orc_mma_nvf4(uint32_t m, uint32_t n, uint32_t k, const uint8_t *a, const uint8_t *sa, const uint8_t *w,
                  const uint8_t *sw, float alpha, float *d, int threads);

typedef struct orc_model orc_model;

/* Random-init model, generated with the same tensor seeds as the device initialiser:
 * every linear N(0, 0.02) -> MXFP4 (config 0 rule), embeddings bf16 N(0, 0.02), norm
 * weights ones, bf16 KV cache.  Tensor seed = orc_hash64(cfg->seed, tensor_id) with
 * tensor_id 0 = embeddings, 1 = lm_head, 16 + 8*layer + {0..6} = q,k,v,o,gate,up,down. */
orc_model *orc_model_create(const orc_config *cfg, int threads);
void orc_model_destroy(orc_model *m);
/* Raw access (for cross-checking device tensors): which = tensor_id as above. */
const uint8_t *orc_model_packed(const orc_model *m, uint32_t tensor_id);
const uint8_t *orc_model_scales(const orc_model *m, uint32_t tensor_id);
const uint16_t *orc_model_embed(const orc_model *m);
/* Replace weights (checkpoint-loader tests): a linear (tensor_id as above, canonical
 * layout), the bf16 embeddings, or a norm weight vector (which: 0..L-1 attention,
 * L..2L-1 FFN, 2L final; ones after orc_model_create). */
void orc_model_set_tensor(orc_model *m, uint32_t tensor_id, const uint8_t *packed, const uint8_t *scales);
void orc_model_set_embed(orc_model *m, const uint16_t *embed);
void orc_model_set_norm(orc_model *m, uint32_t which, const float *w);
/* One token through the model at `pos` (llama_run/src/main.rs:509-535); writes
 * logits[vocab] and returns the argmax (UINT32_MAX, nothing written, if pos >=
 * max_seq or token >= vocab). */
uint32_t orc_forward(orc_model *m, uint32_t token, uint32_t pos, float *logits);
/* Greedy generation as the llama_run loop (llama_run/src/main.rs:544-570), EOS ignored. */
void orc_generate(orc_model *m, const uint32_t *prompt, uint32_t n_prompt, uint32_t n_gen,
                  uint32_t *out_ids);

int orc_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
