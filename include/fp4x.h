/*
 * fp4x.h -- C ABI of the B200 (sm_100a) MXFP4 Llama decode hot path.
 *
 * Drop-in replacement for the operator API that botBehavior/rust-fp4-blackwell
 * generates with cuda-oxide's #[cuda_module] (one typed launch method per
 * #[kernel], examples/llama_run/src/main.rs:13-316, loaded at :488).  Each entry
 * point below names the reference kernel (path:line) it replaces.  Differences
 * from the reference boundary, all deliberate:
 *   - the caller passes a cudaStream_t first and the LIBRARY chooses the launch
 *     geometry (the reference's LaunchConfig, llama_run/src/main.rs:392-397, is
 *     dropped);
 *   - every call validates its arguments and returns an fp4x_status without
 *     launching anything on failure (the reference unwrap()s, :513-535);
 *   - pointers are raw device pointers with explicit sizes; no call allocates
 *     device memory on the per-token path.
 *
 * Thread safety: calls on distinct streams / distinct model handles may run
 * concurrently; the last-error string is thread-local.
 */
#ifndef FP4X_H
#define FP4X_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FP4X_API __attribute__((visibility("default")))
#else
#define FP4X_API
#endif

typedef struct CUstream_st *fp4x_stream_t; /* == cudaStream_t */

typedef enum {
    FP4X_OK = 0,
    FP4X_EINVAL = 1,      /* bad shape / alignment / null pointer; nothing launched */
    FP4X_ECUDA = 2,       /* a CUDA runtime call failed; see fp4x_last_error() */
    FP4X_ETIMEOUT = 3,    /* a bounded device-side wait expired */
    FP4X_ENOMEM = 4,      /* allocation failed (model creation only) */
    FP4X_EUNSUPPORTED = 5 /* valid request this build does not serve */
} fp4x_status;

/* ------------------------------------------------------------ library */

/* Message of the last failing call on this host thread ("" if none). */
FP4X_API const char *fp4x_last_error(void);
/* Library version string. */
FP4X_API const char *fp4x_version(void);
/* Synchronises `stream`, then reads and clears the device error word that
 * kernels set when a bounded wait expires.  Returns FP4X_ETIMEOUT if set. */
FP4X_API int fp4x_device_error(fp4x_stream_t stream, uint32_t *bits_out);
/* Poll bound of the device-side waits on flags that another rank raises (the
 * tensor-parallel exchanges and cross-rank grid barriers) on the CURRENT device;
 * 0 restores each wait's compiled default (about 2 s).  A wait that runs out sets
 * the device error word and the kernel returns, so fp4x_device_error() reports
 * FP4X_ETIMEOUT and the context stays usable.  Replaces the reference's unwrap()
 * panic on a failed launch or sync (examples/llama_run/src/main.rs:513-535) for
 * the multi-GPU case the reference does not have: a rank that stopped issuing is
 * detected in about `polls` x 0.1 us instead of hanging the others.  Not
 * synchronised with kernels already in flight. */
FP4X_API int fp4x_set_wait_limit(uint32_t polls);

/* ------------------------------------------------------------ formats */

/* Quantise an f32 [n][k] matrix to MXFP4 (E2M1 nibbles, two per byte, low
 * nibble = lower k; one E8M0 byte = 2^(floor(log2 amax) - 2) per 32-block),
 * values to the nearest E2M1 level with ties to the smaller magnitude.
 * Replaces quant_fp4, examples/llama_run/src/main.rs:334-376, with the E8M0
 * scale rule of the native format.  k % 32 == 0. */
FP4X_API int fp4_quantize_mxfp4(fp4x_stream_t stream, uint32_t n, uint32_t k, const float *w,
                       uint8_t *packed /* [n][k/2] */, uint8_t *scales /* [n][k/32] */);
/* Reference-layout quantiser, llama_run/src/main.rs:334-376 exactly: f32 scale
 * amax/6 (1.0 for an all-zero block), u32 words of 8 nibbles. */
FP4X_API int fp4_quantize_ref(fp4x_stream_t stream, uint32_t n, uint32_t k, const float *w,
                     uint32_t *packed /* [n][k/8] */, float *scales /* [n][k/32] */);
/* Dequantise MXFP4 to f32 (E2M1 x E8M0, exact). */
FP4X_API int fp4_dequantize_mxfp4(fp4x_stream_t stream, uint32_t n, uint32_t k, const uint8_t *packed,
                         const uint8_t *scales, float *out /* [n][k] */);
/* Seeded synthetic tensors (this library's generator: splitmix64 + Irwin-Hall(12)
 * normal, bit-identical on host and device). */
FP4X_API int fp4x_fill_normal_f32(fp4x_stream_t stream, uint64_t seed, uint64_t offset, float sigma, float *out,
                         size_t n);
FP4X_API int fp4x_fill_normal_bf16(fp4x_stream_t stream, uint64_t seed, uint64_t offset, float sigma,
                          uint16_t *out, size_t n);
/* Generate an [n][k] N(0, sigma) matrix from `seed` and quantise it to MXFP4 in
 * one pass (the f32 matrix is never materialised). */
FP4X_API int fp4x_init_mxfp4(fp4x_stream_t stream, uint64_t seed, float sigma, uint32_t n, uint32_t k,
                    uint8_t *packed, uint8_t *scales);

/* ------------------------------------------------------------ operators */

/* y[n] = sum_k e2m1(W[n,k]) * 2^(S[n,k/32]-127) * x[k]   (fp32 accumulation)
 * Native MXFP4 storage, bf16 activation.  Replaces fp4_gemv,
 * examples/llama_run/src/main.rs:34-77 (also fp4_gemv/src/main.rs:32-92).
 * k % 32 == 0, 32 <= k <= 16384, w 16-byte aligned. */
FP4X_API int fp4_gemv(fp4x_stream_t stream, uint32_t n, uint32_t k, const uint8_t *w /* [n][k/2] */,
             const uint8_t *scales /* [n][k/32] E8M0 */, const uint16_t *x /* bf16 [k] */,
             float *y /* [n] */);
/* Same operator on the reference's own storage: u32 words of 8 nibbles, f32
 * scales, f32 x -- argument-for-argument the reference kernel's signature
 * (llama_run/src/main.rs:35), a literal drop-in for its Layer buffers (:378-390). */
FP4X_API int fp4_gemv_ref(fp4x_stream_t stream, uint32_t n, uint32_t k, const uint32_t *w /* [n][k/8] */,
                 const float *scales /* [n][k/32] */, const float *x /* [k] */, float *y /* [n] */);
/* Native MXFP4 storage with an f32 activation (the decode engine's form). */
FP4X_API int fp4_gemv_f32x(fp4x_stream_t stream, uint32_t n, uint32_t k, const uint8_t *w, const uint8_t *scales,
                  const float *x, float *y);

/* Block-scaled MXFP4 x MXFP4 GEMM on tcgen05.mma.kind::mxf4 (fp32 accumulate):
 *   d[t][r] = sum_k A[t][k] * W[r][k],  A = a [m][k/2] nibbles + a_scales [m][k/32],
 *   W = w [n][k/2] + w_scales [n][k/32] (E8M0), d = [m][n].
 * The reference's MMA is the single-warp m16n8k64 known-answer test
 * fp4_mma_allones (examples/fp4_mma/src/main.rs:18-54, sm_120a mma.sync); this
 * is the batched-decode / prefill GEMM built on it.  k must be a multiple of 64;
 * a and w 16-byte aligned.  When the tile grid is too small to fill the GPU the
 * K range is split: each split stores its fp32 partial tile in the workspace
 * (plain stores, no atomics) and a second kernel (splitk_reduce_kernel, same
 * stream) adds the splits in split order and writes d (deterministic), so the
 * workspace holds fp4_mma_workspace_size(m, n, k) bytes (0 = none needed; may
 * then be NULL). */
FP4X_API size_t fp4_mma_workspace_size(uint32_t m, uint32_t n, uint32_t k);
FP4X_API int fp4_mma(fp4x_stream_t stream, uint32_t m, uint32_t n, uint32_t k, const uint8_t *a,
                     const uint8_t *a_scales, const uint8_t *w, const uint8_t *w_scales, uint16_t *d_bf16,
                     void *workspace, size_t workspace_bytes);
/* Same GEMM with fp32 output (exact accumulator values; no workspace, so no
 * K split: one CTA per output tile). */
FP4X_API int fp4_mma_f32(fp4x_stream_t stream, uint32_t m, uint32_t n, uint32_t k, const uint8_t *a,
                         const uint8_t *a_scales, const uint8_t *w, const uint8_t *w_scales, float *d);
/* NVFP4 form of the same GEMM (the reference's kind::mxf4nvf4 / scale_vec::4X /
 * .ue4m3 variant, trackb/FP4_M16N8K64_LAYOUT.md:7): E2M1 operands with one unsigned
 * E4M3 scale per 16 values ([rows][k/16] bytes), d = alpha * A W^T (alpha carries
 * the operands' per-tensor scales).  Runs tcgen05.mma.kind::mxf4nvf4.block16. */
FP4X_API size_t fp4_mma_nvf4_workspace_size(uint32_t m, uint32_t n, uint32_t k);
FP4X_API int fp4_mma_nvf4(fp4x_stream_t stream, uint32_t m, uint32_t n, uint32_t k, const uint8_t *a,
                          const uint8_t *a_scales, const uint8_t *w, const uint8_t *w_scales, float alpha,
                          uint16_t *d_bf16, void *workspace, size_t workspace_bytes);
FP4X_API int fp4_mma_nvf4_f32(fp4x_stream_t stream, uint32_t m, uint32_t n, uint32_t k, const uint8_t *a,
                              const uint8_t *a_scales, const uint8_t *w, const uint8_t *w_scales, float alpha,
                              float *d);
/* NVFP4 quantiser: per 16-block s = amax / 6 / global_scale rounded to the nearest
 * UE4M3 (ties to even, saturating at 448), values / (UE4M3(s) * global_scale)
 * rounded to E2M1 with the reference's tie rule (llama_run/src/main.rs:350-362).
 * k % 16 == 0; packed [n][k/2], scales [n][k/16]. */
FP4X_API int fp4_quantize_nvfp4(fp4x_stream_t stream, uint32_t n, uint32_t k, const float *w, uint8_t *packed,
                                uint8_t *scales, float global_scale);
/* The reference's known-answer test on the tcgen05 path: A = B = all 1.0
 * (bytes 0x22), every scale 2^0 (0x7F), K = 64; out[16*8] = D, every value 64.0.
 * Replaces fp4_mma_allones, examples/fp4_mma/src/main.rs:18-54 (check :75-85). */
FP4X_API int fp4_mma_allones(fp4x_stream_t stream, float *out);

/* y = x * rsqrt(mean(x^2) + eps) * weight.  Replaces rmsnorm,
 * llama_run/src/main.rs:79-116 (test llama_rmsnorm/src/main.rs:14-56). */
FP4X_API int llama_rmsnorm(fp4x_stream_t stream, uint32_t dim, float eps, const float *x, const float *weight,
                  float *y);
/* In-place rotate-half RoPE on q [num_heads][head_dim] with cos/sin rows at
 * cos_base (= pos * head_dim/2).  Replaces rope, llama_run/src/main.rs:118-138. */
FP4X_API int llama_rope(fp4x_stream_t stream, uint32_t num_heads, uint32_t head_dim, uint32_t cos_base,
               const float *cos_t, const float *sin_t, float *q);
/* Fill RoPE tables [n_pos][head_dim/2]: freq_j = theta^(-2j/hd) and angle
 * pos*freq_j in f64, cast to f32 (llama_run/src/main.rs:462-471); computed on
 * the host and copied to `cos_t`/`sin_t` (device). */
FP4X_API int llama_rope_tables(fp4x_stream_t stream, uint32_t n_pos, uint32_t head_dim, double theta, float *cos_t,
                      float *sin_t);
/* dst[off + i] = src[i], i < n.  Replaces copy_into, llama_run/src/main.rs:140-146. */
FP4X_API int llama_copy_into(fp4x_stream_t stream, uint32_t n, uint32_t off, const float *src, float *dst);
/* bf16 KV append: dst_bf16[off + i] = bf16(src[i]) (the native bf16 cache). */
FP4X_API int llama_kv_append_bf16(fp4x_stream_t stream, uint32_t n, uint32_t off, const float *src, uint16_t *dst);
/* out = g / (1 + exp(-g)) * u.  Replaces swiglu, llama_run/src/main.rs:244-252. */
FP4X_API int llama_swiglu(fp4x_stream_t stream, uint32_t n, const float *gate, const float *up, float *out);
/* x += y.  Replaces residual, llama_run/src/main.rs:254-261. */
FP4X_API int llama_residual(fp4x_stream_t stream, uint32_t n, const float *y, float *x);
/* out[0] = argmax(logits), ties to the lowest index.  Replaces argmax,
 * llama_run/src/main.rs:263-315. */
FP4X_API int llama_argmax(fp4x_stream_t stream, uint32_t n, const float *logits, uint32_t *out);

/* Single-query GQA attention on the reference's f32 cache layout
 * [seq][n_kv][64]: out[h] = softmax(q[h] . K^T / sqrt(64)) V over t < seq.
 * Argument-for-argument attn_decode, llama_run/src/main.rs:149 (head_dim is the
 * reference's compile-time HD = 64, :19); kernel body :148-242, test
 * llama_attn_decode/src/main.rs:18-129.  Any seq >= 1 (the reference caps seq at
 * its shared-memory MAXSEQ).  No workspace: one CTA per q head. */
FP4X_API int llama_attn_decode(fp4x_stream_t stream, uint32_t n_heads, uint32_t n_kv_heads, uint32_t seq,
                      const float *q, const float *kc, const float *vc, float *out);
/* Same with head_dim in {64, 128} and split-KV over the sequence when a
 * workspace of llama_attn_workspace_size() bytes is given (NULL: no split). */
FP4X_API int llama_attn_decode_hd(fp4x_stream_t stream, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                         uint32_t seq, const float *q, const float *kc, const float *vc, float *out,
                         void *workspace, size_t workspace_bytes);
/* Bytes of split-KV partials the batched attention entry points use for this
 * shape (0: no split needed). */
FP4X_API size_t llama_attn_workspace_size(uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                                 uint32_t seq);
/* Batched bf16 flash-decode: q [B][n_heads][hd] bf16,
 * caches [B][max_seq][n_kv][hd] bf16 (the reference's per-sequence layout,
 * llama_run/src/main.rs:388-389, stacked over the batch), out [B][n_heads][hd]
 * bf16; softmax scale 1/sqrt(hd), causal at position seq-1. */
FP4X_API int llama_attn_decode_bf16(fp4x_stream_t stream, uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads,
                           uint32_t head_dim, uint32_t seq, uint32_t max_seq, const uint16_t *q,
                           const uint16_t *kc, const uint16_t *vc, uint16_t *out, void *workspace,
                           size_t workspace_bytes);
/* No counterpart in the reference: an allocation-free llama_attn_decode_bf16
 * for callers that cannot allocate device memory (their device memory belongs
 * to a pool allocator of the host, or their serving loop forbids cudaMalloc /
 * cudaFree).  The split-KV partials live in one static device array of
 * llama_attn_noalloc_max_bytes() bytes (4 MiB) that every GPU loading the
 * library keeps until exit; a shape needing more returns FP4X_EINVAL.  The
 * first call in each CUDA context (per device: its primary context for runtime
 * API callers) looks the array up (make it before any stream capture); the
 * address is cached per context id, so a driver-API context or a context made
 * after a device reset gets its own lookup.  Calls share the array: calls that
 * overlap on the GPU race, so issue them on one stream. */
FP4X_API int llama_attn_decode_bf16_noalloc(fp4x_stream_t stream, uint32_t batch, uint32_t n_heads,
                                            uint32_t n_kv_heads, uint32_t head_dim, uint32_t seq, uint32_t max_seq,
                                            const uint16_t *q, const uint16_t *kc, const uint16_t *vc,
                                            uint16_t *out);
/* Size of the static scratch array used by llama_attn_decode_bf16_noalloc. */
FP4X_API size_t llama_attn_noalloc_max_bytes(void);
/* The decode engine's form: f32 q and out, bf16 caches. */
FP4X_API int llama_attn_decode_f32q_bf16kv(fp4x_stream_t stream, uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads,
                                  uint32_t head_dim, uint32_t seq, uint32_t max_seq, const float *q,
                                  const uint16_t *kc, const uint16_t *vc, float *out, void *workspace,
                                  size_t workspace_bytes);

/* ------------------------------------------------------------ decode engine */

/* Model shape + synthetic-init seed.  The reference hard-codes these as consts
 * (examples/llama_run/src/main.rs:318-330, llama_decode/src/main.rs:289-298). */
typedef struct fp4x_llama_config {
    uint32_t n_layers, dim, ffn, n_heads, n_kv_heads, head_dim, vocab, max_seq;
    float rope_theta, eps;
    uint64_t seed;     /* tensor seeds = splitmix64(seed, tensor id) */
    uint32_t tp_rank;  /* tensor-parallel shard of this process (0 without TP) */
    uint32_t tp_size;  /* 1 (or 0) without TP */
} fp4x_llama_config;

typedef struct fp4x_llama_model fp4x_llama_model;

/* Allocate and random-initialise a model on the current device: every linear
 * (including lm_head) N(0, 0.02) quantised to MXFP4 with the E8M0 rule,
 * embeddings bf16 N(0, 0.02), norm weights ones, bf16 KV cache, RoPE tables;
 * captures the per-token CUDA graph.  Replaces the model set-up of
 * llama_run/src/main.rs:432-489 (real weights) / llama_decode/src/main.rs:367-426
 * (random weights). */
FP4X_API int llama_model_create(const fp4x_llama_config *cfg, fp4x_llama_model **out);
FP4X_API int llama_model_destroy(fp4x_llama_model *m);
/* Model from a real-weight checkpoint: a safetensors file with Hugging Face Llama
 * tensor names (model.embed_tokens.weight, model.layers.N.self_attn.{q,k,v,o}_proj
 * .weight, model.layers.N.mlp.{gate,up,down}_proj.weight, model.layers.N.
 * {input,post_attention}_layernorm.weight, model.norm.weight, lm_head.weight or tied
 * embeddings), dtypes F32 / BF16 / F16, shapes matching cfg.  Every linear is
 * quantised to MXFP4 on the GPU (the fp4_quantize_mxfp4 rule), embeddings kept as
 * bf16, norm weights f32; under tensor parallelism each rank reads its shard.
 * Replaces the reference's loading and host quantisation, llama_run/src/main.rs:
 * 413-460 (f16/bf16 widening :425-427, :591-614; quant_fp4 :334-376). */
FP4X_API int llama_model_create_from_safetensors(const fp4x_llama_config *cfg, const char *path,
                                                 fp4x_llama_model **out);
/* Host-only: dtype (0 F32, 1 BF16, 2 F16, -1 other), rank and shape (up to 8 dims)
 * of tensor `name` in a safetensors file; FP4X_EINVAL if the file is malformed or
 * the tensor is absent. */
FP4X_API int fp4x_safetensors_info(const char *path, const char *name, uint32_t *dtype_out, uint64_t *shape_out,
                                   uint32_t *ndim_out);
/* Zero the KV cache. */
FP4X_API int llama_model_reset(fp4x_llama_model *m, fp4x_stream_t stream);
/* forward(tok, pos) -> next token, llama_run/src/main.rs:492-536: one token at
 * `pos`, writes the argmax (ties to the lowest index) to *next_host and, when
 * non-NULL, the logits [vocab] to logits_host.  Synchronous, as the reference's
 * per-token to_host_vec (:535). */
FP4X_API int llama_forward(fp4x_llama_model *m, fp4x_stream_t stream, uint32_t token, uint32_t pos,
                           uint32_t *next_host, float *logits_host);
/* One token of the device-resident loop (decode_step, llama_decode/src/main.rs:428-477):
 * consumes the device token/position left by the previous step, asynchronous. */
FP4X_API int llama_decode_step(fp4x_llama_model *m, fp4x_stream_t stream);
/* n tokens of the device-resident loop in one call (one launch on the
 * persistent path). */
FP4X_API int llama_decode_steps(fp4x_llama_model *m, fp4x_stream_t stream, uint32_t n);
/* Decode path: 2 = persistent kernel on tcgen05 MXFP4 MMAs (one cooperative
 * launch runs many tokens; default when the shape fits), 1 = persistent kernel
 * with CUDA-core MXFP4 decode, 0 = CUDA graph of fused per-layer kernels.
 * FP4X_DECODE_PATH=graph|persistent selects 0|1 at creation. */
FP4X_API int llama_model_set_path(fp4x_llama_model *m, int path);
/* Tensor parallelism (no counterpart in the single-GPU
 * reference): create the model on every rank with cfg.tp_rank / cfg.tp_size set
 * (one process per GPU; KV heads and ffn/32 must split evenly).  Each rank holds
 * its shard: the q/k/v rows of its heads, the O columns of those heads, its
 * gate/up rows and down columns, and vocab rows [v0, v0 + vocab_local) of
 * lm_head.  Then exchange the 64-byte handles (llama_model_tp_handle on every
 * rank, gathered in rank order by the host) and call llama_model_tp_connect on
 * every rank; it maps the peers' exchange areas (CUDA IPC over NVLink) and builds
 * the decode graph, whose O and down projections end in an in-graph peer-memory
 * allreduce and whose lm_head ends in a cross-rank argmax.  All ranks must then
 * issue the same calls (llama_forward / llama_generate / decode steps) in the
 * same order.  llama_forward returns this rank's logits slice. */
FP4X_API int llama_model_tp_handle(fp4x_llama_model *m, void *handle_out /* 64 bytes */);
FP4X_API int llama_model_tp_connect(fp4x_llama_model *m, const void *handles /* tp_size x 64 bytes */);
FP4X_API int llama_model_shard(const fp4x_llama_model *m, uint32_t *v0, uint32_t *vocab_local);
FP4X_API int llama_model_get_path(const fp4x_llama_model *m);
/* Greedy generation as the llama_run loop (llama_run/src/main.rs:544-587, EOS
 * ignored): prefill the prompt, then n_gen tokens.  The prompt is prefilled in
 * multi-token passes of the batched engine (tcgen05 GEMMs, 64 positions per pass)
 * straight into the model's KV cache; under tensor parallelism, or with the
 * environment variable FP4X_PREFILL=serial, it runs one position at a time
 * through the decode path as the reference does (:550-556).  Either way the last
 * prompt position yields the first generated token.  prompt/out_ids are HOST
 * arrays; *prefill_ms covers the prefill, *decode_ms the remaining n_gen-1
 * tokens (the reference's timed tokens, :554-562). */
FP4X_API int llama_generate(fp4x_llama_model *m, fp4x_stream_t stream, const uint32_t *prompt, uint32_t n_prompt,
                            uint32_t n_gen, uint32_t *out_ids, float *prefill_ms, float *decode_ms);
/* Copy one MXFP4 tensor of the model to host in canonical row order (tensor id
 * 1 = lm_head, 16 + 8*layer + {0..6} = q,k,v,o,gate,up,down); n_out/k_out get
 * its shape.  Test hook for parity with the oracle. */
FP4X_API int llama_model_export_tensor(fp4x_llama_model *m, uint32_t tensor_id, uint8_t *packed_host,
                                       uint8_t *scales_host, uint32_t *n_out, uint32_t *k_out);
/* Copy the bf16 embedding table [vocab][dim] to host. */
FP4X_API int llama_model_embedding(fp4x_llama_model *m, uint16_t *embed_host);
/* Kernel launches in one token's CUDA graph. */
FP4X_API uint32_t llama_model_kernels_per_token(const fp4x_llama_model *m);
/* MXFP4 bytes (packed + scales) streamed per token (all linears incl. lm_head). */
FP4X_API size_t llama_model_weight_bytes(const fp4x_llama_model *m);

/* ---- Batched engine (BASELINE config 4 at batch 64; batched prompt prefill).
 * The reference decodes one sequence and prefills token by token
 * (llama_run/src/main.rs:544-587); here `rows` sequences with their own bf16 KV
 * caches ([layer][rows][max_seq][kvd]) run through the model's weights together,
 * every linear layer on the tcgen05 fp4_mma GEMM (activations as 8-term MXFP4
 * sums, fp32 accumulation).  The model handle must outlive the batch.  Under
 * tensor parallelism (a model created with tp_size > 1) every rank creates its
 * batch over its shard, exchanges the 64-byte handles (llama_batch_tp_handle on
 * every rank, gathered in rank order) and calls llama_batch_tp_connect; the
 * row-parallel O and down outputs are then summed across ranks over NVLink peer
 * memory and the argmax runs across the vocab shards.  All ranks must issue the
 * same batch calls in the same order. */
typedef struct fp4x_llama_batch fp4x_llama_batch;
FP4X_API int llama_batch_create(fp4x_llama_model *m, uint32_t rows /* 1..256 */, fp4x_llama_batch **out);
FP4X_API int llama_batch_destroy(fp4x_llama_batch *b);
/* Prefill n prompt tokens (HOST array) of sequence `seq` after its current
 * length, up to `rows` tokens per pass, each attending causally; the argmax of
 * the last one becomes the sequence's next token. */
FP4X_API int llama_batch_prefill(fp4x_llama_batch *b, fp4x_stream_t stream, uint32_t seq, const uint32_t *tokens,
                                 uint32_t n);
/* Declare sequence `seq` to hold `len` cached positions (whatever the cache
 * holds there, zeros after creation) with `next_token` at position len: a
 * context set-up for throughput runs without a prefill. */
FP4X_API int llama_batch_set_length(fp4x_llama_batch *b, fp4x_stream_t stream, uint32_t seq, uint32_t len,
                                    uint32_t next_token);
/* n_steps greedy decode steps of all `rows` sequences (one CUDA graph each). */
FP4X_API int llama_batch_decode(fp4x_llama_batch *b, fp4x_stream_t stream, uint32_t n_steps);
/* Token history of sequence `seq` (positions 0..len-1, the last one the next
 * token to be consumed) to a HOST array; *len_out gets len.  Synchronous. */
FP4X_API int llama_batch_tokens(fp4x_llama_batch *b, uint32_t seq, uint32_t *out_host, uint32_t n,
                                uint32_t *len_out);
/* Logits of the last pass to a HOST array [*rows_out][vocab] (decode: one row
 * per sequence; prefill: the last prompt token).  Synchronous. */
FP4X_API int llama_batch_logits(fp4x_llama_batch *b, float *logits_host, uint32_t *rows_out);
FP4X_API int llama_batch_tp_handle(fp4x_llama_batch *b, void *handle_out /* 64 bytes */);
FP4X_API int llama_batch_tp_connect(fp4x_llama_batch *b, const void *handles /* tp_size x 64 bytes */);
/* Bytes of the batch's KV caches. */
FP4X_API size_t llama_batch_kv_bytes(const fp4x_llama_batch *b);

#ifdef __cplusplus
}
#endif
#endif /* FP4X_H */
