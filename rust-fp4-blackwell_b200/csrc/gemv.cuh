// gemv.cuh -- arguments of the fused MXFP4 GEMV kernel (gemv.cu), shared with
// the decode engine (engine.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fp4x {
namespace gemv {

constexpr int kRows = 16;              // rows per CTA (one mma M tile)
constexpr int kWarps = 8;              // K split across warps
constexpr int kThreads = kWarps * 32;
constexpr uint32_t kMaxK = 16384;

// Prologue: how the activation vector is produced.
enum { PRO_NONE = 0, PRO_RMSNORM = 1, PRO_EMBED_RMSNORM = 2 };
// Epilogue: what happens to the 16 row results of a tile.
enum { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_QKV_ROPE = 3 };

struct Args {
    uint32_t n, k;             // rows (stored order), contraction length
    const uint8_t *w;          // [n][k/2] packed E2M1
    const void *scales;        // [n][k/32] E8M0 bytes (or f32 for the reference layout)
    const void *x;             // activation [k] (bf16 or f32)
    float *y;                  // EPI_STORE/EPI_SWIGLU output, EPI_RESIDUAL residual stream (in place)
    // RMSNorm prologue
    const float *norm_w;
    float eps;
    // embedding prologue
    const uint16_t *embed;     // [vocab][k] bf16
    const uint32_t *tok;       // device token id
    float *x_out;              // residual stream written by CTA 0
    // QKV + RoPE + KV-append epilogue
    uint32_t q_tiles, k_tiles, n_kv, head_dim;
    const float *cos_t, *sin_t;  // [max_seq][hd/2]
    const uint32_t *pos;         // device position
    uint32_t max_seq;            // cache capacity (positions)
    float *q_out;                // [n_heads][hd]
    uint16_t *kc, *vc;           // this layer's cache [max_seq][n_kv][hd] bf16
};

// Launch one fused variant (E8M0 scales, f32 activation) with optional PDL.
int launch_fused(cudaStream_t stream, int pro, int epi, const Args &a, bool pdl);

}  // namespace gemv
}  // namespace fp4x
