// attention.cuh -- parameters of the split-KV flash-decode kernels (attention.cu),
// shared with the decode engine (engine.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fp4x {
namespace attn {

struct Params {
    uint32_t batch, n_heads, n_kv, seq, max_seq, splits, split_len;
    float scale;
    const void *q;            // [B][n_heads][hd]
    const void *kc;           // [B][max_seq][n_kv][hd]
    const void *vc;
    void *out;                // [B][n_heads][hd]
    float *ws;                // [B][n_heads][splits][hd + 2] partials (splits > 1)
    const uint32_t *pos_ptr;  // engine: seq = *pos_ptr + 1 read on the device (else seq)
};

// Engine form: f32 q/out, bf16 caches, fixed grid of p.splits slices.
int launch_engine(cudaStream_t stream, const Params &p, uint32_t head_dim, bool pdl);

}  // namespace attn
}  // namespace fp4x
