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
    // batched engine (both null otherwise): row b attends over positions
    // 0..row_pos[b] of cache row_cache[b] (prompt rows of one sequence share a cache)
    const uint32_t *row_pos = nullptr;
    const uint32_t *row_cache = nullptr;
};

// Sequence length and cache index of batch row b.
__device__ __forceinline__ uint32_t seq_of(const Params &p, uint32_t b) {
    if (p.row_pos) return min(p.row_pos[b] + 1, p.max_seq);
    return p.pos_ptr ? min(*p.pos_ptr + 1, p.max_seq) : p.seq;
}
__device__ __forceinline__ size_t cache_of(const Params &p, uint32_t b) { return p.row_cache ? p.row_cache[b] : b; }

// Engine form: f32 q/out, bf16 caches, fixed grid of p.splits slices.
int launch_engine(cudaStream_t stream, const Params &p, uint32_t head_dim, bool pdl);

}  // namespace attn
}  // namespace fp4x
