// persist.cuh -- the persistent decode kernel's schedule and parameters.
//
// One CTA per SM runs every token of a generation.  Each CTA owns a fixed
// share of every linear layer (the static schedule below); its weights are
// pre-packed into one contiguous per-CTA byte stream of "chunks" in exactly the
// order it consumes them, so a producer warp can stream them through a
// shared-memory ring with cp.async.bulk, running ahead across phases, layers
// and tokens, while the consumer warps wait on grid barriers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fp4x {
namespace persist {

constexpr int kConsumerWarps = 16;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + one producer warp
constexpr int kMaxSlots = 16;
constexpr int kMaxA = 8;      // QKV tiles per CTA
constexpr int kMaxUnits = 16;  // FFN half-block units per CTA
constexpr int kMaxL = 64;     // lm_head tiles per CTA
constexpr int kMaxBHeads = 4;  // attention heads whose O columns one CTA covers

// Per-CTA share of the model (identical for every layer and token).
struct CtaSched {
    uint32_t n_a, a_tile[kMaxA];      // QKV row tiles (engine QKV row order)
    uint32_t b_p0, b_p1;              // O "pairs" [p0, p1): pair = head * (dim/16) + row tile
    uint32_t n_c, c_unit[kMaxUnits];  // FFN units: unit = 2 * block + half (16 FFN indices)
    uint32_t n_l, l_tile[kMaxL];      // lm_head row tiles
    uint32_t n_chunks;                // chunks per token
    uint32_t pad;
    uint64_t stream_off;              // byte offset of this CTA's chunk stream in the arena
};

struct Params {
    uint32_t n_layers, dim, ffn, n_heads, n_kv, hd, vocab, max_seq;
    float eps;
    uint32_t q_tiles, k_tiles, o_tiles;  // o_tiles = dim / 16
    uint32_t slot_bytes, n_slots, pairs_per_chunk;
    const uint8_t *arena;
    const uint32_t *chunk_bytes;  // [grid][chunk_stride]
    uint32_t chunk_stride;
    const CtaSched *sched;
    const float *attn_norm, *ffn_norm;  // [n_layers][dim]
    const float *final_norm;
    const uint16_t *embed;              // [vocab][dim] bf16
    const float *cos_t, *sin_t;         // [max_seq][hd/2]
    uint16_t *kc, *vc;                  // [n_layers][max_seq][n_kv][hd] bf16
    float *X, *Y, *q, *logits;          // residual stream, FFN delta, q, logits
    float *cand_val;                    // [grid] per-CTA argmax candidates
    uint32_t *cand_idx;
    uint32_t *state;                    // [0] tok [1] pos [2] next [3] n_prompt [4] out capacity
    const uint32_t *prompt;
    uint32_t *out;
    uint32_t n_tokens;                  // forward passes in this launch
    uint32_t *bar;                      // [0] grid-barrier counter (zeroed before launch), [1] abort
};

// Byte sizes of the packed records.
constexpr uint32_t kBlockRec = 256 + 16;  // one 32-k block of a 16-row tile: nibbles + 16 scales
constexpr uint32_t kHalfRec = 128 + 16;   // one 16-k half block of a 16-row tile

}  // namespace persist
}  // namespace fp4x
