// persist_tc.cuh -- schedule and parameters of the tensor-core persistent decode
// kernel (tcgen05.mma.kind::mxf4; see persist_tc.cu).
//
// Every weight byte a CTA needs for a token is pre-packed, in consumption order,
// into one contiguous stream of "chunks".  A chunk is a run of MMA blocks of
// one (phase, unit) followed by their scale atoms:
//   * MMA block, K64 form (4096 B full): 128 weight rows x 64 k, K-major without
//     swizzle: 8-row group g, 32-k column c (0, 1), row r%8 -> byte
//     g*256 + c*128 + (r%8)*16 (16 bytes = 32 packed values); descriptor
//     LBO 128, SBO 256.
//   * MMA block, K32 form (2048 B full): 128 rows x 32 k (column 0 only), LBO 128,
//     SBO 128; the MMA's second k half reads neighbouring bytes and meets zero
//     activation terms.
//   * scale atom (512 B): blocks 2a, 2a+1 of the chunk, row r at
//     16*(r%32) + 4*(r/32) + byte, bytes {0,1} for block 2a, {2,3} for 2a+1
//     (a K32 block repeats its one scale in both bytes).
// A partial tile stores only its rows8 row groups (block bytes scale with it);
// the MMA still reads 16 groups, the missing ones from the bytes that follow
// (finite garbage: every E2M1 code is finite), and the epilogue ignores those rows.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fp4x {
namespace ptc {

constexpr int kCW = 16;                   // consumer warps
constexpr int kCons = kCW * 32;           // consumer threads
constexpr int kThreads = kCons + 64;      // + MMA warp + producer warp
constexpr int kMaxSlots = 16;                // chunks in flight (barrier pairs)
constexpr int kMaxOps = 48;               // chunk ops of one layer
constexpr int kMaxLmOps = 64;             // chunk ops of the lm_head
constexpr int kMaxAUnits = 4;             // QKV (tile, k-range) units per CTA
constexpr int kMaxPairs = 12;             // (head, O tile) pairs per CTA
constexpr int kMaxHeads = 4;              // heads attended per CTA
constexpr int kMaxGroup = 8;              // q heads per KV head (split attention units)
constexpr int kMaxTp = 8;                 // tensor-parallel ranks
constexpr uint32_t kSplitMinSeq = 512;    // longer contexts: attention split over (KV head, slice) units
constexpr int kMaxLm = 8;                 // lm_head tiles per CTA
constexpr int kMaxBlkPerChunk = 8;
constexpr uint32_t kSlotTarget = 34816;  // chunk bytes aimed at (one cp.async.bulk each)
constexpr uint32_t kBlk64 = 4096, kBlk32 = 2048, kAtom = 512;

enum : uint8_t { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DOWN = 3, PH_LM = 4, PH_N = 5 };

struct ChunkOp {
    uint32_t bytes;   // blocks + atoms
    uint8_t phase;
    uint8_t nblk;     // MMA blocks
    uint8_t kmode;    // 0: K64 blocks, 1: K32 blocks
    uint8_t bpa;      // blocks per accumulator (consecutive blocks share one)
    uint16_t bk0;     // operand-B k block (64 or 32 wide, as kmode) of block 0
    uint8_t acc0;     // accumulator of block 0 (8 TMEM columns each)
    uint8_t cont;     // block 0 continues the previous chunk's accumulation
    uint8_t rows8;    // 8-row groups stored per block (16 = a full 128-row tile)
    uint8_t pad[3];
};

struct Sched {
    uint32_t n_ops, n_lm_ops;
    uint32_t n_a, a_tile[kMaxAUnits];                            // QKV unit u: logical 128-row tile
    uint32_t n_pairs, pair_head[kMaxPairs], pair_tile[kMaxPairs];  // O pair i: acc i
    uint32_t h0, nh;                                             // attended heads [h0, h0 + nh)
    uint32_t f0, U;                                              // FFN indices [f0, f0 + U)
    uint32_t n_l, l_tile[kMaxLm];                                // lm_head tiles
    // FFN K split: ks CTAs share [f0, f0 + U), CTA part kh of them holding K range
    // kh / ks of gate/up and down output tiles [kh mt / ks, (kh + 1) mt / ks)
    uint32_t ks, kh;
    uint32_t pad;
    uint64_t stream_off;
    uint64_t layer_bytes, lm_bytes;
    ChunkOp ops[kMaxOps];
    ChunkOp lm_ops[kMaxLmOps];
    // per phase: the B scale atoms this CTA's blocks read, as up to two runs
    // (start, count, start, count), copied at phase start
    uint8_t batoms[PH_N][4];
    uint8_t pad2[4];
};

struct Params {
    uint32_t n_layers, dim, ffn, n_heads, n_kv, hd, vocab, max_seq;
    float eps;
    uint32_t qd, kvd;
    uint32_t ring_bytes, n_inflight;  // byte ring of chunks; chunks in flight (<= kMaxSlots)
    uint32_t acc_cols, sfb_col0, sfa_col0, tmem_cols;
    const uint8_t *arena;
    const Sched *sched;
    const float *attn_norm, *ffn_norm, *final_norm;  // [n_layers][dim]
    const uint16_t *embed;                           // [vocab][dim] bf16
    const float *cos_t, *sin_t;                      // [max_seq][hd/2]
    uint16_t *kc, *vc;                               // [n_layers][max_seq][kvd] bf16
    float *X, *Y, *qkv, *logits;                     // residual, FFN delta, QKV sums, logits
    float *attn_part;                                // [n_heads][attn_slices][hd + 2] split-attention partials
    uint32_t attn_slices;                            // sequence slices per KV head (0: no split attention)
    float *cand_val;
    uint32_t *cand_idx;
    uint32_t *state;  // [0] tok [1] pos [2] next [3] n_prompt [4] out capacity
    const uint32_t *prompt;
    uint32_t *out;
    uint32_t n_tokens;
    uint32_t *bar;        // [0] grid-barrier counter, [1] abort, [2] cross-rank release word
    uint64_t *ffx;        // FFN split partial gate/up sums [ffn / 64][2][128] as {tag, f32} words
    uint32_t launch_seq;  // launches of this engine so far (this one included): FFN split tags
    // tensor parallelism (tp_size 1: xr[0] = X, yr[0] = Y, cvr[0] = cand_val, cir[0] = cand_idx)
    uint32_t tp_rank, tp_size, v0;             // this rank, ranks, first vocab row of the lm_head shard
    float *xr[kMaxTp], *yr[kMaxTp];            // every rank's X and Y (row-parallel outputs add into all)
    float *cvr[kMaxTp];                        // every rank's candidate values [kMaxTp * grid]
    uint32_t *cir[kMaxTp];                     // ... and indices
    uint32_t *flagr[kMaxTp];                   // every rank's barrier flags, one 32-word line per source rank
    uint32_t *epoch;                           // cross-rank barrier epochs done so far (kept across launches)
    // Row-parallel exchange (tp_size > 1): the O and down partials are added into this
    // rank's own accumulators tpo / tpd (local atomics); after a local grid barrier
    // CTA i pushes its slice of them into every peer's receive slots
    // t{ro,rd}[peer][parity][this rank][dim] as tagged 64-bit words, polls its own
    // slots for every peer's slice, adds the ranks' slices in rank order into X, and
    // a local grid barrier follows.
    uint64_t *tro[kMaxTp], *trd[kMaxTp];
    float *tpo, *tpd;
    uint32_t *xepoch;                          // exchanges of each kind done so far (kept across launches)
};

}  // namespace ptc
}  // namespace fp4x
