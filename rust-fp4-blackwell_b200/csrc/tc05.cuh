// tc05.cuh -- sm_100a tensor-core (tcgen05) and TMA building blocks for the
// block-scaled MXFP4 MMA (tcgen05.mma.kind::mxf4.block_scale.block32).
//
// Operand staging (both operands K-major, one 128-byte row = 256 E2M1 values):
//   * A tile = 128 rows, B tile = N rows (8..256), each row 128 bytes of packed
//     nibbles (low nibble = lower k), stored with the 128-byte swizzle that a
//     TMA load with CU_TENSOR_MAP_SWIZZLE_128B produces: the 16-byte chunk c of
//     row r sits at r*128 + ((c ^ (r % 8)) * 16) inside a 1024-byte-aligned
//     tile.  One MMA consumes K = 64 (32 bytes); the 4 MMAs of a row advance the
//     descriptor start address by 32 bytes (the swizzle is applied by the
//     hardware on absolute address bits, so the advance stays inside the atom).
//   * Scale factors (E8M0, one per 32 values) live in tensor memory.  A 512-byte
//     shared "scale atom" holds 128 rows x 4 consecutive k-blocks at byte
//     16*(r%32) + 4*(r/32) + j; tcgen05.cp.32x128b.warpx4 copies it to 4 TMEM
//     columns (lane r%32 of every lane quarter, column r/32, byte j), and the two
//     K=64 MMAs of that K=128 range select bytes {0,1} and {2,3} (scale id 0, 2).
//   * The accumulator is fp32 in TMEM: lane = A row, column = B row.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace fp4x {
namespace tc {

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (sm_100 format): start, leading and stride
// byte offsets in 16-byte units, version 1, layout type in bits 61..63.
enum : uint32_t { kLayoutNone = 0, kLayoutSw128 = 2 };

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
    d |= (uint64_t)(layout & 7u) << 61;
    return d;
}

// K-major operand tile with 128-byte swizzle: 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) { return smem_desc(saddr, 16, 1024, kLayoutSw128); }

// 512-byte scale atom as the source of tcgen05.cp.32x128b: 32 rows of 16 bytes,
// 8-row core matrices 128 bytes apart.
__device__ __forceinline__ uint64_t desc_scale_atom(uint32_t saddr) {
    return smem_desc(saddr, 128, 128, kLayoutNone);
}

// Instruction descriptor of kind::mxf4 (E2M1 x E2M1, E8M0 scales, K = 64 dense,
// both operands K-major, fp32 accumulate), M = 128, N = n (multiple of 8).
__host__ __device__ constexpr uint32_t idesc_mxf4(uint32_t n) {
    return (1u << 7)              // a format E2M1
           | (1u << 10)           // b format E2M1
           | ((n >> 3) << 17)     // N / 8
           | (1u << 23)           // scale format E8M0
           | ((128u >> 4) << 24);  // M / 16
}

// Instruction descriptor of kind::mxf4nvf4 with UE4M3 scales per 16 values
// (NVFP4, scale_vec::4X), otherwise as idesc_mxf4.
__host__ __device__ constexpr uint32_t idesc_nvf4(uint32_t n) {
    return (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);  // scale format bit 23 = 0: UE4M3
}

// ---------------------------------------------------------------- TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 32 bits, 8 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- MMA issue (one thread)
// (no memory clobber: ordering against the mbarrier waits comes from volatile-asm order)
__device__ __forceinline__ void utccp_scale_atom(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc));
}

// D[tmem_d] (+)= A * B^T with block scales; scale ids ride in bits 30..31 of the
// scale-factor TMEM addresses and in the instruction descriptor.
__device__ __forceinline__ void mma_mxf4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
    const uint32_t id = idesc | ((tsfa >> 30) << 29) | ((tsfb >> 30) << 4);
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(id), "r"(tsfa), "r"(tsfb), "r"(accumulate));
}

// NVFP4 form: 4 UE4M3 scales per row per K=64 (one 32-bit TMEM column), no scale id.
__device__ __forceinline__ void mma_nvf4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(tsfa), "r"(tsfb), "r"(accumulate));
}

// Arrive on `bar` once every tcgen05 operation issued so far by this thread is done.
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// ---------------------------------------------------------------- TMA (no cluster forms)
__device__ __forceinline__ void tma_load_2d(void *dst_smem, const CUtensorMap *map, int32_t x, int32_t y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst_smem)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Tile stores shared -> global (bulk async-group of the issuing thread).  The box
// is written where it lies inside the tensor; parts outside it are dropped.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, int32_t x, int32_t y, const void *src_smem) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(smem_u32(src_smem))
                 : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, int32_t x, int32_t y, int32_t z,
                                             const void *src_smem) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(z), "r"(smem_u32(src_smem))
                 : "memory");
}
// Element-wise add of the box into global memory (performed by the L2).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, int32_t x, int32_t y,
                                                  const void *src_smem) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(smem_u32(src_smem))
                 : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Byte offset of scale (row r, block j in 0..3) inside a 512-byte scale atom.
__host__ __device__ constexpr uint32_t scale_atom_off(uint32_t r, uint32_t j) {
    return 16u * (r & 31u) + 4u * (r >> 5) + j;
}

// Host: 2-D row-major byte matrix [rows][pitch] as a tensor map with a
// 128-byte x box_rows box and the 128-byte swizzle.  Returns false on failure.
bool make_map_sw128(CUtensorMap *map, const void *base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows);

// Host: output tensor [planes][rows][cols] of bf16 (elem 2) or f32 (elem 4),
// row-major, as a tensor map with a box of box_cols x box_rows (x 1 plane), no
// swizzle: the shared-memory image of a box is [box_rows][box_cols].  cols x elem
// must be a multiple of 16.  Returns false on failure.
bool make_map_out(CUtensorMap *map, void *base, uint32_t elem, uint64_t cols, uint64_t rows, uint64_t planes,
                  uint32_t box_cols, uint32_t box_rows);

// Bulk reduction of `bytes` (multiple of 16) of f32 from shared memory into global
// memory (element-wise add, performed by the L2 a sector at a time), tracked by
// the issuing thread's bulk async-group.
__device__ __forceinline__ void bulk_reduce_add_f32(float *gdst, const void *ssrc, uint32_t bytes) {
    asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(gdst),
                 "r"(smem_u32(ssrc)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk operation of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

}  // namespace tc
}  // namespace fp4x
