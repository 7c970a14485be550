// common.cuh -- shared device helpers for the sm_100a MXFP4 decode kernels.
//
// Formats (fixed by the reference and BASELINE config 0):
//   * E2M1 nibble: bit3 sign, bits2..1 exponent, bit0 mantissa; magnitudes
//     {0, .5, 1, 1.5, 2, 3, 4, 6} (examples/llama_run/src/main.rs:21-32).
//   * Packed weights: two nibbles per byte, low nibble = lower k; a row of K
//     weights is K/2 bytes.  The reference's u32 words (8 nibbles, low nibble
//     first, llama_run/src/main.rs:367-374) have the same little-endian bytes.
//   * E8M0 scale byte e: 2^(e-127) for one 32-element block along K.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "fp4x.h"

namespace fp4x {

// ---------------------------------------------------------------- errors
// Device-side error word (bit set by a kernel whose bounded wait expired);
// read and cleared by fp4x_device_error().
enum : uint32_t {
    DEVERR_MBAR_TIMEOUT = 1u << 0,
    DEVERR_FLAG_TIMEOUT = 1u << 1,
    DEVERR_BAD_ARG = 1u << 2,
};
// Defined here: the library is a single translation unit (fp4x_all.cu).
__device__ uint32_t g_device_error = 0;

__device__ __forceinline__ void raise_device_error(uint32_t bit) { atomicOr(&g_device_error, bit); }

// Upper bound on polling iterations of any mbarrier spin-wait.  Each poll may
// suspend for at most kSuspendHintNs, so the bound is ~2 s of wall time: far
// above any legitimate wait, far below a watchdog.
constexpr uint32_t kSpinLimit = 1u << 21;
constexpr uint32_t kSuspendHintNs = 1000;

// Poll bound of the waits on flags that ANOTHER rank raises (tensor-parallel
// exchanges and cross-rank grid barriers); 0 = each wait's compiled default.
// Set per device by fp4x_set_wait_limit, so that a caller (or a test) can make a
// wait on a rank that stopped issuing expire in about a millisecond.
__device__ uint32_t g_flag_wait_limit = 0;

__device__ __forceinline__ uint32_t flag_wait_limit(uint32_t dflt) {
    const uint32_t v = *(volatile uint32_t *)&g_flag_wait_limit;
    return v ? v : dflt;
}

// ---------------------------------------------------------------- smem/mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase), "r"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and raises the device error
// word) if the phase did not complete within kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase) {
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (mbar_try_wait(bar, phase)) return true;
    raise_device_error(DEVERR_MBAR_TIMEOUT);
    return false;
}

// Non-tensor bulk copy global -> shared, completion counted on `bar` in bytes.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same, with an L2 eviction hint policy (evict_first for streamed-once weights).
__device__ __forceinline__ void bulk_g2s_hint(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void prefetch_l2_bulk(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_l2_line(const void *src) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(src) : "memory");
}

// ---------------------------------------------------------------- PDL
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch with programmatic dependent launch: the kernel may be scheduled while the
// previous kernel of the stream finishes, so it must call pdl_wait() before it
// touches memory that kernel writes (or reads).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid, cfg.blockDim = block, cfg.dynamicSmemBytes = smem, cfg.stream = st;
    cfg.attrs = attr, cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ---------------------------------------------------------------- tensor-core fragments
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void *smem_row_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(smem_row_addr)));
}

__device__ __forceinline__ void ldmatrix_x2(uint32_t (&r)[2], const void *smem_row_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(smem_u32(smem_row_addr)));
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, f32 accumulate.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                              const float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + C, f32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                               const float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

// ---------------------------------------------------------------- E2M1 / E8M0
// One packed byte (two E2M1 codes, low nibble = lower k) -> f16x2 with the lower
// k in the low half, using the sm_100a hardware conversion.  E2M1 values are
// exact in f16.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
    uint32_t out;
    asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(out) : "r"(byte));
    return out;
}

// Eight codes of one 32-bit word -> four f16x2 (pairs (k0,k1) (k2,k3) (k4,k5) (k6,k7)).
// The word is split into its four bytes by one vector move (no per-byte
// extraction and narrowing), then one conversion per byte.
__device__ __forceinline__ void decode_word_f16(uint32_t w, uint32_t (&h)[4]) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
        : "r"(w));
}

// Scalar E2M1 decode in f32, exact; restates llama_run/src/main.rs:21-32 with
// the value table.
__device__ __forceinline__ float e2m1_to_f32(uint32_t code) {
    const uint32_t e = (code >> 1) & 3u, m = code & 1u;
    // e>0: 2^(e-1) * (1 + m/2)  ->  f32 exponent field 126+e, mantissa msb = m;  e==0: 0.5*m
    const float v = e ? __uint_as_float(((126u + e) << 23) | (m << 22)) : (m ? 0.5f : 0.0f);
    return (code & 8u) ? -v : v;
}

__device__ __forceinline__ float e8m0_to_f32(uint32_t e) {
    return e == 0 ? __uint_as_float(0x00400000u) : (e == 255 ? __uint_as_float(0x7FC00000u) : __uint_as_float(e << 23));
}

// ---------------------------------------------------------------- misc
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    __nv_bfloat16 h = __float2bfloat16_rn(f);
    return *reinterpret_cast<uint16_t *>(&h);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// splitmix64 output i for state `seed` (shared bit-for-bit with the host generator).
__host__ __device__ __forceinline__ uint64_t hash64(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Irwin-Hall(12) normal draw in exact integer arithmetic; one f32 multiply by sigma.
__host__ __device__ __forceinline__ float normal_draw(uint64_t seed, uint64_t i, float sigma) {
    int64_t acc = 0;
#pragma unroll
    for (int h = 0; h < 3; ++h) {
        uint64_t r = hash64(seed, 3 * i + (uint64_t)h);
        acc += (int64_t)(r & 0xFFFF) + (int64_t)((r >> 16) & 0xFFFF) + (int64_t)((r >> 32) & 0xFFFF) +
               (int64_t)(r >> 48);
    }
    float z = (float)(acc - 393210) * (1.0f / 65536.0f);
    return z * sigma;
}

}  // namespace fp4x

// ---------------------------------------------------------------- host side
namespace fp4x {
// Thread-local last-error message, returned by fp4x_last_error().
void set_error(const char *fmt, ...);
int check_launch(const char *what);
__host__ __device__ inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
int num_sms();
}  // namespace fp4x

#define FP4X_REQUIRE(cond, ...)              \
    do {                                     \
        if (!(cond)) {                       \
            ::fp4x::set_error(__VA_ARGS__);  \
            return FP4X_EINVAL;              \
        }                                    \
    } while (0)
