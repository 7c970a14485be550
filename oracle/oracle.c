/*
 * oracle.c -- CPU restatement of the reference's MXFP4 decode path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Compiled with -O2 -ffp-contract=off
 * so that every a*b+c stays two roundings, as in the Rust reference.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static int nthreads(int t) { return t > 0 ? t : orc_max_threads(); }

/* ------------------------------------------------------------------ RNG */

/* examples/fp4_gemv/src/main.rs:102-107 */
uint32_t orc_xorshift32(uint32_t *s) {
    uint32_t x = *s;
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    *s = x;
    return x;
}

void orc_xorshift32_fill(uint32_t seed, uint32_t *out, size_t n) {
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) out[i] = orc_xorshift32(&s);
}

/* splitmix64: output i of the generator whose state starts at `seed`. */
uint64_t orc_hash64(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Irwin-Hall(12): twelve 16-bit uniforms from three hashes, summed as integers.
 * The centred sum has standard deviation 65536 (to 1 part in 10^9), so
 * z = (sum - 393210) / 65536 is exact in f32 and approximately N(0, 1). */
float orc_normal(uint64_t seed, uint64_t i, float sigma) {
    int64_t acc = 0;
    for (int h = 0; h < 3; ++h) {
        uint64_t r = orc_hash64(seed, 3 * i + (uint64_t)h);
        acc += (int64_t)(r & 0xFFFF) + (int64_t)((r >> 16) & 0xFFFF) +
               (int64_t)((r >> 32) & 0xFFFF) + (int64_t)(r >> 48);
    }
    float z = (float)(acc - 393210) * (1.0f / 65536.0f);
    return z * sigma;
}

void orc_fill_normal(uint64_t seed, uint64_t offset, float sigma, float *out, size_t n) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; ++i) out[i] = orc_normal(seed, offset + i, sigma);
}

void orc_fill_normal_bf16(uint64_t seed, uint64_t offset, float sigma, uint16_t *out, size_t n) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_bf16(orc_normal(seed, offset + i, sigma));
}

void orc_fill_uniform_ids(uint64_t seed, uint32_t vocab, uint32_t *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = (uint32_t)(orc_hash64(seed, i) % vocab);
}

/* ------------------------------------------------------------- formats */

/* llama_run/src/main.rs:21-32 */
float orc_e2m1_decode(uint32_t code) {
    uint32_t e = (code >> 1) & 3;
    float m = (float)(code & 1);
    float mag;
    if (e == 0) {
        mag = 0.5f * m;
    } else {
        float base = (float)(1u << (e - 1));
        mag = base + base * 0.5f * m;
    }
    return (code & 8) ? -mag : mag;
}

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* llama_run/src/main.rs:425: bf16 bits << 16 */
float orc_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

uint16_t orc_f32_to_bf16(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return (uint16_t)(u >> 16);
}

/* llama_run/src/main.rs:591-614 */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 0x1f, mant = h & 0x3ff, f;
    if (exp == 0) {
        if (mant == 0) {
            f = sign << 31;
        } else {
            int32_t e = -14;
            uint32_t m = mant;
            while ((m & 0x400) == 0) { m <<= 1; e -= 1; }
            m &= 0x3ff;
            f = (sign << 31) | ((uint32_t)(e + 127) << 23) | (m << 13);
        }
    } else if (exp == 0x1f) {
        f = (sign << 31) | (0xffu << 23) | (mant << 13);
    } else {
        f = (sign << 31) | ((exp - 15 + 127) << 23) | (mant << 13);
    }
    return u2f(f);
}

/* floor(log2(a)) of a positive finite float, from its bits. */
static int floor_log2_bits(float a) {
    uint32_t u = f2u(a) & 0x7FFFFFFFu;
    int ef = (int)(u >> 23);
    if (ef != 0) return ef - 127;
    /* subnormal: value = m * 2^-149 */
    uint32_t m = u & 0x7FFFFFu;
    return (31 - __builtin_clz(m)) - 149;
}

uint8_t orc_e8m0_from_amax(float amax) {
    if (!(amax > 0.0f)) return 127; /* zero block: scale 1.0, as llama_run:345 */
    int e = floor_log2_bits(amax) - 2 + 127;
    if (e < 0) e = 0;
    if (e > 254) e = 254;
    return (uint8_t)e;
}

float orc_e8m0_to_f32(uint8_t e) {
    if (e == 0) return u2f(0x00400000u); /* 2^-127, subnormal */
    if (e == 255) return u2f(0x7FC00000u);
    return u2f((uint32_t)e << 23);
}

/* llama_run/src/main.rs:332 */
static const float LEVELS[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

/* llama_run/src/main.rs:348-363 */
uint32_t orc_e2m1_nearest(float v) {
    float a = fabsf(v);
    uint32_t bc = 0;
    float bd = 3.40282347e+38f; /* f32::MAX */
    for (uint32_t ci = 0; ci < 8; ++ci) {
        float d = fabsf(a - LEVELS[ci]);
        if (d < bd) { bd = d; bc = ci; }
    }
    uint32_t code = bc;
    if (v < 0.0f) code |= 8;
    return code;
}

/* llama_run/src/main.rs:334-376 */
void orc_quant_ref(const float *w, size_t outd, size_t ind, uint32_t *packed, float *scales) {
    size_t nb = ind / 32;
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < outd; ++r) {
        for (size_t b = 0; b < nb; ++b) {
            size_t base = r * ind + b * 32;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(w[base + i]));
            float scale = amax > 0.0f ? amax / 6.0f : 1.0f;
            scales[r * nb + b] = scale;
            uint32_t words[4] = {0, 0, 0, 0};
            for (int i = 0; i < 32; ++i) {
                float v = w[base + i] / scale;
                words[i / 8] |= orc_e2m1_nearest(v) << ((i % 8) * 4);
            }
            for (int j = 0; j < 4; ++j) packed[base / 8 + j] = words[j];
        }
    }
}

void orc_quant_mxfp4(const float *w, size_t outd, size_t ind, uint8_t *packed, uint8_t *scales) {
    size_t nb = ind / 32;
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < outd; ++r) {
        for (size_t b = 0; b < nb; ++b) {
            size_t base = r * ind + b * 32;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(w[base + i]));
            uint8_t e = orc_e8m0_from_amax(amax);
            float scale = orc_e8m0_to_f32(e);
            scales[r * nb + b] = e;
            for (int i = 0; i < 32; i += 2) {
                uint32_t lo = orc_e2m1_nearest(w[base + i] / scale);
                uint32_t hi = orc_e2m1_nearest(w[base + i + 1] / scale);
                packed[base / 2 + i / 2] = (uint8_t)(lo | (hi << 4));
            }
        }
    }
}

void orc_dequant_mxfp4(const uint8_t *packed, const uint8_t *scales, size_t n, size_t k, float *out) {
    for (size_t r = 0; r < n; ++r)
        for (size_t i = 0; i < k; ++i) {
            uint8_t byte = packed[(r * k + i) / 2];
            uint32_t code = (i & 1) ? (byte >> 4) : (byte & 0xF);
            out[r * k + i] = orc_e2m1_decode(code) * orc_e8m0_to_f32(scales[r * (k / 32) + i / 32]);
        }
}

/* ----------------------------------------------------------------- ops */

/* examples/fp4_gemv/src/main.rs:130-142 */
void orc_gemv_ref(uint32_t n, uint32_t k, const uint32_t *w, const float *scales,
                  const float *x, float *y, int threads) {
    uint32_t blocks = k / 32;
#pragma omp parallel for schedule(static) num_threads(nthreads(threads))
    for (uint32_t r = 0; r < n; ++r) {
        float acc = 0.0f;
        for (uint32_t kk = 0; kk < k; ++kk) {
            size_t idx = (size_t)r * k + kk;
            uint32_t code = (w[idx / 8] >> ((idx % 8) * 4)) & 0xF;
            acc += orc_e2m1_decode(code) * scales[(size_t)r * blocks + kk / 32] * x[kk];
        }
        y[r] = acc;
    }
}

static float decode_lut[16];
static int lut_ready = 0;
static void ensure_lut(void) {
    if (!lut_ready) {
        for (uint32_t c = 0; c < 16; ++c) decode_lut[c] = orc_e2m1_decode(c);
        lut_ready = 1;
    }
}

void orc_gemv_mxfp4(uint32_t n, uint32_t k, const uint8_t *w, const uint8_t *scales,
                    const float *x, float *y, int threads) {
    ensure_lut();
    uint32_t blocks = k / 32;
#pragma omp parallel for schedule(static) num_threads(nthreads(threads))
    for (uint32_t r = 0; r < n; ++r) {
        const uint8_t *row = w + (size_t)r * (k / 2);
        const uint8_t *srow = scales + (size_t)r * blocks;
        float acc = 0.0f;
        for (uint32_t b = 0; b < blocks; ++b) {
            float sc = orc_e8m0_to_f32(srow[b]);
            for (uint32_t i = 0; i < 32; ++i) {
                uint32_t kk = b * 32 + i;
                uint8_t byte = row[kk / 2];
                uint32_t code = (kk & 1) ? (uint32_t)(byte >> 4) : (uint32_t)(byte & 0xF);
                acc += decode_lut[code] * sc * x[kk];
            }
        }
        y[r] = acc;
    }
}

void orc_gemv_mxfp4_bf16x(uint32_t n, uint32_t k, const uint8_t *w, const uint8_t *scales,
                          const uint16_t *x, float *y, int threads) {
    float *xf = (float *)malloc(sizeof(float) * k);
    for (uint32_t i = 0; i < k; ++i) xf[i] = orc_bf16_to_f32(x[i]);
    orc_gemv_mxfp4(n, k, w, scales, xf, y, threads);
    free(xf);
}

/* examples/llama_rmsnorm/src/main.rs:75-77 */
void orc_rmsnorm(uint32_t dim, float eps, const float *x, const float *weight, float *y) {
    float ss = 0.0f;
    for (uint32_t i = 0; i < dim; ++i) ss += x[i] * x[i];
    float rms = 1.0f / sqrtf(ss / (float)dim + eps);
    for (uint32_t i = 0; i < dim; ++i) y[i] = x[i] * rms * weight[i];
}

/* llama_run/src/main.rs:462-471 */
void orc_rope_tables(uint32_t n_pos, uint32_t head_dim, double theta, float *cos_t, float *sin_t) {
    uint32_t half = head_dim / 2;
    for (uint32_t pos = 0; pos < n_pos; ++pos)
        for (uint32_t j = 0; j < half; ++j) {
            double freq = 1.0 / pow(theta, 2.0 * (double)j / (double)head_dim);
            double a = (double)pos * freq;
            cos_t[(size_t)pos * half + j] = (float)cos(a);
            sin_t[(size_t)pos * half + j] = (float)sin(a);
        }
}

/* llama_rope/src/main.rs:74-84; table offset as llama_run/src/main.rs:118-138 */
void orc_rope(uint32_t num_heads, uint32_t head_dim, uint32_t cos_base,
              const float *cos_t, const float *sin_t, float *q) {
    uint32_t half = head_dim / 2;
    for (uint32_t h = 0; h < num_heads; ++h) {
        uint32_t base = h * head_dim;
        for (uint32_t j = 0; j < half; ++j) {
            float c = cos_t[cos_base + j], s = sin_t[cos_base + j];
            float x0 = q[base + j], x1 = q[base + j + half];
            q[base + j] = x0 * c - x1 * s;
            q[base + j + half] = x1 * c + x0 * s;
        }
    }
}

/* llama_run/src/main.rs:140-146 */
void orc_copy_into(uint32_t n, uint32_t off, const float *src, float *dst) {
    for (uint32_t i = 0; i < n; ++i) dst[off + i] = src[i];
}

/* llama_attn_decode/src/main.rs:148-179 */
void orc_attn_decode(uint32_t n_heads, uint32_t n_kv, uint32_t head_dim, uint32_t seq,
                     const float *q, const float *kc, const float *vc, float *out, int threads) {
    uint32_t group = n_heads / n_kv;
    float scale = 1.0f / sqrtf((float)head_dim);
#pragma omp parallel for schedule(static) num_threads(nthreads(threads))
    for (uint32_t h = 0; h < n_heads; ++h) {
        uint32_t kvh = h / group;
        float *sc = (float *)malloc(sizeof(float) * (seq ? seq : 1));
        float m = -3.40282347e+38f; /* f32::MIN */
        for (uint32_t t = 0; t < seq; ++t) {
            float d = 0.0f;
            for (uint32_t i = 0; i < head_dim; ++i)
                d += q[h * head_dim + i] * kc[((size_t)t * n_kv + kvh) * head_dim + i];
            sc[t] = d * scale;
            if (sc[t] > m) m = sc[t];
        }
        float l = 0.0f;
        for (uint32_t t = 0; t < seq; ++t) {
            sc[t] = expf(sc[t] - m);
            l += sc[t];
        }
        for (uint32_t i = 0; i < head_dim; ++i) {
            float acc = 0.0f;
            for (uint32_t t = 0; t < seq; ++t) acc += sc[t] * vc[((size_t)t * n_kv + kvh) * head_dim + i];
            out[h * head_dim + i] = acc / l;
        }
        free(sc);
    }
}

void orc_attn_decode_bf16(uint32_t batch, uint32_t n_heads, uint32_t n_kv, uint32_t head_dim,
                          uint32_t seq, uint32_t max_seq, const uint16_t *q, const uint16_t *kc,
                          const uint16_t *vc, uint16_t *out, int threads) {
    uint32_t group = n_heads / n_kv;
    float scale = 1.0f / sqrtf((float)head_dim);
#pragma omp parallel for collapse(2) schedule(static) num_threads(nthreads(threads))
    for (uint32_t b = 0; b < batch; ++b)
        for (uint32_t h = 0; h < n_heads; ++h) {
            uint32_t kvh = h / group;
            const uint16_t *qh = q + ((size_t)b * n_heads + h) * head_dim;
            const uint16_t *kb = kc + (size_t)b * max_seq * n_kv * head_dim;
            const uint16_t *vb = vc + (size_t)b * max_seq * n_kv * head_dim;
            float *sc = (float *)malloc(sizeof(float) * (seq ? seq : 1));
            float *qf = (float *)malloc(sizeof(float) * head_dim);
            for (uint32_t i = 0; i < head_dim; ++i) qf[i] = orc_bf16_to_f32(qh[i]);
            float m = -3.40282347e+38f;
            for (uint32_t t = 0; t < seq; ++t) {
                float d = 0.0f;
                const uint16_t *kr = kb + ((size_t)t * n_kv + kvh) * head_dim;
                for (uint32_t i = 0; i < head_dim; ++i) d += qf[i] * orc_bf16_to_f32(kr[i]);
                sc[t] = d * scale;
                if (sc[t] > m) m = sc[t];
            }
            float l = 0.0f;
            for (uint32_t t = 0; t < seq; ++t) {
                sc[t] = expf(sc[t] - m);
                l += sc[t];
            }
            for (uint32_t i = 0; i < head_dim; ++i) {
                float acc = 0.0f;
                for (uint32_t t = 0; t < seq; ++t)
                    acc += sc[t] * orc_bf16_to_f32(vb[((size_t)t * n_kv + kvh) * head_dim + i]);
                out[((size_t)b * n_heads + h) * head_dim + i] = orc_f32_to_bf16(acc / l);
            }
            free(qf);
            free(sc);
        }
}

/* llama_run/src/main.rs:244-252 */
void orc_swiglu(uint32_t n, const float *gate, const float *up, float *out) {
    for (uint32_t i = 0; i < n; ++i) {
        float g = gate[i];
        float s = g / (1.0f + expf(-g));
        out[i] = s * up[i];
    }
}

/* llama_run/src/main.rs:254-261 */
void orc_residual(uint32_t n, const float *y, float *x) {
    for (uint32_t i = 0; i < n; ++i) x[i] = x[i] + y[i];
}

/* llama_run/src/main.rs:263-315: largest value, ties to the lowest index;
 * the running best starts at -1e30 with index 0. */
uint32_t orc_argmax(uint32_t n, const float *logits) {
    float bv = -1e30f;
    uint32_t bi = 0;
    for (uint32_t i = 0; i < n; ++i)
        if (logits[i] > bv) { bv = logits[i]; bi = i; }
    return bi;
}

/* trackb/fp4_scale_test.cu:112 order: s += A*SFA*B*SFB over k. */
void orc_mma_mxf4(uint32_t m, uint32_t n, uint32_t k, const uint8_t *a, const uint8_t *sa,
                  const uint8_t *w, const uint8_t *sw, float *d, int threads) {
    ensure_lut();
    uint32_t kb = k / 32;
#pragma omp parallel for schedule(static) num_threads(nthreads(threads))
    for (uint32_t i = 0; i < m; ++i)
        for (uint32_t j = 0; j < n; ++j) {
            float s = 0.0f;
            for (uint32_t kk = 0; kk < k; ++kk) {
                uint8_t ab = a[((size_t)i * k + kk) / 2], wb = w[((size_t)j * k + kk) / 2];
                float av = decode_lut[(kk & 1) ? (ab >> 4) : (ab & 0xF)];
                float wv = decode_lut[(kk & 1) ? (wb >> 4) : (wb & 0xF)];
                s += av * orc_e8m0_to_f32(sa[(size_t)i * kb + kk / 32]) * wv *
                     orc_e8m0_to_f32(sw[(size_t)j * kb + kk / 32]);
            }
            d[(size_t)i * n + j] = s;
        }
}

/* ------------------------------------------------------------- NVFP4 */
/* NVFP4 (the reference's kind::mxf4nvf4 / scale_vec::4X / .ue4m3 variant,
 * trackb/FP4_M16N8K64_LAYOUT.md:7, trackb/nvf4_m16n8k64_template.ptx): E2M1 codes
 * with one unsigned E4M3 scale per 16 values and a per-tensor f32 scale g.  The
 * reference ships no quantiser for it; this library's rule, shared bit for bit
 * with the device: per 16-block s = amax / 6 / g rounded to the nearest UE4M3
 * (ties to even, saturating at 448, zero for s <= 0), then each value divided by
 * UE4M3(s) * g and rounded to E2M1 with the reference's tie rule (quant_fp4,
 * llama_run/src/main.rs:350-362). */
float orc_ue4m3_to_f32(uint8_t b) {
    uint32_t e = (b >> 3) & 15u, m = b & 7u;
    return e == 0 ? ldexpf((float)m, -9) : ldexpf((float)(8u + m), (int)e - 10);
}

uint8_t orc_f32_to_ue4m3(float s) {
    if (!(s > 0.0f)) return 0;
    if (s >= 448.0f) return 0x7E;
    if (s < 0.015625f) { /* below 2^-6: subnormal step 2^-9 */
        float m = rintf(s * 512.0f);
        return (uint8_t)m; /* m == 8 is the smallest normal, 0x08 */
    }
    uint32_t bits;
    memcpy(&bits, &s, 4);
    int e = (int)((bits >> 23) & 0xFFu) - 127;
    float mant = ldexpf(s, -e) - 1.0f; /* exact */
    int E = e + 7, m = (int)rintf(mant * 8.0f);
    if (m == 8) E += 1, m = 0;
    if (E > 15 || (E == 15 && m == 7)) return 0x7E;
    return (uint8_t)((E << 3) | m);
}

void orc_quant_nvfp4(const float *w, size_t n, size_t k, uint8_t *packed, uint8_t *scales, float g) {
    size_t nb = k / 16;
    for (size_t r = 0; r < n; ++r)
        for (size_t b = 0; b < nb; ++b) {
            size_t base = r * k + b * 16;
            float amax = 0.0f;
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(w[base + i]));
            uint8_t S = orc_f32_to_ue4m3(amax / 6.0f / g);
            float eff = orc_ue4m3_to_f32(S) * g;
            scales[r * nb + b] = S;
            for (int i = 0; i < 16; i += 2) {
                uint32_t lo = eff > 0.0f ? orc_e2m1_nearest(w[base + i] / eff) : 0u;
                uint32_t hi = eff > 0.0f ? orc_e2m1_nearest(w[base + i + 1] / eff) : 0u;
                packed[base / 2 + i / 2] = (uint8_t)(lo | (hi << 4));
            }
        }
}

/* d[t][r] = alpha * sum_k e2m1(A[t][k]) UE4M3(SA[t][k/16]) e2m1(W[r][k]) UE4M3(SW[r][k/16]). */
void orc_mma_nvf4(uint32_t m, uint32_t n, uint32_t k, const uint8_t *a, const uint8_t *sa, const uint8_t *w,
                  const uint8_t *sw, float alpha, float *d, int threads) {
    ensure_lut();
    uint32_t kb = k / 16;
#pragma omp parallel for schedule(static) num_threads(nthreads(threads))
    for (uint32_t i = 0; i < m; ++i)
        for (uint32_t j = 0; j < n; ++j) {
            float s = 0.0f;
            for (uint32_t kk = 0; kk < k; ++kk) {
                uint8_t ab = a[((size_t)i * k + kk) / 2], wb = w[((size_t)j * k + kk) / 2];
                float av = decode_lut[(kk & 1) ? (ab >> 4) : (ab & 0xF)];
                float wv = decode_lut[(kk & 1) ? (wb >> 4) : (wb & 0xF)];
                s += av * orc_ue4m3_to_f32(sa[(size_t)i * kb + kk / 16]) * wv *
                     orc_ue4m3_to_f32(sw[(size_t)j * kb + kk / 16]);
            }
            d[(size_t)i * n + j] = alpha * s;
        }
}

/* --------------------------------------------------------------- model */

enum { T_EMBED = 0, T_LMHEAD = 1, T_LAYER0 = 16 };
enum { M_Q = 0, M_K, M_V, M_O, M_GATE, M_UP, M_DOWN, M_COUNT };

typedef struct {
    uint8_t *packed;
    uint8_t *scales;
    uint32_t n, k;
} qmat;

struct orc_model {
    orc_config c;
    int threads;
    qmat *lin; /* [n_layers * 7] */
    qmat lm_head;
    uint16_t *embed;
    float *norms;      /* [2 n_layers + 1][dim]: attention norms, FFN norms, final norm (ones) */
    uint16_t *kc, *vc; /* [n_layers][max_seq][n_kv][hd] bf16 */
    float *cos_t, *sin_t;
    float *x, *h, *q, *k, *v, *a, *ao, *g, *u, *s, *d, *logits;
};

static void mat_dims(const orc_config *c, int which, uint32_t *n, uint32_t *k) {
    uint32_t qd = c->n_heads * c->head_dim, kvd = c->n_kv_heads * c->head_dim;
    switch (which) {
    case M_Q: *n = qd; *k = c->dim; break;
    case M_K: *n = kvd; *k = c->dim; break;
    case M_V: *n = kvd; *k = c->dim; break;
    case M_O: *n = c->dim; *k = qd; break;
    case M_GATE: *n = c->ffn; *k = c->dim; break;
    case M_UP: *n = c->ffn; *k = c->dim; break;
    default: *n = c->dim; *k = c->ffn; break;
    }
}

/* Generate N(0, 0.02) weights of one tensor and quantise them, one row at a time
 * (keeps host memory at the packed size). */
static void make_qmat(qmat *m, uint64_t tseed, uint32_t n, uint32_t k) {
    m->n = n;
    m->k = k;
    m->packed = (uint8_t *)malloc((size_t)n * k / 2);
    m->scales = (uint8_t *)malloc((size_t)n * k / 32);
#pragma omp parallel
    {
        float *row = (float *)malloc(sizeof(float) * k);
#pragma omp for schedule(static)
        for (uint32_t r = 0; r < n; ++r) {
            for (uint32_t i = 0; i < k; ++i) row[i] = orc_normal(tseed, (uint64_t)r * k + i, 0.02f);
            orc_quant_mxfp4(row, 1, k, m->packed + (size_t)r * k / 2, m->scales + (size_t)r * k / 32);
        }
        free(row);
    }
}

orc_model *orc_model_create(const orc_config *cfg, int threads) {
    orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
    m->c = *cfg;
    m->threads = threads;
    const orc_config *c = cfg;
    m->lin = (qmat *)calloc((size_t)c->n_layers * M_COUNT, sizeof(qmat));
    for (uint32_t l = 0; l < c->n_layers; ++l)
        for (int w = 0; w < M_COUNT; ++w) {
            uint32_t n, k;
            mat_dims(c, w, &n, &k);
            make_qmat(&m->lin[l * M_COUNT + w], orc_hash64(c->seed, T_LAYER0 + 8u * l + (uint32_t)w), n, k);
        }
    make_qmat(&m->lm_head, orc_hash64(c->seed, T_LMHEAD), c->vocab, c->dim);
    size_t ne = (size_t)c->vocab * c->dim;
    m->embed = (uint16_t *)malloc(ne * 2);
    orc_fill_normal_bf16(orc_hash64(c->seed, T_EMBED), 0, 0.02f, m->embed, ne);
    m->norms = (float *)malloc(sizeof(float) * (2 * (size_t)c->n_layers + 1) * c->dim);
    for (size_t i = 0; i < (2 * (size_t)c->n_layers + 1) * c->dim; ++i) m->norms[i] = 1.0f;
    size_t kvn = (size_t)c->n_layers * c->max_seq * c->n_kv_heads * c->head_dim;
    m->kc = (uint16_t *)calloc(kvn, 2);
    m->vc = (uint16_t *)calloc(kvn, 2);
    m->cos_t = (float *)malloc(sizeof(float) * c->max_seq * (c->head_dim / 2));
    m->sin_t = (float *)malloc(sizeof(float) * c->max_seq * (c->head_dim / 2));
    orc_rope_tables(c->max_seq, c->head_dim, (double)c->rope_theta, m->cos_t, m->sin_t);
    uint32_t qd = c->n_heads * c->head_dim, kvd = c->n_kv_heads * c->head_dim;
    m->x = (float *)malloc(sizeof(float) * c->dim);
    m->h = (float *)malloc(sizeof(float) * c->dim);
    m->q = (float *)malloc(sizeof(float) * qd);
    m->k = (float *)malloc(sizeof(float) * kvd);
    m->v = (float *)malloc(sizeof(float) * kvd);
    m->a = (float *)malloc(sizeof(float) * qd);
    m->ao = (float *)malloc(sizeof(float) * c->dim);
    m->g = (float *)malloc(sizeof(float) * c->ffn);
    m->u = (float *)malloc(sizeof(float) * c->ffn);
    m->s = (float *)malloc(sizeof(float) * c->ffn);
    m->d = (float *)malloc(sizeof(float) * c->dim);
    m->logits = (float *)malloc(sizeof(float) * c->vocab);
    return m;
}

void orc_model_destroy(orc_model *m) {
    if (!m) return;
    free(m->norms);
    for (uint32_t i = 0; i < m->c.n_layers * M_COUNT; ++i) {
        free(m->lin[i].packed);
        free(m->lin[i].scales);
    }
    free(m->lin);
    free(m->lm_head.packed);
    free(m->lm_head.scales);
    free(m->embed);
    free(m->kc);
    free(m->vc);
    free(m->cos_t);
    free(m->sin_t);
    free(m->x); free(m->h); free(m->q); free(m->k); free(m->v); free(m->a);
    free(m->ao); free(m->g); free(m->u); free(m->s); free(m->d); free(m->logits);
    free(m);
}

const uint8_t *orc_model_packed(const orc_model *m, uint32_t id) {
    if (id == T_LMHEAD) return m->lm_head.packed;
    if (id < T_LAYER0) return NULL;
    uint32_t l = (id - T_LAYER0) / 8, w = (id - T_LAYER0) % 8;
    if (l >= m->c.n_layers || w >= M_COUNT) return NULL;
    return m->lin[l * M_COUNT + w].packed;
}

const uint8_t *orc_model_scales(const orc_model *m, uint32_t id) {
    if (id == T_LMHEAD) return m->lm_head.scales;
    if (id < T_LAYER0) return NULL;
    uint32_t l = (id - T_LAYER0) / 8, w = (id - T_LAYER0) % 8;
    if (l >= m->c.n_layers || w >= M_COUNT) return NULL;
    return m->lin[l * M_COUNT + w].scales;
}

const uint16_t *orc_model_embed(const orc_model *m) { return m->embed; }

/* Replace model weights (tests of the checkpoint loader): tensor_id as in
 * orc_model_packed, canonical [n][k/2] nibbles + [n][k/32] E8M0 scales. */
void orc_model_set_tensor(orc_model *m, uint32_t tensor_id, const uint8_t *packed, const uint8_t *scales) {
    qmat *q = tensor_id == 1 ? &m->lm_head : &m->lin[((tensor_id - 16) / 8) * M_COUNT + (tensor_id - 16) % 8];
    memcpy(q->packed, packed, (size_t)q->n * q->k / 2);
    memcpy(q->scales, scales, (size_t)q->n * q->k / 32);
}
void orc_model_set_embed(orc_model *m, const uint16_t *embed) {
    memcpy(m->embed, embed, (size_t)m->c.vocab * m->c.dim * 2);
}
/* which: 0..L-1 attention norm of layer which, L..2L-1 FFN norm of layer which-L,
 * 2L the final norm (llama_run/src/main.rs:79-116 weight vector). */
void orc_model_set_norm(orc_model *m, uint32_t which, const float *w) {
    memcpy(m->norms + (size_t)which * m->c.dim, w, sizeof(float) * m->c.dim);
}

static void lin(orc_model *m, const qmat *w, const float *x, float *y) {
    orc_gemv_mxfp4(w->n, w->k, w->packed, w->scales, x, y, m->threads);
}

/* llama_run/src/main.rs:509-535 with bf16 embeddings and a bf16 KV cache: K/V rows
 * are rounded to bf16 when appended and widened when read. */
uint32_t orc_forward(orc_model *m, uint32_t token, uint32_t pos, float *logits) {
    const orc_config *c = &m->c;
    if (pos >= c->max_seq || token >= c->vocab) return UINT32_MAX; /* nothing written */
    uint32_t hd = c->head_dim, half = hd / 2, nkv = c->n_kv_heads, nh = c->n_heads;
    uint32_t kvd = nkv * hd, seq = pos + 1;
    const uint16_t *er = m->embed + (size_t)token * c->dim;
    for (uint32_t i = 0; i < c->dim; ++i) m->x[i] = orc_bf16_to_f32(er[i]);
    float *kf = (float *)malloc(sizeof(float) * (size_t)seq * kvd);
    float *vf = (float *)malloc(sizeof(float) * (size_t)seq * kvd);
    uint32_t cos_base = pos * half;
    for (uint32_t l = 0; l < c->n_layers; ++l) {
        qmat *L = &m->lin[l * M_COUNT];
        orc_rmsnorm(c->dim, c->eps, m->x, m->norms + (size_t)l * c->dim, m->h);
        lin(m, &L[M_Q], m->h, m->q);
        lin(m, &L[M_K], m->h, m->k);
        lin(m, &L[M_V], m->h, m->v);
        orc_rope(nh, hd, cos_base, m->cos_t, m->sin_t, m->q);
        orc_rope(nkv, hd, cos_base, m->cos_t, m->sin_t, m->k);
        uint16_t *kcl = m->kc + (size_t)l * c->max_seq * kvd;
        uint16_t *vcl = m->vc + (size_t)l * c->max_seq * kvd;
        for (uint32_t i = 0; i < kvd; ++i) {
            kcl[(size_t)pos * kvd + i] = orc_f32_to_bf16(m->k[i]);
            vcl[(size_t)pos * kvd + i] = orc_f32_to_bf16(m->v[i]);
        }
        for (size_t i = 0; i < (size_t)seq * kvd; ++i) {
            kf[i] = orc_bf16_to_f32(kcl[i]);
            vf[i] = orc_bf16_to_f32(vcl[i]);
        }
        orc_attn_decode(nh, nkv, hd, seq, m->q, kf, vf, m->a, m->threads);
        lin(m, &L[M_O], m->a, m->ao);
        orc_residual(c->dim, m->ao, m->x);
        orc_rmsnorm(c->dim, c->eps, m->x, m->norms + (size_t)(c->n_layers + l) * c->dim, m->h);
        lin(m, &L[M_GATE], m->h, m->g);
        lin(m, &L[M_UP], m->h, m->u);
        orc_swiglu(c->ffn, m->g, m->u, m->s);
        lin(m, &L[M_DOWN], m->s, m->d);
        orc_residual(c->dim, m->d, m->x);
    }
    orc_rmsnorm(c->dim, c->eps, m->x, m->norms + (size_t)2 * c->n_layers * c->dim, m->h);
    lin(m, &m->lm_head, m->h, m->logits);
    free(kf);
    free(vf);
    if (logits) memcpy(logits, m->logits, sizeof(float) * c->vocab);
    return orc_argmax(c->vocab, m->logits);
}

/* llama_run/src/main.rs:544-570 (EOS and MAXSEQ stops left to the caller). */
void orc_generate(orc_model *m, const uint32_t *prompt, uint32_t n_prompt, uint32_t n_gen,
                  uint32_t *out_ids) {
    uint32_t pos = 0, gen = 0, tok = prompt[0];
    while (gen < n_gen) {
        uint32_t next = orc_forward(m, tok, pos, NULL);
        pos++;
        if (pos < n_prompt) {
            tok = prompt[pos];
        } else {
            out_ids[gen++] = next;
            tok = next;
        }
    }
}
