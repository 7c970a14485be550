"""Generate tests/golden/reference_kats.npz: known answers for the oracle.

The reference (botBehavior/rust-fp4-blackwell) ships no golden files; its tests
generate inputs from xorshift32 seeds and compare against scalar CPU loops.  This
script restates those loops INDEPENDENTLY of oracle.c -- plain Python/numpy with
explicit float32 rounding after every operation, in the reference's order -- so
that the C oracle can be pinned against it.  Sources (paths inside the reference):

  * xorshift32 streams: examples/*/src/main.rs (seeds 0x12345678 fp4_gemv:101,
    0x9e3779b9 llama_rmsnorm:63, 0x13579bdf llama_rope:53, 0xabcd1234
    llama_attn_decode:138, 0xdeadbeef llama_decode:369); Marsaglia's published
    first output 723471715 for state 2463534242.
  * E2M1 table: trackb/FP4_M16N8K64_LAYOUT.md:25-26, fp4_gemv/src/main.rs:130-134.
  * MMA KATs: all-ones -> 64.0 (examples/fp4_mma/src/main.rs:24-31,75;
    trackb/fp4_mma_m16n8k64_reference.cu:7-9,32); patterned A/B
    (trackb/fp4_mapping_test.cu:38-40); power-of-two scales
    (trackb/fp4_scale_test.cu:34-37,112).
  * GEMV / RMSNorm / RoPE / attention CPU loops: fp4_gemv/src/main.rs:109-142,
    llama_rmsnorm/src/main.rs:63-77, llama_rope/src/main.rs:53-84,
    llama_attn_decode/src/main.rs:138-179 (smaller sizes where noted).
  * Quantiser: llama_run/src/main.rs:332-376.

Run:  python tests/golden/make_golden.py   (writes reference_kats.npz next to it)
"""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np

f32 = np.float32
OUT = Path(__file__).resolve().parent / "reference_kats.npz"


def xorshift32(seed, n):
    s = seed & 0xFFFFFFFF
    out = []
    for _ in range(n):
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        out.append(s)
    return out


MAGS = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]


def fp4(c):
    m = f32(MAGS[c & 7])
    return f32(-m) if c & 8 else m


def quant_ref_block(vals):
    """llama_run/src/main.rs:340-364 for one 32-block (f32 arithmetic)."""
    amax = f32(0.0)
    for v in vals:
        amax = max(amax, f32(abs(f32(v))))
    scale = f32(amax / f32(6.0)) if amax > 0 else f32(1.0)
    codes = []
    for v in vals:
        v = f32(f32(v) / scale)
        a = f32(abs(v))
        bc, bd = 0, f32(3.4028235e38)
        for ci, lv in enumerate(MAGS):
            d = f32(abs(f32(a - f32(lv))))
            if d < bd:
                bd, bc = d, ci
        code = bc | (8 if v < 0 else 0)
        codes.append(code)
    return codes, scale


def main():
    g = {}
    seeds = {"gemv": 0x12345678, "rmsnorm": 0x9E3779B9, "rope": 0x13579BDF, "attn": 0xABCD1234,
             "decode": 0xDEADBEEF, "marsaglia": 2463534242}
    for k, s in seeds.items():
        g[f"xs_{k}"] = np.array(xorshift32(s, 8), np.uint32)

    g["e2m1_table"] = np.array([fp4(c) for c in range(16)], np.float32)

    # ---- MMA KATs (D = A(16x64) . B(64x8), per-32-block scales) ----
    A = np.array([[MAGS[(i * 7 + k * 3) % 8] for k in range(64)] for i in range(16)], np.float32)
    B = np.array([[MAGS[(k * 5 + j * 2) % 8] for j in range(8)] for k in range(64)], np.float32)
    D = np.zeros((16, 8), np.float32)
    for i in range(16):
        for j in range(8):
            s = f32(0)
            for k in range(64):
                s = f32(s + f32(A[i, k] * B[k, j]))
            D[i, j] = s
    g["kat_pattern_A"], g["kat_pattern_B"], g["kat_pattern_D"] = A, B, D
    SV = [0.5, 1.0, 2.0, 4.0]
    SFA = np.array([[SV[(i + b) % 4] for b in range(2)] for i in range(16)], np.float32)
    SFB = np.array([[SV[(j + b * 2) % 4] for j in range(8)] for b in range(2)], np.float32)
    DS = np.zeros((16, 8), np.float32)
    for i in range(16):
        for j in range(8):
            s = f32(0)
            for k in range(64):
                s = f32(s + f32(f32(f32(A[i, k] * SFA[i, k // 32]) * B[k, j]) * SFB[k // 32, j]))
            DS[i, j] = s
    g["kat_scale_SFA"], g["kat_scale_SFB"], g["kat_scale_D"] = SFA, SFB, DS
    g["kat_allones_D"] = np.full((16, 8), 64.0, np.float32)

    # ---- GEMV (fp4_gemv/src/main.rs:109-142), N=64, K=256 from the same stream ----
    N, K = 64, 256
    r = xorshift32(0x12345678, N * K + N * K // 32 + K)
    codes = [v & 0xF for v in r[: N * K]]
    scales = [f32(f32(0.5) + f32(f32(v % 8) * f32(0.25))) for v in r[N * K: N * K + N * K // 32]]
    x = [f32(f32(f32(v % 17) - f32(8.0)) * f32(0.1)) for v in r[N * K + N * K // 32:]]
    y = []
    for n in range(N):
        acc = f32(0)
        for k in range(K):
            acc = f32(acc + f32(f32(fp4(codes[n * K + k]) * scales[n * (K // 32) + k // 32]) * x[k]))
        y.append(acc)
    words = np.zeros(N * K // 8, np.uint32)
    for i in range(N * K // 8):
        w = 0
        for p in range(8):
            w |= codes[i * 8 + p] << (p * 4)
        words[i] = w
    g["gemv_words"] = words.reshape(N, K // 8)
    g["gemv_scales"] = np.array(scales, np.float32).reshape(N, K // 32)
    g["gemv_x"] = np.array(x, np.float32)
    g["gemv_y"] = np.array(y, np.float32)

    # ---- RMSNorm (llama_rmsnorm/src/main.rs:60-77), dim 2048 ----
    DIM, EPS = 2048, f32(1e-5)
    r = xorshift32(0x9E3779B9, 2 * DIM)
    xr = [f32(f32(f32(v % 2001) - f32(1000.0)) / f32(500.0)) for v in r[:DIM]]
    wr = [f32(f32(0.5) + f32(f32(v % 1000) / f32(1000.0))) for v in r[DIM:]]
    ss = f32(0)
    for v in xr:
        ss = f32(ss + f32(v * v))
    rms = f32(f32(1.0) / f32(math.sqrt(float(f32(f32(ss / f32(DIM)) + EPS)))))
    g["rms_x"] = np.array(xr, np.float32)
    g["rms_w"] = np.array(wr, np.float32)
    g["rms_y"] = np.array([f32(f32(xr[i] * rms) * wr[i]) for i in range(DIM)], np.float32)

    # ---- RoPE (llama_rope/src/main.rs:47-84): 32 heads x 64, pos 37, theta 5e5 ----
    H, HD = 32, 64
    half = HD // 2
    r = xorshift32(0x13579BDF, H * HD)
    q = [f32(f32(f32(v % 2001) - f32(1000.0)) / f32(500.0)) for v in r]
    cos = [f32(math.cos(37.0 * (1.0 / 500000.0 ** (2.0 * j / HD)))) for j in range(half)]
    sin = [f32(math.sin(37.0 * (1.0 / 500000.0 ** (2.0 * j / HD)))) for j in range(half)]
    out = list(q)
    for h in range(H):
        b = h * HD
        for j in range(half):
            x0, x1 = q[b + j], q[b + j + half]
            out[b + j] = f32(f32(x0 * cos[j]) - f32(x1 * sin[j]))
            out[b + j + half] = f32(f32(x1 * cos[j]) + f32(x0 * sin[j]))
    g["rope_q"] = np.array(q, np.float32)
    g["rope_cos"] = np.array(cos, np.float32)
    g["rope_sin"] = np.array(sin, np.float32)
    g["rope_out"] = np.array(out, np.float32)

    # ---- attention (llama_attn_decode/src/main.rs:133-179), 32q/8kv, hd 64, seq 64 ----
    NH, NKV, SEQ = 32, 8, 64
    r = xorshift32(0xABCD1234, NH * HD + 2 * SEQ * NKV * HD)
    vals = [f32(f32(f32(v % 2001) - f32(1000.0)) / f32(700.0)) for v in r]
    qa = vals[: NH * HD]
    kc = vals[NH * HD: NH * HD + SEQ * NKV * HD]
    vc = vals[NH * HD + SEQ * NKV * HD:]
    scale = f32(f32(1.0) / f32(math.sqrt(64.0)))
    oref = []
    grp = NH // NKV
    for h in range(NH):
        kvh = h // grp
        sc = []
        m = f32(-3.4028235e38)
        for t in range(SEQ):
            d = f32(0)
            for i in range(HD):
                d = f32(d + f32(qa[h * HD + i] * kc[(t * NKV + kvh) * HD + i]))
            s = f32(d * scale)
            sc.append(s)
            m = max(m, s)
        lsum = f32(0)
        for t in range(SEQ):
            sc[t] = f32(math.exp(float(f32(sc[t] - m))))
            lsum = f32(lsum + sc[t])
        for i in range(HD):
            acc = f32(0)
            for t in range(SEQ):
                acc = f32(acc + f32(sc[t] * vc[(t * NKV + kvh) * HD + i]))
            oref.append(f32(acc / lsum))
    g["attn_q"] = np.array(qa, np.float32)
    g["attn_k"] = np.array(kc, np.float32)
    g["attn_v"] = np.array(vc, np.float32)
    g["attn_out"] = np.array(oref, np.float32)

    # ---- quantiser (llama_run/src/main.rs:334-376) on hand-picked blocks ----
    tie = [0.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.75, -0.2, -1e-9, 0.3, 0.8, 2.2, 4.9,
           -6.0, -5.0, -3.5, -2.5, -1.75, -1.25, -0.25, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 5.5, 0.1, -0.0]
    rnd = [f32(f32(f32(v % 2001) - f32(1000.0)) / f32(333.0)) for v in xorshift32(0xDEADBEEF, 32)]
    zero = [0.0] * 32
    blocks = [tie, rnd, zero]
    qc, qs = [], []
    for blk in blocks:
        c, s = quant_ref_block([f32(v) for v in blk])
        qc.append(c)
        qs.append(s)
    g["quant_in"] = np.array(blocks, np.float32)
    g["quant_codes"] = np.array(qc, np.uint8)
    g["quant_scales"] = np.array(qs, np.float32)

    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
