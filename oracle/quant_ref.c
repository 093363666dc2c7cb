/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the weight-only quantized
 * decode GEMV.  Nothing in the product (sonata_b200/) links or calls this file;
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do, and
 * only as the checker.
 *
 * Plain-C restatement of the reference's weight quantisation so that the
 * int8 / e4m3 codes and per-row fp32 scales can be compared bit for bit.
 *
 *   int8  : scripts/fake_quant.py:16-42 (fake_quantize_weights)
 *           amax  = max|w| over the (row, group)        (:37)
 *           amax  = max(amax, 1e-8)                      (:37, clamp_min)
 *           scale = amax / qmax     (fp32)               (:38)
 *           q     = round_half_even(w / scale), clamped to [-qmax, qmax] (:40)
 *           wdq   = q * scale (fp32), cast back to w.dtype (:41-42)
 *   e4m3  : no reference code exists; BASELINE config 3 defines it as
 *           scale = max|row| / 448, q = e4m3(w / scale) with torch's
 *           float -> float8_e4m3fn conversion (round to nearest even, values
 *           that round past 448 become NaN), dequant = float(q) * scale.
 *           The same 1e-8 dead-row clamp as the int8 path is applied.
 *
 * All arithmetic is IEEE fp32 (no fast-math), matching torch's CPU kernels,
 * which perform exactly one correctly rounded fp32 division per element.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bits_to_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float oracle_bf16_to_f32(uint16_t h) { return bits_to_f32((uint32_t)h << 16); }

/* fp32 -> bf16, round to nearest even; NaN stays a quiet NaN (torch's rule). */
uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u = f32_to_bits(f);
    if (isnan(f)) return (uint16_t)((u >> 16) | 0x0040u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return (uint16_t)(u >> 16);
}

/* e4m3 (fn variant: no infinities, 0x7F/0xFF are NaN) -> fp32, exact. */
float oracle_e4m3_to_f32(uint8_t b) {
    int sign = (b >> 7) & 1;
    int e = (b >> 3) & 0xF;
    int m = b & 7;
    float v;
    if (e == 0xF && m == 7) return sign ? -NAN : NAN;
    if (e == 0) v = ldexpf((float)m, -9);              /* subnormal: m * 2^-9 */
    else v = ldexpf((float)(8 + m), e - 7 - 3);         /* (1 + m/8) * 2^(e-7) */
    return sign ? -v : v;
}

/* fp32 -> e4m3, round to nearest even; anything that rounds beyond 448 is NaN. */
uint8_t oracle_f32_to_e4m3(float f) {
    uint8_t sign = signbit(f) ? 0x80 : 0x00;
    if (isnan(f)) return (uint8_t)(sign | 0x7F);
    float a = fabsf(f);
    if (a == 0.0f) return sign;
    if (a < ldexpf(1.0f, -6)) {
        /* subnormal range: units of 2^-9; m == 8 encodes the smallest normal. */
        float m = nearbyintf(ldexpf(a, 9));
        return (uint8_t)(sign | (uint8_t)m);
    }
    int e2;
    frexpf(a, &e2);               /* a = fr * 2^e2, fr in [0.5, 1) */
    int e = e2 - 1;               /* a in [2^e, 2^(e+1)) */
    if (e > 8) return (uint8_t)(sign | 0x7F);
    float m = nearbyintf(ldexpf(a, 3 - e));   /* in [8, 16] */
    int mi = (int)m;
    if (mi == 16) { mi = 8; e += 1; }
    if (e > 8) return (uint8_t)(sign | 0x7F);
    int code = ((e + 7) << 3) | (mi - 8);
    if (code >= 0x7F) return (uint8_t)(sign | 0x7F);
    return (uint8_t)(sign | code);
}

/*
 * Symmetric signed integer quantisation of a bf16 [N, K] row-major matrix
 * (row stride ldw elements), one scale per (row, group).  bits in [2, 8].
 * q is [N, K] int8 (row stride K), scale is [N, K / group] fp32.
 */
int oracle_quant_int_rows(const uint16_t *w, long ldw, int N, int K, int group,
                          int bits, int8_t *q, float *scale) {
    if (group <= 0) group = K;
    if (K % group != 0 || bits < 2 || bits > 8) return -1;
    const float qmax = (float)((1 << (bits - 1)) - 1);
    const int G = K / group;
    for (int n = 0; n < N; ++n) {
        for (int g = 0; g < G; ++g) {
            const uint16_t *row = w + (long)n * ldw + (long)g * group;
            float amax = 0.0f;
            for (int k = 0; k < group; ++k) {
                float v = fabsf(oracle_bf16_to_f32(row[k]));
                if (v > amax || isnan(v)) amax = v;
            }
            if (amax < 1e-8f) amax = 1e-8f;
            float s = amax / qmax;
            scale[(long)n * G + g] = s;
            for (int k = 0; k < group; ++k) {
                float r = nearbyintf(oracle_bf16_to_f32(row[k]) / s);
                if (r > qmax) r = qmax;
                if (r < -qmax) r = -qmax;
                q[(long)n * K + (long)g * group + k] = (int8_t)r;
            }
        }
    }
    return 0;
}

/* Per-row e4m3 quantisation: scale = max(max|row|, 1e-8) / 448. */
int oracle_quant_e4m3_rows(const uint16_t *w, long ldw, int N, int K,
                           uint8_t *q, float *scale) {
    for (int n = 0; n < N; ++n) {
        const uint16_t *row = w + (long)n * ldw;
        float amax = 0.0f;
        for (int k = 0; k < K; ++k) {
            float v = fabsf(oracle_bf16_to_f32(row[k]));
            if (v > amax) amax = v;
        }
        if (amax < 1e-8f) amax = 1e-8f;
        float s = amax / 448.0f;
        scale[n] = s;
        for (int k = 0; k < K; ++k)
            q[(long)n * K + k] = oracle_f32_to_e4m3(oracle_bf16_to_f32(row[k]) / s);
    }
    return 0;
}

/*
 * Dequantise-then-matmul in double precision:
 *   y[m, n] = sum_k x[m, k] * (decode(q[n, k]) * scale[n])
 * which is the "dequantize to fp32 then matmul" oracle of BASELINE config 3
 * (the dequantised weight q*scale is formed in fp32 first, as fake_quant.py:41
 * does, then the dot product is accumulated in double).
 * kind: 0 = int8 codes, 1 = e4m3 codes.  x is bf16 [M, K].
 */
void oracle_dequant_gemv(const void *q, const float *scale, const uint16_t *x,
                         int M, int N, int K, int kind, double *y) {
    for (int m = 0; m < M; ++m) {
        for (int n = 0; n < N; ++n) {
            double acc = 0.0;
            for (int k = 0; k < K; ++k) {
                float c = kind == 0 ? (float)((const int8_t *)q)[(long)n * K + k]
                                    : oracle_e4m3_to_f32(((const uint8_t *)q)[(long)n * K + k]);
                float wdq = c * scale[n];
                acc += (double)wdq * (double)oracle_bf16_to_f32(x[(long)m * K + k]);
            }
            y[(long)m * N + n] = acc;
        }
    }
}

/* bf16 GEMV in double: y[m, n] = sum_k x[m, k] * W[n, k] (F.linear, fp32 truth). */
void oracle_gemv_bf16(const uint16_t *W, long ldw, const uint16_t *x, int M, int N,
                      int K, double *y) {
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            double acc = 0.0;
            for (int k = 0; k < K; ++k)
                acc += (double)oracle_bf16_to_f32(W[(long)n * ldw + k]) *
                       (double)oracle_bf16_to_f32(x[(long)m * K + k]);
            y[(long)m * N + n] = acc;
        }
}
