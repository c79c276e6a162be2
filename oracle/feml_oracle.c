/*
 * feml_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the feml reference algorithms on the mul_mat /
 * mul_mat_id path, used as the checker by tests/, by __graft_entry__.smoke()
 * and by bench.py's CPU-baseline leg. Nothing in the product links or calls
 * this file.
 *
 * Build: gcc -O2 -ffp-contract=off -fno-fast-math -fPIC -shared -pthread
 * (oracle/build_oracle.py). Contraction is off so that `acc += x * y` rounds
 * the product and the sum separately, exactly as Rust does for
 * feml-cpu/src/ops/mul_mat.rs:46-48 (Rust never fuses a*b+c implicitly).
 *
 * What each function restates:
 *  - oracle_mul_mat_f32: feml-cpu/src/ops/mul_mat.rs:14-58 (loop order m, n, k;
 *    sequential f32 accumulation; ggml byte strides).
 *  - quant block formats Q8_0 / Q4_0 / Q4_K: the reference carries only their
 *    sizes (feml-core/src/dtype.rs:60,64,68). The layouts and the Q8_0/Q4_0
 *    quantizers below restate the public ggml/GGUF block-format description
 *    (block_q8_0 = {f16 d; i8 qs[32]}, block_q4_0 = {f16 d; u8 qs[16]},
 *    block_q4_K = {f16 d; f16 dmin; u8 scales[12]; u8 qs[128]}); the Q4_K
 *    quantizer is this project's own deterministic scheme (ggml's iterative
 *    search is not reproduced), so Q4_K quantizer bytes are parity-unpinned.
 *  - Q5_K / Q6_K (block_q5_K = {f16 d; f16 dmin; u8 scales[12]; u8 qh[32];
 *    u8 qs[128]}, block_q6_K = {u8 ql[128]; u8 qh[64]; i8 scales[16];
 *    f16 d}): dequantizers restate the public layouts; the quantizers are
 *    this project's deterministic single-pass schemes (parity-unpinned, like
 *    Q4_K's). The dequantizers of all K-quants are pinned to llama.cpp's
 *    gguf-py implementation in tests.
 *  - per-block int32 dot products and MoE routing: the integer work the
 *    B200 kernels must reproduce bit-for-bit.
 *  - planner/layout golden values are checked in tests against the product
 *    host library directly (feml-core/src/planner.rs:284-398,
 *    feml-core/src/layout.rs:68-113).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QK8_0 32
#define QK4_0 32
#define QK_K 256
#define Q8_0_BYTES 34
#define Q4_0_BYTES 18
#define Q4_K_BYTES 144
#define Q5_K_BYTES 176
#define Q6_K_BYTES 210

/* ------------------------------------------------------------------------ */
/* IEEE binary16 <-> binary32, round-to-nearest-even (bit-level, portable).  */
/* ------------------------------------------------------------------------ */
uint16_t oracle_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u); /* overflow -> inf */
    if (e <= 0) {                                    /* subnormal / zero */
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t half = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (half & 1u))) half++;
        return (uint16_t)(sign | half);
    }
    uint32_t half = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half++; /* carry may bump exp: still correct */
    return (uint16_t)half;
}

float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else { /* normalise subnormal */
            int e = -1;
            do { e++; man <<= 1; } while (!(man & 0x400u));
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static inline uint16_t rd_u16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline void wr_u16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)(v & 0xff); p[1] = (uint8_t)(v >> 8); }

/* ------------------------------------------------------------------------ */
/* Q8_0                                                                      */
/* ------------------------------------------------------------------------ */
/* quantize_row_q8_0: d = amax/127 (f32), stored as f16 (RNE);
 * q = roundf(x * (1/d)) (half away from zero), all-zero when d == 0. */
void oracle_quantize_row_q8_0(const float *x, uint8_t *y, int64_t k) {
    const int64_t nb = k / QK8_0;
    for (int64_t i = 0; i < nb; i++) {
        const float *xb = x + i * QK8_0;
        uint8_t *yb = y + i * Q8_0_BYTES;
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; j++) {
            float v = fabsf(xb[j]);
            amax = amax > v ? amax : v;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        wr_u16(yb, oracle_f32_to_f16(d));
        for (int j = 0; j < QK8_0; j++) {
            const float v = xb[j] * id;
            yb[2 + j] = (uint8_t)(int8_t)roundf(v);
        }
    }
}

void oracle_dequantize_row_q8_0(const uint8_t *y, float *x, int64_t k) {
    const int64_t nb = k / QK8_0;
    for (int64_t i = 0; i < nb; i++) {
        const uint8_t *yb = y + i * Q8_0_BYTES;
        const float d = oracle_f16_to_f32(rd_u16(yb));
        for (int j = 0; j < QK8_0; j++) x[i * QK8_0 + j] = (float)(int8_t)yb[2 + j] * d;
    }
}

/* ------------------------------------------------------------------------ */
/* Q4_0                                                                      */
/* ------------------------------------------------------------------------ */
/* d = max / -8 where max is the signed value of largest magnitude (first
 * occurrence wins); nibble = min(15, trunc(x * (1/d) + 8.5)); element j in the
 * low nibble of byte j, element j+16 in its high nibble. */
void oracle_quantize_row_q4_0(const float *x, uint8_t *y, int64_t k) {
    const int64_t nb = k / QK4_0;
    for (int64_t i = 0; i < nb; i++) {
        const float *xb = x + i * QK4_0;
        uint8_t *yb = y + i * Q4_0_BYTES;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < QK4_0; j++) {
            const float v = xb[j];
            if (amax < fabsf(v)) { amax = fabsf(v); max = v; }
        }
        const float d = max / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        wr_u16(yb, oracle_f32_to_f16(d));
        for (int j = 0; j < QK4_0 / 2; j++) {
            const float x0 = xb[j] * id;
            const float x1 = xb[j + QK4_0 / 2] * id;
            int q0 = (int)(int8_t)(x0 + 8.5f);
            int q1 = (int)(int8_t)(x1 + 8.5f);
            if (q0 > 15) q0 = 15;
            if (q1 > 15) q1 = 15;
            yb[2 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

void oracle_dequantize_row_q4_0(const uint8_t *y, float *x, int64_t k) {
    const int64_t nb = k / QK4_0;
    for (int64_t i = 0; i < nb; i++) {
        const uint8_t *yb = y + i * Q4_0_BYTES;
        const float d = oracle_f16_to_f32(rd_u16(yb));
        for (int j = 0; j < QK4_0 / 2; j++) {
            const int x0 = (yb[2 + j] & 0x0f) - 8;
            const int x1 = (yb[2 + j] >> 4) - 8;
            x[i * QK4_0 + j] = (float)x0 * d;
            x[i * QK4_0 + j + QK4_0 / 2] = (float)x1 * d;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Q4_K                                                                      */
/* ------------------------------------------------------------------------ */
/* 6-bit (scale, min) pair j of a super-block from its 12 packed bytes. */
void oracle_q4k_scale_min(int j, const uint8_t *q, int *sc, int *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* Deterministic single-pass Q4_K quantizer (this project's scheme):
 *   per sub-block j: lo = min(0, min x), hi = max(0, max x),
 *                    scale_j = (hi - lo) / 15, minv_j = -lo
 *   d = f16(max_j scale_j / 63), dmin = f16(max_j minv_j / 63)
 *   sc_j = min(63, roundf(scale_j / d)), m_j = min(63, roundf(minv_j / dmin))
 *   q = clamp(roundf((x + dmin*m_j) / (d*sc_j)), 0, 15)
 * Every step is a correctly rounded IEEE operation, so the device quantizer
 * reproduces it bit for bit. */
void oracle_quantize_row_q4_k(const float *x, uint8_t *y, int64_t k) {
    const int64_t nb = k / QK_K;
    for (int64_t i = 0; i < nb; i++) {
        const float *xb = x + i * QK_K;
        uint8_t *yb = y + i * Q4_K_BYTES;
        float scale[8], minv[8];
        float max_scale = 0.0f, max_min = 0.0f;
        for (int j = 0; j < 8; j++) {
            float lo = 0.0f, hi = 0.0f;
            for (int l = 0; l < 32; l++) {
                const float v = xb[32 * j + l];
                lo = v < lo ? v : lo;
                hi = v > hi ? v : hi;
            }
            scale[j] = (hi - lo) / 15.0f;
            minv[j] = -lo;
            max_scale = scale[j] > max_scale ? scale[j] : max_scale;
            max_min = minv[j] > max_min ? minv[j] : max_min;
        }
        const uint16_t dh = oracle_f32_to_f16(max_scale / 63.0f);
        const uint16_t mh = oracle_f32_to_f16(max_min / 63.0f);
        const float df = oracle_f16_to_f32(dh);
        const float mf = oracle_f16_to_f32(mh);
        int sc[8], mm[8];
        for (int j = 0; j < 8; j++) {
            int s = df > 0.0f ? (int)roundf(scale[j] / df) : 0;
            int m = mf > 0.0f ? (int)roundf(minv[j] / mf) : 0;
            sc[j] = s > 63 ? 63 : s;
            mm[j] = m > 63 ? 63 : m;
        }
        wr_u16(yb, dh);
        wr_u16(yb + 2, mh);
        uint8_t *scales = yb + 4;
        memset(scales, 0, 12);
        for (int j = 0; j < 8; j++) {
            if (j < 4) {
                scales[j] = (uint8_t)sc[j];
                scales[j + 4] = (uint8_t)mm[j];
            } else {
                scales[j + 4] = (uint8_t)((sc[j] & 0x0f) | ((mm[j] & 0x0f) << 4));
                scales[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
                scales[j] |= (uint8_t)((mm[j] >> 4) << 6);
            }
        }
        uint8_t q[QK_K];
        for (int j = 0; j < 8; j++) {
            const float ds = df * (float)sc[j];
            const float dm = mf * (float)mm[j];
            for (int l = 0; l < 32; l++) {
                int v = 0;
                if (ds > 0.0f) {
                    v = (int)roundf((xb[32 * j + l] + dm) / ds);
                    v = v < 0 ? 0 : (v > 15 ? 15 : v);
                }
                q[32 * j + l] = (uint8_t)v;
            }
        }
        uint8_t *qs = yb + 16;
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 32; l++)
                qs[32 * g + l] = (uint8_t)(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
    }
}

/* Value = d*sc*q - dmin*m, evaluated as (d*sc)*q - (dmin*m) in f32. */
void oracle_dequantize_row_q4_k(const uint8_t *y, float *x, int64_t k) {
    const int64_t nb = k / QK_K;
    for (int64_t i = 0; i < nb; i++) {
        const uint8_t *yb = y + i * Q4_K_BYTES;
        const float d = oracle_f16_to_f32(rd_u16(yb));
        const float dmin = oracle_f16_to_f32(rd_u16(yb + 2));
        const uint8_t *scales = yb + 4;
        const uint8_t *qs = yb + 16;
        float *out = x + i * QK_K;
        for (int g = 0; g < 4; g++) {
            int sc, m;
            oracle_q4k_scale_min(2 * g, scales, &sc, &m);
            const float d1 = d * (float)sc, m1 = dmin * (float)m;
            oracle_q4k_scale_min(2 * g + 1, scales, &sc, &m);
            const float d2 = d * (float)sc, m2 = dmin * (float)m;
            for (int l = 0; l < 32; l++) out[64 * g + l] = d1 * (float)(qs[32 * g + l] & 0x0f) - m1;
            for (int l = 0; l < 32; l++) out[64 * g + 32 + l] = d2 * (float)(qs[32 * g + l] >> 4) - m2;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Q5_K and Q6_K                                                             */
/* ------------------------------------------------------------------------ */
/* Q5_K quantizer (this project's scheme): the Q4_K scheme with 31 levels;
 * the 5-bit value's low nibble goes to qs (as in Q4_K), its bit 4 to qh:
 * element l of sub-block j sets bit j of qh[l]. */
void oracle_quantize_row_q5_k(const float *x, uint8_t *y, int64_t k) {
    const int64_t nb = k / QK_K;
    for (int64_t i = 0; i < nb; i++) {
        const float *xb = x + i * QK_K;
        uint8_t *yb = y + i * Q5_K_BYTES;
        float scale[8], minv[8];
        float max_scale = 0.0f, max_min = 0.0f;
        for (int j = 0; j < 8; j++) {
            float lo = 0.0f, hi = 0.0f;
            for (int l = 0; l < 32; l++) {
                const float v = xb[32 * j + l];
                lo = v < lo ? v : lo;
                hi = v > hi ? v : hi;
            }
            scale[j] = (hi - lo) / 31.0f;
            minv[j] = -lo;
            max_scale = scale[j] > max_scale ? scale[j] : max_scale;
            max_min = minv[j] > max_min ? minv[j] : max_min;
        }
        const uint16_t dh = oracle_f32_to_f16(max_scale / 63.0f);
        const uint16_t mh = oracle_f32_to_f16(max_min / 63.0f);
        const float df = oracle_f16_to_f32(dh);
        const float mf = oracle_f16_to_f32(mh);
        int sc[8], mm[8];
        for (int j = 0; j < 8; j++) {
            int s = df > 0.0f ? (int)roundf(scale[j] / df) : 0;
            int m = mf > 0.0f ? (int)roundf(minv[j] / mf) : 0;
            sc[j] = s > 63 ? 63 : s;
            mm[j] = m > 63 ? 63 : m;
        }
        wr_u16(yb, dh);
        wr_u16(yb + 2, mh);
        uint8_t *scales = yb + 4;
        memset(scales, 0, 12);
        for (int j = 0; j < 8; j++) {
            if (j < 4) {
                scales[j] = (uint8_t)sc[j];
                scales[j + 4] = (uint8_t)mm[j];
            } else {
                scales[j + 4] = (uint8_t)((sc[j] & 0x0f) | ((mm[j] & 0x0f) << 4));
                scales[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
                scales[j] |= (uint8_t)((mm[j] >> 4) << 6);
            }
        }
        uint8_t q[QK_K];
        for (int j = 0; j < 8; j++) {
            const float ds = df * (float)sc[j];
            const float dm = mf * (float)mm[j];
            for (int l = 0; l < 32; l++) {
                int v = 0;
                if (ds > 0.0f) {
                    v = (int)roundf((xb[32 * j + l] + dm) / ds);
                    v = v < 0 ? 0 : (v > 31 ? 31 : v);
                }
                q[32 * j + l] = (uint8_t)v;
            }
        }
        uint8_t *qh = yb + 16, *qs = yb + 48;
        memset(qh, 0, 32);
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 32; l++) {
                const uint8_t a = q[64 * g + l], b = q[64 * g + 32 + l];
                qs[32 * g + l] = (uint8_t)((a & 0x0f) | ((b & 0x0f) << 4));
                qh[l] |= (uint8_t)(((a >> 4) << (2 * g)) | ((b >> 4) << (2 * g + 1)));
            }
    }
}

/* Value = (d*sc)*q - (dmin*m), q = low nibble + 16 * high bit. */
void oracle_dequantize_row_q5_k(const uint8_t *y, float *x, int64_t k) {
    const int64_t nb = k / QK_K;
    for (int64_t i = 0; i < nb; i++) {
        const uint8_t *yb = y + i * Q5_K_BYTES;
        const float d = oracle_f16_to_f32(rd_u16(yb));
        const float dmin = oracle_f16_to_f32(rd_u16(yb + 2));
        const uint8_t *scales = yb + 4, *qh = yb + 16, *qs = yb + 48;
        float *out = x + i * QK_K;
        for (int g = 0; g < 4; g++) {
            int sc, m;
            oracle_q4k_scale_min(2 * g, scales, &sc, &m);
            const float d1 = d * (float)sc, m1 = dmin * (float)m;
            oracle_q4k_scale_min(2 * g + 1, scales, &sc, &m);
            const float d2 = d * (float)sc, m2 = dmin * (float)m;
            for (int l = 0; l < 32; l++) {
                const int q = (qs[32 * g + l] & 0x0f) + (((qh[l] >> (2 * g)) & 1) << 4);
                out[64 * g + l] = d1 * (float)q - m1;
            }
            for (int l = 0; l < 32; l++) {
                const int q = (qs[32 * g + l] >> 4) + (((qh[l] >> (2 * g + 1)) & 1) << 4);
                out[64 * g + 32 + l] = d2 * (float)q - m2;
            }
        }
    }
}

/* Element e (0..255) of a Q6_K super-block: half h = e / 128, within it
 * quarter t = (e % 128) / 32 and lane l = e % 32; its low 4 bits are the low
 * (t < 2) or high (t >= 2) nibble of ql[64h + 32(t % 2) + l], its top 2 bits
 * are bits 2t..2t+1 of qh[32h + l]; its scale is scales[8h + 2t + l / 16]. */
static int q6k_index(int e, int *ql_byte, int *ql_hi, int *qh_byte, int *qh_shift, int *sc_index) {
    const int h = e / 128, t = (e % 128) / 32, l = e % 32;
    *ql_byte = 64 * h + 32 * (t % 2) + l;
    *ql_hi = t >= 2;
    *qh_byte = 32 * h + l;
    *qh_shift = 2 * t;
    *sc_index = 8 * h + 2 * t + l / 16;
    return 0;
}

/* Q6_K quantizer (this project's scheme): per 16-element group g,
 * scale_g = amax_g / 31; d = f16(max_g scale_g / 127);
 * sc_g = min(127, roundf(scale_g / d)); q = clamp(roundf(x / (d*sc_g)), -32, 31)
 * stored as q + 32. */
void oracle_quantize_row_q6_k(const float *x, uint8_t *y, int64_t k) {
    const int64_t nb = k / QK_K;
    for (int64_t i = 0; i < nb; i++) {
        const float *xb = x + i * QK_K;
        uint8_t *yb = y + i * Q6_K_BYTES;
        float scale[16], max_scale = 0.0f;
        for (int g = 0; g < 16; g++) {
            float amax = 0.0f;
            for (int l = 0; l < 16; l++) {
                const float a = fabsf(xb[16 * g + l]);
                amax = a > amax ? a : amax;
            }
            scale[g] = amax / 31.0f;
            max_scale = scale[g] > max_scale ? scale[g] : max_scale;
        }
        const uint16_t dh = oracle_f32_to_f16(max_scale / 127.0f);
        const float df = oracle_f16_to_f32(dh);
        memset(yb, 0, Q6_K_BYTES);
        int8_t *scales = (int8_t *)(yb + 192);
        for (int g = 0; g < 16; g++) {
            int s = df > 0.0f ? (int)roundf(scale[g] / df) : 0;
            scales[g] = (int8_t)(s > 127 ? 127 : s);
        }
        for (int e = 0; e < QK_K; e++) {
            int qb, qhi, hb, hs, si;
            q6k_index(e, &qb, &qhi, &hb, &hs, &si);
            const float ds = df * (float)scales[si];
            int v = 0;
            if (ds > 0.0f) {
                v = (int)roundf(xb[e] / ds);
                v = v < -32 ? -32 : (v > 31 ? 31 : v);
            }
            const int u = v + 32;
            yb[qb] |= (uint8_t)((u & 0x0f) << (qhi ? 4 : 0));
            yb[128 + hb] |= (uint8_t)((u >> 4) << hs);
        }
        wr_u16(yb + 208, dh);
    }
}

/* Value = (d*sc)*(q - 32). */
void oracle_dequantize_row_q6_k(const uint8_t *y, float *x, int64_t k) {
    const int64_t nb = k / QK_K;
    for (int64_t i = 0; i < nb; i++) {
        const uint8_t *yb = y + i * Q6_K_BYTES;
        const float d = oracle_f16_to_f32(rd_u16(yb + 208));
        const int8_t *scales = (const int8_t *)(yb + 192);
        for (int e = 0; e < QK_K; e++) {
            int qb, qhi, hb, hs, si;
            q6k_index(e, &qb, &qhi, &hb, &hs, &si);
            const int lo = qhi ? (yb[qb] >> 4) : (yb[qb] & 0x0f);
            const int q = (lo | (((yb[128 + hb] >> hs) & 3) << 4)) - 32;
            x[i * QK_K + e] = (d * (float)scales[si]) * (float)q;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Row-wise helpers over a [rows, k] matrix (ggml layout: row r at r*row_bytes) */
/* ------------------------------------------------------------------------ */
/* dtype codes follow feml-core/src/dtype.rs:14-35 discriminants. */
#define DT_F32 5
#define DT_Q4_0 7
#define DT_Q8_0 11
#define DT_Q4_K 15
#define DT_Q5_K 16
#define DT_Q6_K 17

int64_t oracle_row_bytes(int dtype, int64_t k) {
    switch (dtype) {
    case DT_F32: return 4 * k;
    case DT_Q8_0: return (k / 32) * Q8_0_BYTES;
    case DT_Q4_0: return (k / 32) * Q4_0_BYTES;
    case DT_Q4_K: return (k / 256) * Q4_K_BYTES;
    case DT_Q5_K: return (k / 256) * Q5_K_BYTES;
    case DT_Q6_K: return (k / 256) * Q6_K_BYTES;
    default: return -1;
    }
}

int oracle_quantize_rows(int dtype, const float *x, uint8_t *y, int64_t rows, int64_t k) {
    const int64_t rb = oracle_row_bytes(dtype, k);
    if (rb < 0) return -1;
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * k;
        uint8_t *yr = y + r * rb;
        switch (dtype) {
        case DT_F32: memcpy(yr, xr, (size_t)rb); break;
        case DT_Q8_0: oracle_quantize_row_q8_0(xr, yr, k); break;
        case DT_Q4_0: oracle_quantize_row_q4_0(xr, yr, k); break;
        case DT_Q4_K: oracle_quantize_row_q4_k(xr, yr, k); break;
        case DT_Q5_K: oracle_quantize_row_q5_k(xr, yr, k); break;
        case DT_Q6_K: oracle_quantize_row_q6_k(xr, yr, k); break;
        }
    }
    return 0;
}

int oracle_dequantize_rows(int dtype, const uint8_t *y, float *x, int64_t rows, int64_t k) {
    const int64_t rb = oracle_row_bytes(dtype, k);
    if (rb < 0) return -1;
    for (int64_t r = 0; r < rows; r++) {
        const uint8_t *yr = y + r * rb;
        float *xr = x + r * k;
        switch (dtype) {
        case DT_F32: memcpy(xr, yr, (size_t)rb); break;
        case DT_Q8_0: oracle_dequantize_row_q8_0(yr, xr, k); break;
        case DT_Q4_0: oracle_dequantize_row_q4_0(yr, xr, k); break;
        case DT_Q4_K: oracle_dequantize_row_q4_k(yr, xr, k); break;
        case DT_Q5_K: oracle_dequantize_row_q5_k(yr, xr, k); break;
        case DT_Q6_K: oracle_dequantize_row_q6_k(yr, xr, k); break;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* F32 mul_mat (feml-cpu/src/ops/mul_mat.rs:36-57)                           */
/* ------------------------------------------------------------------------ */
/* dst[m*c_nb0 + n*c_nb1] = sum_k a[k*4 + m*a_nb1] * b[k*4 + n*b_nb1], with a
 * sequential f32 accumulator. Threads split the m range; every output is
 * computed by the same sequential k loop, so the result does not depend on
 * the thread count. */
typedef struct {
    const uint8_t *a; const uint8_t *b; uint8_t *c;
    int64_t K, M, N, a_nb1, b_nb1, c_nb1;
    int64_t m0, m1;
} mm_job;

static void *mm_worker(void *arg) {
    const mm_job *j = (const mm_job *)arg;
    for (int64_t mm = j->m0; mm < j->m1; mm++) {
        const float *ar = (const float *)(j->a + mm * j->a_nb1);
        for (int64_t nn = 0; nn < j->N; nn++) {
            const float *br = (const float *)(j->b + nn * j->b_nb1);
            float acc = 0.0f;
            for (int64_t kk = 0; kk < j->K; kk++) {
                acc += ar[kk] * br[kk];
            }
            *(float *)(j->c + mm * 4 + nn * j->c_nb1) = acc;
        }
    }
    return NULL;
}

void oracle_mul_mat_f32(const void *a, const void *b, void *c, int64_t K, int64_t M, int64_t N,
                        int64_t a_nb1, int64_t b_nb1, int64_t c_nb1, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if ((int64_t)nthreads > M) nthreads = (int)(M > 0 ? M : 1);
    pthread_t th[256];
    mm_job jobs[256];
    for (int t = 0; t < nthreads; t++) {
        jobs[t] = (mm_job){(const uint8_t *)a, (const uint8_t *)b, (uint8_t *)c, K, M, N,
                           a_nb1, b_nb1, c_nb1, M * t / nthreads, M * (t + 1) / nthreads};
    }
    if (nthreads == 1) {
        mm_worker(&jobs[0]);
        return;
    }
    for (int t = 0; t < nthreads; t++) pthread_create(&th[t], NULL, mm_worker, &jobs[t]);
    for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* Per-block int32 dot products against Q8_0 activations                     */
/* ------------------------------------------------------------------------ */
/* out[(r*N + n)*nblk + b] = sum over the 32 elements of 32-block b of
 * (weight integer) * (activation q8 integer), for weight row r and activation
 * column n. Weight integers: Q8_0 -> q; Q4_0 -> nibble - 8; Q4_K -> nibble
 * (0..15; the min term is carried by the activation block sum below).
 * xsum (optional) receives sum of activation q8 integers per (n, b). */
int oracle_block_dots(int dtype, const uint8_t *w, const uint8_t *xq, int32_t *out, int32_t *xsum,
                      int64_t rows, int64_t K, int64_t N) {
    const int64_t nblk = K / 32;
    const int64_t rb = oracle_row_bytes(dtype, K);
    const int64_t xb = oracle_row_bytes(DT_Q8_0, K);
    if (rb < 0 || dtype == DT_F32) return -1;
    for (int64_t n = 0; n < N; n++) {
        const uint8_t *xr = xq + n * xb;
        if (xsum) {
            for (int64_t b = 0; b < nblk; b++) {
                int32_t s = 0;
                for (int l = 0; l < 32; l++) s += (int8_t)xr[b * Q8_0_BYTES + 2 + l];
                xsum[n * nblk + b] = s;
            }
        }
        for (int64_t r = 0; r < rows; r++) {
            const uint8_t *wr = w + r * rb;
            for (int64_t b = 0; b < nblk; b++) {
                const int8_t *xs = (const int8_t *)(xr + b * Q8_0_BYTES + 2);
                int32_t s = 0;
                for (int l = 0; l < 32; l++) {
                    int wi = 0;
                    if (dtype == DT_Q8_0) {
                        wi = (int8_t)wr[b * Q8_0_BYTES + 2 + l];
                    } else if (dtype == DT_Q4_0) {
                        const uint8_t byte = wr[b * Q4_0_BYTES + 2 + (l & 15)];
                        wi = (l < 16 ? (byte & 0x0f) : (byte >> 4)) - 8;
                    } else { /* Q4_K: super-block b/8, sub-block j = b%8 */
                        const uint8_t *sb = wr + (b / 8) * Q4_K_BYTES;
                        const int j = (int)(b % 8);
                        const uint8_t byte = sb[16 + 32 * (j / 2) + l];
                        wi = (j & 1) ? (byte >> 4) : (byte & 0x0f);
                    }
                    s += wi * xs[l];
                }
                out[(r * N + n) * nblk + b] = s;
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* mul_mat_id routing (ggml semantics: ids [n_sel, N], entry i = s + t*n_sel) */
/* ------------------------------------------------------------------------ */
/* counts[e]: number of (s, t) slots routed to expert e; offsets[e]: exclusive
 * prefix sum; rows[offsets[e] + r]: the r-th slot index i (ascending) routed
 * to e. Slots whose id is outside [0, n_experts) are skipped and counted in
 * the return value. */
int64_t oracle_moe_route(const int32_t *ids, int64_t n_slots, int64_t n_experts, int32_t *counts,
                         int32_t *offsets, int32_t *rows) {
    int64_t bad = 0;
    for (int64_t e = 0; e < n_experts; e++) counts[e] = 0;
    for (int64_t i = 0; i < n_slots; i++) {
        const int32_t e = ids[i];
        if (e < 0 || e >= n_experts) { bad++; continue; }
        counts[e]++;
    }
    int32_t run = 0;
    for (int64_t e = 0; e < n_experts; e++) { offsets[e] = run; run += counts[e]; }
    int32_t *fill = (int32_t *)calloc((size_t)(n_experts > 0 ? n_experts : 1), sizeof(int32_t));
    for (int64_t i = 0; i < n_slots; i++) {
        const int32_t e = ids[i];
        if (e < 0 || e >= n_experts) continue;
        rows[offsets[e] + fill[e]++] = (int32_t)i;
    }
    free(fill);
    return bad;
}
