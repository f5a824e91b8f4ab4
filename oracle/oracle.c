/*
 * oracle.c — CPU restatement of llmtoy-zig's quantized MoE forward path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path and the
 * timed CPU baseline (bench.py's cpu_baseline leg and --impl reference arm).
 * The product never links or calls this file.
 *
 * Build: oracle/Makefile (-O3 -ffp-contract=off, so a*b+c always rounds
 * twice, exactly like Zig's strict float mode).  Each function names the
 * reference function it restates as path:line within llmtoy-zig.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ── f16 ──────────────────────────────────────────────────────────────────── */

/* src/quant/dequant.zig:302-305 — @floatCast of an f16 is exact. */
float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t exp = (h >> 10) & 0x1fu;
    const uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        /* zero or subnormal: value = mant * 2^-24, exactly representable */
        float v = ldexpf((float)mant, -24);
        memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp - 15u + 127u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u);
    if (ax >= 0x477ff000u) return sign | 0x7c00u; /* rounds to inf */
    if (ax < 0x38800000u) {                        /* f16 subnormal or zero */
        float a;
        memcpy(&a, &ax, 4);
        /* a * 2^24 rounded to nearest even integer = subnormal mantissa */
        float m = nearbyintf(ldexpf(a, 24));
        return sign | (uint16_t)m;
    }
    uint32_t mant = ax & 0x7fffffu;
    uint32_t e = (ax >> 23) - 127u + 15u;
    uint32_t r = (e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r += 1u;
    return sign | (uint16_t)r;
}

static inline float f16_at(const uint8_t *p) {
    return orc_f16_to_f32((uint16_t)(p[0] | (p[1] << 8)));
}

/* ── block codecs (src/quant/dequant.zig) ──────────────────────────────────── */

#define Q8_0_BLOCK_ELEMS 32
#define Q8_0_BLOCK_BYTES 34
#define QK_K 256
#define Q4_K_BLOCK_BYTES 144
#define Q6_K_BLOCK_BYTES 210

/* dequant.zig:17-20 */
void orc_dequant_f32(const uint8_t *data, float *out, size_t n) { memcpy(out, data, n * 4); }

/* dequant.zig:24-29 */
void orc_dequant_f16(const uint8_t *data, float *out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = f16_at(data + 2 * i);
}

/* dequant.zig:42-52: val = d * q */
void orc_dequant_q8_0(const uint8_t *data, float *out, size_t n) {
    const size_t nb = n / Q8_0_BLOCK_ELEMS;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = data + b * Q8_0_BLOCK_BYTES;
        const float d = f16_at(blk);
        for (size_t i = 0; i < Q8_0_BLOCK_ELEMS; i++)
            out[b * Q8_0_BLOCK_ELEMS + i] = d * (float)(int8_t)blk[2 + i];
    }
}

/* dequant.zig:59-78: per block, 8 lanes x 4 groups (mul then add), ordered
 * lane reduction, times d, accumulated block by block. */
float orc_dot_q8_0(const uint8_t *data, const float *vec, size_t n) {
    const size_t nb = n / Q8_0_BLOCK_ELEMS;
    float total = 0.0f;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = data + b * Q8_0_BLOCK_BYTES;
        const float d = f16_at(blk);
        const int8_t *qs = (const int8_t *)(blk + 2);
        const float *v = vec + b * Q8_0_BLOCK_ELEMS;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 4; j++)
            for (int l = 0; l < 8; l++) acc[l] += (float)qs[j * 8 + l] * v[j * 8 + l];
        float r = -0.0f;
        for (int l = 0; l < 8; l++) r += acc[l];
        total += r * d;
    }
    return total;
}

/* dequant.zig:291-300 (get_scale_min_k4) */
static inline void scale_min(int j, const uint8_t *s, uint8_t *sc, uint8_t *mn) {
    if (j < 4) {
        *sc = s[j] & 0x3f;
        *mn = s[j + 4] & 0x3f;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4));
        *mn = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* dequant.zig:157-187: out = (d*sc)*q - dmin*mn, two roundings */
void orc_dequant_q4_k(const uint8_t *data, float *out, size_t n) {
    const size_t nb = n / QK_K;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = data + b * Q4_K_BLOCK_BYTES;
        const float d = f16_at(blk);
        const float dmin = f16_at(blk + 2);
        const uint8_t *scales = blk + 4;
        const uint8_t *qs = blk + 16;
        int sub = 0;
        for (int chunk = 0; chunk < QK_K; chunk += 64) {
            uint8_t sc1, mn1, sc2, mn2;
            scale_min(sub, scales, &sc1, &mn1);
            scale_min(sub + 1, scales, &sc2, &mn2);
            sub += 2;
            const float d1 = d * (float)sc1, m1 = dmin * (float)mn1;
            const float d2 = d * (float)sc2, m2 = dmin * (float)mn2;
            for (int i = 0; i < 32; i++) {
                const uint8_t byte = qs[chunk / 2 + i];
                out[b * QK_K + chunk + i] = d1 * (float)(byte & 0x0f) - m1;
                out[b * QK_K + chunk + 32 + i] = d2 * (float)(byte >> 4) - m2;
            }
        }
    }
}

/* dequant.zig:282-287 */
static inline float q6val(uint8_t ql_byte, uint8_t qh_byte, int qh_shift, int ql_shift) {
    const uint8_t lo4 = (ql_byte >> ql_shift) & 0x0f;
    const uint8_t hi2 = (qh_byte >> qh_shift) & 0x03;
    const uint8_t raw = (uint8_t)(lo4 | (hi2 << 4));
    return (float)((int)raw - 32);
}

/* dequant.zig:237-277: out = (d * sc_i8) * (q6 - 32) */
void orc_dequant_q6_k(const uint8_t *data, float *out, size_t n) {
    const size_t nb = n / QK_K;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = data + b * Q6_K_BLOCK_BYTES;
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t *sc = (const int8_t *)(blk + 192);
        const float d = f16_at(blk + 208);
        int ql_off = 0, qh_off = 0, sc_off = 0;
        for (int chunk = 0; chunk < QK_K; chunk += 128, ql_off += 64, qh_off += 32, sc_off += 8) {
            for (int l = 0; l < 32; l++) {
                const int is = l / 16;
                const float q1 = q6val(ql[ql_off + l], qh[qh_off + l], 0, 0);
                const float q2 = q6val(ql[ql_off + l + 32], qh[qh_off + l], 2, 0);
                const float q3 = q6val(ql[ql_off + l], qh[qh_off + l], 4, 4);
                const float q4 = q6val(ql[ql_off + l + 32], qh[qh_off + l], 6, 4);
                const float s0 = d * (float)sc[sc_off + is + 0];
                const float s2 = d * (float)sc[sc_off + is + 2];
                const float s4 = d * (float)sc[sc_off + is + 4];
                const float s6 = d * (float)sc[sc_off + is + 6];
                const size_t base = b * QK_K + (size_t)chunk + (size_t)l;
                out[base + 0] = s0 * q1;
                out[base + 32] = s2 * q2;
                out[base + 64] = s4 * q3;
                out[base + 96] = s6 * q4;
            }
        }
    }
}

/* dequant.zig:201-217: d * ((nibble | qh bit << 4) - 16); element j < 16 takes
 * the low nibble of qs[j] and qh bit j, element j + 16 the high nibble and bit
 * j + 16. */
void orc_dequant_q5_0(const uint8_t *data, float *out, size_t n) {
    for (size_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + b * 22;
        const float d = f16_at(blk);
        const uint32_t qh = (uint32_t)blk[2] | (uint32_t)blk[3] << 8 | (uint32_t)blk[4] << 16 | (uint32_t)blk[5] << 24;
        const uint8_t *qs = blk + 6;
        for (int j = 0; j < 16; j++) {
            const int x0 = (int)((qs[j] & 0x0f) | (((qh >> j) & 1u) << 4)) - 16;
            const int x1 = (int)((qs[j] >> 4) | (((qh >> (j + 16)) & 1u) << 4)) - 16;
            out[b * 32 + j] = d * (float)x0;
            out[b * 32 + j + 16] = d * (float)x1;
        }
    }
}

/* dequant.zig:92-133: per block 8 lanes x 4 groups of (q5 - 16) * v (mul then
 * add), ordered lane reduction, times d, accumulated block by block. */
float orc_dot_q5_0(const uint8_t *data, const float *vec, size_t n) {
    float total = 0.0f;
    for (size_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + b * 22;
        const float d = f16_at(blk);
        const uint32_t qh = (uint32_t)blk[2] | (uint32_t)blk[3] << 8 | (uint32_t)blk[4] << 16 | (uint32_t)blk[5] << 24;
        const uint8_t *qs = blk + 6;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int g = 0; g < 4; g++) {
            const int qs_off = (g & 1) * 8, hi = g >= 2, qh_off = g < 2 ? g * 8 : (g - 2) * 8 + 16;
            for (int l = 0; l < 8; l++) {
                const uint8_t nib = hi ? (uint8_t)(qs[qs_off + l] >> 4) : (uint8_t)(qs[qs_off + l] & 0x0f);
                const uint8_t hb = (uint8_t)((qh >> (qh_off + l)) & 1u);
                const float q5 = (float)(nib | (hb << 4)) - 16.0f;
                acc[l] += q5 * vec[b * 32 + g * 8 + l];
            }
        }
        float r = -0.0f;
        for (int l = 0; l < 8; l++) r += acc[l];
        total += r * d;
    }
    return total;
}

/* dequant.zig:469-487: d * q + m (two roundings) */
void orc_dequant_q5_1(const uint8_t *data, float *out, size_t n) {
    for (size_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + b * 24;
        const float d = f16_at(blk), m = f16_at(blk + 2);
        const uint8_t *qh = blk + 4, *qs = blk + 8;
        for (int j = 0; j < 16; j++) {
            const uint8_t hi0 = (uint8_t)(((qh[j / 8] >> (j % 8)) & 1) << 4);
            const uint8_t hi1 = (uint8_t)(((qh[(j + 16) / 8] >> ((j + 16) % 8)) & 1) << 4);
            out[b * 32 + j] = d * (float)((qs[j] & 0x0f) | hi0) + m;
            out[b * 32 + j + 16] = d * (float)((qs[j] >> 4) | hi1) + m;
        }
    }
}

/* dequant.zig:324-367: Q4_K's (d*sc) * q - dmin*mn with q = nibble + 16 * bit,
 * the bit from qh[l] & (1 << 2c) (low nibbles) or (2 << 2c) (high nibbles). */
void orc_dequant_q5_k(const uint8_t *data, float *out, size_t n) {
    for (size_t b = 0; b < n / QK_K; b++) {
        const uint8_t *blk = data + b * 176;
        const float d = f16_at(blk), dmin = f16_at(blk + 2);
        const uint8_t *scales = blk + 4, *qh = blk + 16, *ql = blk + 48;
        uint8_t um1 = 1, um2 = 2;
        for (int c = 0; c < 4; c++) {
            uint8_t sc1, mn1, sc2, mn2;
            scale_min(2 * c, scales, &sc1, &mn1);
            scale_min(2 * c + 1, scales, &sc2, &mn2);
            const float d1 = d * (float)sc1, m1 = dmin * (float)mn1;
            const float d2 = d * (float)sc2, m2 = dmin * (float)mn2;
            for (int l = 0; l < 32; l++) {
                const float hi = (qh[l] & um1) ? 16.0f : 0.0f;
                out[b * QK_K + 64 * c + l] = d1 * ((float)(ql[32 * c + l] & 0x0f) + hi) - m1;
            }
            for (int l = 0; l < 32; l++) {
                const float hi = (qh[l] & um2) ? 16.0f : 0.0f;
                out[b * QK_K + 64 * c + 32 + l] = d2 * ((float)(ql[32 * c + l] >> 4) + hi) - m2;
            }
            um1 = (uint8_t)(um1 * 4);
            um2 = (uint8_t)(um2 * 4);
        }
    }
}

/* dequant.zig:388-464: sixteen 6-bit scales unpacked from 12 bytes with the
 * kmask steps, dl = d * (sc - 32); value dl * ((qs >> shift & 3) - (hmask bit ? 0 : 4)). */
void orc_dequant_q3_k(const uint8_t *data, float *out, size_t n) {
    for (size_t b = 0; b < n / QK_K; b++) {
        const uint8_t *blk = data + b * 110;
        const uint8_t *hmask = blk, *qs = blk + 32;
        const float d_all = f16_at(blk + 108);
        uint32_t aux[4], tmp;
        memcpy(&aux[0], blk + 96, 4);
        memcpy(&aux[1], blk + 100, 4);
        memcpy(&tmp, blk + 104, 4);
        const uint32_t k1 = 0x03030303u, k2 = 0x0f0f0f0fu;
        aux[2] = ((aux[0] >> 4) & k2) | (((tmp >> 4) & k1) << 4);
        aux[3] = ((aux[1] >> 4) & k2) | (((tmp >> 6) & k1) << 4);
        aux[0] = (aux[0] & k2) | (((tmp >> 0) & k1) << 4);
        aux[1] = (aux[1] & k2) | (((tmp >> 2) & k1) << 4);
        uint8_t sc[16];
        memcpy(sc, aux, 16);
        int is = 0;
        uint8_t m = 1;
        size_t o = b * QK_K;
        for (int half = 0; half < 2; half++) {
            const uint8_t *q = qs + 32 * half;
            int shift = 0;
            for (int j = 0; j < 4; j++) {
                for (int g = 0; g < 2; g++) {
                    const float dl = d_all * ((float)sc[is++] - 32.0f);
                    for (int l = 0; l < 16; l++) {
                        const int lo2 = (q[16 * g + l] >> shift) & 3;
                        const int v = lo2 - ((hmask[16 * g + l] & m) ? 0 : 4);
                        out[o++] = (float)v * dl;
                    }
                }
                shift += 2;
                m = (uint8_t)(m << 1);
            }
        }
    }
}

static const float kIq4Table[16] = {-127.0f, -104.0f, -83.0f, -65.0f, -49.0f, -35.0f, -22.0f, -10.0f,
                                    1.0f,    13.0f,   25.0f,  38.0f,  53.0f,  69.0f,  89.0f,  113.0f};

/* dequant.zig:623-640 */
void orc_dequant_iq4_nl(const uint8_t *data, float *out, size_t n) {
    for (size_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + b * 18;
        const float d = f16_at(blk);
        for (int j = 0; j < 16; j++) {
            out[b * 32 + j] = d * kIq4Table[blk[2 + j] & 0x0f];
            out[b * 32 + j + 16] = d * kIq4Table[blk[2 + j] >> 4];
        }
    }
}

/* dequant.zig:642-660: one scalar accumulator per block (low nibble's term,
 * then the high nibble's), d * acc added block by block. */
float orc_dot_iq4_nl(const uint8_t *data, const float *vec, size_t n) {
    float total = 0.0f;
    for (size_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + b * 18;
        const float d = f16_at(blk);
        float acc = 0.0f;
        for (int j = 0; j < 16; j++) {
            const uint8_t q = blk[2 + j];
            acc += kIq4Table[q & 0x0f] * vec[b * 32 + j];
            acc += kIq4Table[q >> 4] * vec[b * 32 + j + 16];
        }
        total += d * acc;
    }
    return total;
}

/* dequant.zig:517-547: d = amax / 127, q = clamp(round(x / d)) with Zig's
 * @round (halves away from zero), s = d * sum(q), both stored as f16. */
void orc_quantize_q8_1(const float *in, uint8_t *out, size_t n) {
    for (size_t b = 0; b < n / 32; b++) {
        const float *src = in + b * 32;
        uint8_t *blk = out + b * 36;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) {
            const float a = fabsf(src[i]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        const float inv_d = d != 0.0f ? 1.0f / d : 0.0f;
        int32_t sum_qs = 0;
        const uint16_t dh = orc_f32_to_f16(d);
        blk[0] = (uint8_t)(dh & 0xff);
        blk[1] = (uint8_t)(dh >> 8);
        for (int i = 0; i < 32; i++) {
            float q = roundf(src[i] * inv_d);
            q = q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
            const int32_t qi = (int32_t)q;
            sum_qs += qi;
            blk[4 + i] = (uint8_t)(int8_t)qi;
        }
        const uint16_t sh = orc_f32_to_f16(d * (float)sum_qs);
        blk[2] = (uint8_t)(sh & 0xff);
        blk[3] = (uint8_t)(sh >> 8);
    }
}

/* dequant.zig:549-558 */
void orc_dequant_q8_1(const uint8_t *data, float *out, size_t n) {
    for (size_t b = 0; b < n / 32; b++) {
        const uint8_t *blk = data + b * 36;
        const float d = f16_at(blk);
        for (int i = 0; i < 32; i++) out[b * 32 + i] = d * (float)(int8_t)blk[4 + i];
    }
}

/* dequant.zig:569-586: groups of four blocks as {ds[4], qs[4][32]}, the last
 * group zero-padded. */
void orc_pack_q8_1_x4(const uint8_t *basic, size_t n_blocks, uint8_t *x4) {
    const size_t n_groups = (n_blocks + 3) / 4;
    memset(x4, 0, n_groups * 144);
    for (size_t bi = 0; bi < n_blocks; bi++) {
        const size_t g = bi / 4, i = bi % 4;
        memcpy(x4 + g * 144 + i * 4, basic + bi * 36, 4);
        memcpy(x4 + g * 144 + 16 + i * 32, basic + bi * 36 + 4, 32);
    }
}

/* dequant.zig:588-613 */
void orc_unpack_q8_1_x4(const uint8_t *x4, size_t n_groups, uint8_t *basic) {
    for (size_t g = 0; g < n_groups; g++)
        for (int i = 0; i < 4; i++) {
            memcpy(basic + (g * 4 + i) * 36, x4 + g * 144 + i * 4, 4);
            memcpy(basic + (g * 4 + i) * 36 + 4, x4 + g * 144 + 16 + i * 32, 32);
        }
}

/* math.zig:194-208 */
size_t orc_row_bytes(uint32_t type, size_t cols) {
    switch (type) {
    case ORC_F32: return cols * 4;
    case ORC_F16: return cols * 2;
    case ORC_Q8_0: return (cols / Q8_0_BLOCK_ELEMS) * Q8_0_BLOCK_BYTES;
    case ORC_Q4_K: return (cols / QK_K) * Q4_K_BLOCK_BYTES;
    case ORC_Q6_K: return (cols / QK_K) * Q6_K_BLOCK_BYTES;
    case ORC_Q5_0: return (cols / 32) * 22;
    case ORC_Q5_1: return (cols / 32) * 24;
    case ORC_Q5_K: return (cols / QK_K) * 176;
    case ORC_Q3_K: return (cols / QK_K) * 110;
    case ORC_IQ4_NL: return (cols / 32) * 18;
    default: return 0;
    }
}

/* math.zig:211-225 */
int orc_dequant_row(const uint8_t *data, float *out, size_t n, uint32_t type) {
    switch (type) {
    case ORC_F32: orc_dequant_f32(data, out, n); return 0;
    case ORC_F16: orc_dequant_f16(data, out, n); return 0;
    case ORC_Q8_0: orc_dequant_q8_0(data, out, n); return 0;
    case ORC_Q4_K: orc_dequant_q4_k(data, out, n); return 0;
    case ORC_Q6_K: orc_dequant_q6_k(data, out, n); return 0;
    case ORC_Q5_0: orc_dequant_q5_0(data, out, n); return 0;
    case ORC_Q5_1: orc_dequant_q5_1(data, out, n); return 0;
    case ORC_Q5_K: orc_dequant_q5_k(data, out, n); return 0;
    case ORC_Q3_K: orc_dequant_q3_k(data, out, n); return 0;
    case ORC_IQ4_NL: orc_dequant_iq4_nl(data, out, n); return 0;
    default: return -1;
    }
}

/* ── src/ops/math.zig ──────────────────────────────────────────────────────── */

/* math.zig:8-17 */
void orc_matvec(float *out, const float *mat, const float *vec, size_t rows, size_t cols) {
    for (size_t i = 0; i < rows; i++) {
        float sum = 0.0f;
        for (size_t j = 0; j < cols; j++) sum += mat[i * cols + j] * vec[j];
        out[i] = sum;
    }
}

/* math.zig:96-116: 4 accumulators x 8 lanes over 32-element strides,
 * (a0+a1)+(a2+a3), an 8-wide tail, ordered lane reduction, scalar tail. */
float orc_dotf32(const float *a, const float *b, size_t n) {
    float acc0[8] = {0}, acc1[8] = {0}, acc2[8] = {0}, acc3[8] = {0};
    size_t i = 0;
    for (; i + 32 <= n; i += 32) {
        for (int l = 0; l < 8; l++) acc0[l] += a[i + l] * b[i + l];
        for (int l = 0; l < 8; l++) acc1[l] += a[i + 8 + l] * b[i + 8 + l];
        for (int l = 0; l < 8; l++) acc2[l] += a[i + 16 + l] * b[i + 16 + l];
        for (int l = 0; l < 8; l++) acc3[l] += a[i + 24 + l] * b[i + 24 + l];
    }
    float acc[8];
    for (int l = 0; l < 8; l++) acc[l] = (acc0[l] + acc1[l]) + (acc2[l] + acc3[l]);
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) acc[l] += a[i + l] * b[i + l];
    float sum = -0.0f;
    for (int l = 0; l < 8; l++) sum += acc[l];
    for (; i < n; i++) sum += a[i] * b[i];
    return sum;
}

/* math.zig:133-171 (plus RowJob.run :243-269, which is the same loop) */
static int quant_matvec_rows(float *out, const uint8_t *mat, uint32_t type, const float *vec,
                             size_t row_start, size_t n_rows, size_t cols, float *row_buf) {
    const size_t rb = orc_row_bytes(type, cols);
    if (rb == 0) return -1;
    for (size_t i = 0; i < n_rows; i++) {
        const uint8_t *row = mat + (row_start + i) * rb;
        if (type == ORC_Q8_0) {
            out[i] = orc_dot_q8_0(row, vec, cols);
            continue;
        }
        if (type == ORC_Q5_0) {
            out[i] = orc_dot_q5_0(row, vec, cols);
            continue;
        }
        if (type == ORC_IQ4_NL) {
            out[i] = orc_dot_iq4_nl(row, vec, cols);
            continue;
        }
        if (type == ORC_F32 && ((uintptr_t)row % 4) == 0) {
            out[i] = orc_dotf32((const float *)row, vec, cols);
            continue;
        }
        orc_dequant_row(row, row_buf, cols, type);
        out[i] = orc_dotf32(row_buf, vec, cols);
    }
    return 0;
}

int orc_quant_matvec(float *out, const uint8_t *mat, uint32_t type, const float *vec,
                     size_t rows, size_t cols, float *row_buf) {
    return quant_matvec_rows(out, mat, type, vec, 0, rows, cols, row_buf);
}

/* math.zig:20-26 */
void orc_rmsnorm(float *out, const float *x, const float *w, size_t n, float eps) {
    float ss = 0.0f;
    for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
    const float rms_inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (size_t i = 0; i < n; i++) out[i] = x[i] * rms_inv * w[i];
}

/* math.zig:43-48 */
void orc_rmsnorm_raw(float *out, const float *x, size_t n, float eps) {
    float ss = 0.0f;
    for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
    const float rms_inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (size_t i = 0; i < n; i++) out[i] = x[i] * rms_inv;
}

/* math.zig:29-35 */
void orc_softmax(float *x, size_t n) {
    float max = x[0];
    for (size_t i = 1; i < n; i++)
        if (x[i] > max) max = x[i];
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        x[i] = expf(x[i] - max);
        sum += x[i];
    }
    for (size_t i = 0; i < n; i++) x[i] /= sum;
}

/* math.zig:38-40 */
float orc_silu(float x) { return x / (1.0f + expf(-x)); }

/* math.zig:85-88 */
float orc_gelu(float x) {
    const float c = 0.7978845608028654f;
    return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

/* ── worker pool (src/ops/thread_pool.zig:15-112) ──────────────────────────── */

typedef void (*orc_func)(void *);
typedef struct { orc_func func; void *ctx; } orc_entry;

struct orc_pool {
    pthread_t *threads;
    int n_threads;
    orc_entry *queue;
    size_t cap, head, tail, pending;
    int shutdown;
    pthread_mutex_t mutex;
    pthread_cond_t work_ready, all_done, not_full;
};

static void *worker_loop(void *arg) {
    orc_pool *p = (orc_pool *)arg;
    pthread_mutex_lock(&p->mutex);
    for (;;) {
        while (p->head == p->tail && !p->shutdown) pthread_cond_wait(&p->work_ready, &p->mutex);
        if (p->shutdown && p->head == p->tail) {
            pthread_mutex_unlock(&p->mutex);
            return NULL;
        }
        orc_entry e = p->queue[p->tail % p->cap];
        p->tail++;
        pthread_cond_signal(&p->not_full);
        pthread_mutex_unlock(&p->mutex);
        e.func(e.ctx);
        pthread_mutex_lock(&p->mutex);
        p->pending--;
        if (p->pending == 0) pthread_cond_signal(&p->all_done);
    }
}

orc_pool *orc_pool_create(int n) {
    if (n < 1) n = 1;
    orc_pool *p = (orc_pool *)calloc(1, sizeof(*p));
    if (!p) return NULL;
    p->n_threads = n;
    p->cap = (size_t)(n * 4 > 64 ? n * 4 : 64);
    p->queue = (orc_entry *)calloc(p->cap, sizeof(orc_entry));
    p->threads = (pthread_t *)calloc((size_t)n, sizeof(pthread_t));
    pthread_mutex_init(&p->mutex, NULL);
    pthread_cond_init(&p->work_ready, NULL);
    pthread_cond_init(&p->all_done, NULL);
    pthread_cond_init(&p->not_full, NULL);
    for (int i = 0; i < n; i++) pthread_create(&p->threads[i], NULL, worker_loop, p);
    return p;
}

void orc_pool_destroy(orc_pool *p) {
    if (!p) return;
    pthread_mutex_lock(&p->mutex);
    p->shutdown = 1;
    pthread_cond_broadcast(&p->work_ready);
    pthread_mutex_unlock(&p->mutex);
    for (int i = 0; i < p->n_threads; i++) pthread_join(p->threads[i], NULL);
    free(p->threads);
    free(p->queue);
    free(p);
}

int orc_pool_threads(const orc_pool *p) { return p ? p->n_threads : 1; }

static void pool_submit(orc_pool *p, orc_func f, void *ctx) {
    pthread_mutex_lock(&p->mutex);
    while (p->head - p->tail >= p->cap) pthread_cond_wait(&p->not_full, &p->mutex);
    p->queue[p->head % p->cap] = (orc_entry){f, ctx};
    p->head++;
    p->pending++;
    pthread_cond_signal(&p->work_ready);
    pthread_mutex_unlock(&p->mutex);
}

static void pool_wait(orc_pool *p) {
    pthread_mutex_lock(&p->mutex);
    while (p->pending > 0) pthread_cond_wait(&p->all_done, &p->mutex);
    pthread_mutex_unlock(&p->mutex);
}

/* ── quantMatvecPar (math.zig:227-320) ─────────────────────────────────────── */

typedef struct {
    const uint8_t *mat;
    uint32_t type;
    const float *vec;
    float *out;
    float *row_buf;
    size_t row_start, n_rows, cols;
} row_job;

static void row_job_run(void *ctx) {
    row_job *j = (row_job *)ctx;
    quant_matvec_rows(j->out, j->mat, j->type, j->vec, j->row_start, j->n_rows, j->cols, j->row_buf);
}

int orc_quant_matvec_par(float *out, const uint8_t *mat, uint32_t type, const float *vec,
                         size_t rows, size_t cols, float *scratch, orc_pool *pool) {
    if (orc_row_bytes(type, cols) == 0) return -1;
    const size_t min_rows = 64;
    const size_t n = (size_t)orc_pool_threads(pool);
    size_t nt = (rows + min_rows - 1) / min_rows;
    if (n < nt) nt = n;
    if (nt <= 1 || pool == NULL) return orc_quant_matvec(out, mat, type, vec, rows, cols, scratch);
    if (nt > 64) nt = 64;
    row_job jobs[64];
    const size_t base = rows / nt, extra = rows % nt;
    size_t row = 0;
    for (size_t t = 0; t < nt; t++) {
        const size_t n_rows = base + (t < extra ? 1 : 0);
        jobs[t] = (row_job){mat, type, vec, out + row, scratch + t * cols, row, n_rows, cols};
        pool_submit(pool, row_job_run, &jobs[t]);
        row += n_rows;
    }
    pool_wait(pool);
    return 0;
}

/* ── router (src/model/gemma4/forward.zig) ─────────────────────────────────── */

/* forward.zig:598-629: one pass, online softmax denominator + insertion top-k
 * with strict '>' so the lowest index wins ties. */
orc_softmax_stats orc_topk_with_softmax_stats(const float *scores, size_t n, uint32_t *out, size_t k) {
    float max = scores[0];
    float exp_sum = 0.0f;
    size_t filled = 0;
    for (size_t j = 0; j < n; j++) {
        const float s = scores[j];
        if (s > max) {
            exp_sum = exp_sum * expf(max - s) + 1.0f;
            max = s;
        } else {
            exp_sum += expf(s - max);
        }
        if (filled < k) {
            size_t pos = filled++;
            while (pos > 0 && s > scores[out[pos - 1]]) {
                out[pos] = out[pos - 1];
                pos--;
            }
            out[pos] = (uint32_t)j;
        } else if (s > scores[out[k - 1]]) {
            size_t pos = k - 1;
            while (pos > 0 && s > scores[out[pos - 1]]) {
                out[pos] = out[pos - 1];
                pos--;
            }
            out[pos] = (uint32_t)j;
        }
    }
    return (orc_softmax_stats){max, exp_sum};
}

/* forward.zig:637-643 */
void orc_softmax_topk(float *scores, size_t n, uint32_t *out, size_t k) {
    const orc_softmax_stats st = orc_topk_with_softmax_stats(scores, n, out, k);
    for (size_t i = 0; i < k; i++) scores[out[i]] = expf(scores[out[i]] - st.max) / st.exp_sum;
}

/* forward.zig:748-767 */
static void insert_topk_index(uint32_t *out, float *sel, size_t k, size_t *filled, uint32_t idx, float score) {
    if (*filled < k) {
        size_t pos = (*filled)++;
        while (pos > 0 && score > sel[pos - 1]) {
            sel[pos] = sel[pos - 1];
            out[pos] = out[pos - 1];
            pos--;
        }
        sel[pos] = score;
        out[pos] = idx;
    } else if (score > sel[k - 1]) {
        size_t pos = k - 1;
        while (pos > 0 && score > sel[pos - 1]) {
            sel[pos] = sel[pos - 1];
            out[pos] = out[pos - 1];
            pos--;
        }
        sel[pos] = score;
        out[pos] = idx;
    }
}

/* forward.zig:672-712: streamed router logits (dotf32 per expert row). */
orc_softmax_stats orc_topk_matvec_f32(const float *w, const float *vec, size_t rows, size_t cols,
                                      uint32_t *out, float *selected, size_t k) {
    float max = -INFINITY;
    float exp_sum = 0.0f;
    size_t filled = 0;
    for (size_t j = 0; j < rows; j++) {
        const float score = orc_dotf32(w + j * cols, vec, cols);
        if (score > max) {
            exp_sum = exp_sum * expf(max - score) + 1.0f;
            max = score;
        } else {
            exp_sum += expf(score - max);
        }
        insert_topk_index(out, selected, k, &filled, (uint32_t)j, score);
    }
    return (orc_softmax_stats){max, exp_sum};
}

typedef struct {
    const float *w, *vec;
    size_t row_start, rows, cols, k;
    uint32_t top_idx[16];
    float top_scores[16];
    orc_softmax_stats stats;
} router_job;

/* forward.zig:730-745 */
static void router_job_run(void *ctx) {
    router_job *j = (router_job *)ctx;
    uint32_t local_idx[16];
    float local_scores[16];
    j->stats = orc_topk_matvec_f32(j->w + j->row_start * j->cols, j->vec, j->rows, j->cols,
                                   local_idx, local_scores, j->k);
    for (size_t i = 0; i < j->k; i++) {
        j->top_idx[i] = (uint32_t)j->row_start + local_idx[i];
        j->top_scores[i] = local_scores[i];
    }
}

/* forward.zig:769-821: row ranges per job, merged in ascending row order. */
orc_softmax_stats orc_topk_matvec_f32_par(const float *w, const float *vec, size_t rows, size_t cols,
                                          uint32_t *out, float *selected, size_t k, orc_pool *pool) {
    const size_t min_rows_per_job = 16;
    size_t nt = (rows + min_rows_per_job - 1) / min_rows_per_job;
    const size_t n = (size_t)orc_pool_threads(pool);
    if (n < nt) nt = n;
    if (nt <= 1 || pool == NULL) return orc_topk_matvec_f32(w, vec, rows, cols, out, selected, k);
    if (nt > 64) nt = 64;
    router_job jobs[64];
    const size_t base = rows / nt, extra = rows % nt;
    size_t row = 0;
    for (size_t t = 0; t < nt; t++) {
        const size_t n_rows = base + (t < extra ? 1 : 0);
        memset(&jobs[t], 0, sizeof(jobs[t]));
        jobs[t].w = w;
        jobs[t].vec = vec;
        jobs[t].row_start = row;
        jobs[t].rows = n_rows;
        jobs[t].cols = cols;
        jobs[t].k = k;
        pool_submit(pool, router_job_run, &jobs[t]);
        row += n_rows;
    }
    pool_wait(pool);

    float max = -INFINITY;
    float exp_sum = 0.0f;
    size_t filled = 0;
    for (size_t t = 0; t < nt; t++) {
        const router_job *j = &jobs[t];
        if (j->stats.max > max) {
            exp_sum = exp_sum * expf(max - j->stats.max) + j->stats.exp_sum;
            max = j->stats.max;
        } else {
            exp_sum += j->stats.exp_sum * expf(j->stats.max - max);
        }
        for (size_t i = 0; i < k; i++) insert_topk_index(out, selected, k, &filled, j->top_idx[i], j->top_scores[i]);
    }
    return (orc_softmax_stats){max, exp_sum};
}

/* forward.zig:648-668 (aligned f32 router weights branch) */
void orc_router_topk_softmax(float *scores, uint32_t *out, size_t k, const float *router_w,
                             size_t rows, size_t cols, const float *router_in, orc_pool *pool) {
    float selected[16];
    const orc_softmax_stats st = orc_topk_matvec_f32_par(router_w, router_in, rows, cols, out, selected, k, pool);
    for (size_t i = 0; i < k; i++) scores[out[i]] = expf(selected[i] - st.max) / st.exp_sum;
}

/* src/ops/moe.zig:80-91 */
void orc_moe_topk(const float *scores, size_t n, uint32_t *out, size_t k) {
    for (size_t i = 0; i < k; i++) {
        size_t best = 0;
        float best_val = -INFINITY;
        for (size_t j = 0; j < n; j++) {
            int already = 0;
            for (size_t p = 0; p < i; p++)
                if (out[p] == j) { already = 1; break; }
            if (!already && scores[j] > best_val) {
                best_val = scores[j];
                best = j;
            }
        }
        out[i] = (uint32_t)best;
    }
}

/* ── MoE FFN ──────────────────────────────────────────────────────────────── */

static size_t max_sz(size_t a, size_t b) { return a > b ? a : b; }

/* src/ops/moe.zig:18-77 */
int orc_moe_forward(float *out, const float *router_w, size_t n_experts,
                    const uint8_t *gate_up, uint32_t gate_up_type,
                    const uint8_t *down, uint32_t down_type,
                    const float *x, size_t d_model, size_t n_used, size_t d_expert,
                    orc_pool *pool) {
    const size_t nthr = (size_t)orc_pool_threads(pool);
    const size_t max_cols = max_sz(d_model, d_expert);
    float *gate_buf = (float *)malloc(d_expert * 4), *up_buf = (float *)malloc(d_expert * 4);
    float *down_buf = (float *)malloc(d_model * 4), *scratch = (float *)malloc(nthr * max_cols * 4);
    float *scores = (float *)malloc(n_experts * 4);
    uint32_t top_idx[64];
    int rc = 0;
    if (n_used > 64 || !gate_buf || !up_buf || !down_buf || !scratch || !scores) { rc = -1; goto done; }

    orc_quant_matvec(scores, (const uint8_t *)router_w, ORC_F32, x, n_experts, d_model, scratch);
    orc_softmax(scores, n_experts);
    orc_moe_topk(scores, n_experts, top_idx, n_used);

    const size_t gu_row_bytes = orc_row_bytes(gate_up_type, d_model);
    const size_t gu_per_expert = 2 * d_expert * gu_row_bytes;
    const size_t dn_row_bytes = orc_row_bytes(down_type, d_expert);
    const size_t dn_per_expert = d_model * dn_row_bytes;
    if (gu_row_bytes == 0 || dn_row_bytes == 0) { rc = -1; goto done; }

    for (size_t i = 0; i < n_used; i++) {
        const uint32_t e = top_idx[i];
        const float w = scores[e];
        const uint8_t *gate_data = gate_up + e * gu_per_expert;
        orc_quant_matvec_par(gate_buf, gate_data, gate_up_type, x, d_expert, d_model, scratch, pool);
        const uint8_t *up_data = gate_data + d_expert * gu_row_bytes;
        orc_quant_matvec_par(up_buf, up_data, gate_up_type, x, d_expert, d_model, scratch, pool);
        for (size_t r = 0; r < d_expert; r++) gate_buf[r] = orc_silu(gate_buf[r]) * up_buf[r];
        orc_quant_matvec_par(down_buf, down + e * dn_per_expert, down_type, gate_buf, d_model, d_expert, scratch, pool);
        for (size_t r = 0; r < d_model; r++) out[r] += w * down_buf[r];
    }
done:
    free(gate_buf); free(up_buf); free(down_buf); free(scratch); free(scores);
    return rc;
}

int orc_moe_layer(float *out, const float *x, size_t n_tok, size_t d_model,
                  const float *router_w, size_t n_experts, size_t k, int norm_topk,
                  const float *expert_scale,
                  const uint8_t *gate, const uint8_t *up, uint32_t gate_type,
                  const uint8_t *down, uint32_t down_type, size_t d_expert, int act,
                  orc_pool *pool, uint32_t *ids_out, float *w_out) {
    if (k == 0 || k > 16 || k > n_experts) return -1;
    const size_t gu_rb = orc_row_bytes(gate_type, d_model);
    const size_t dn_rb = orc_row_bytes(down_type, d_expert);
    if (gu_rb == 0 || dn_rb == 0) return -1;
    /* fused gate_up: gate rows [0,F), up rows [F,2F) of one expert
     * (gemma4/forward.zig:464-471); separate: F rows per expert each. */
    const size_t gate_per_expert = (up ? 1 : 2) * d_expert * gu_rb;
    const size_t up_per_expert = d_expert * gu_rb;
    const size_t dn_per_expert = d_model * dn_rb;

    const size_t nthr = (size_t)orc_pool_threads(pool);
    const size_t max_cols = max_sz(d_model, d_expert);
    float *eg = (float *)malloc(d_expert * 4), *eu = (float *)malloc(d_expert * 4);
    float *ed = (float *)malloc(d_model * 4), *scratch = (float *)malloc(nthr * max_cols * 4);
    float *scores = (float *)malloc(n_experts * 4);
    int rc = 0;
    if (!eg || !eu || !ed || !scratch || !scores) { rc = -1; goto done; }

    for (size_t t = 0; t < n_tok; t++) {
        const float *xt = x + t * d_model;
        float *ot = out + t * d_model;
        uint32_t top_idx[16];
        float w[16];
        orc_router_topk_softmax(scores, top_idx, k, router_w, n_experts, d_model, xt, pool);
        for (size_t i = 0; i < k; i++) w[i] = scores[top_idx[i]];
        if (norm_topk) {
            float s = 0.0f;
            for (size_t i = 0; i < k; i++) s += w[i];
            for (size_t i = 0; i < k; i++) w[i] = w[i] / s;
        }
        if (expert_scale)
            for (size_t i = 0; i < k; i++) w[i] = expert_scale[top_idx[i]] * w[i];

        memset(ot, 0, d_model * 4);
        for (size_t i = 0; i < k; i++) {
            const uint32_t e = top_idx[i];
            const uint8_t *gate_data = gate + e * gate_per_expert;
            const uint8_t *up_data = up ? up + e * up_per_expert : gate_data + d_expert * gu_rb;
            orc_quant_matvec_par(eg, gate_data, gate_type, xt, d_expert, d_model, scratch, pool);
            orc_quant_matvec_par(eu, up_data, gate_type, xt, d_expert, d_model, scratch, pool);
            if (act == 1)
                for (size_t r = 0; r < d_expert; r++) eg[r] = orc_gelu(eg[r]) * eu[r];
            else
                for (size_t r = 0; r < d_expert; r++) eg[r] = orc_silu(eg[r]) * eu[r];
            orc_quant_matvec_par(ed, down + e * dn_per_expert, down_type, eg, d_model, d_expert, scratch, pool);
            for (size_t r = 0; r < d_model; r++) ot[r] += w[i] * ed[r];
        }
        if (ids_out) memcpy(ids_out + t * k, top_idx, k * 4);
        if (w_out) memcpy(w_out + t * k, w, k * 4);
    }
done:
    free(eg); free(eu); free(ed); free(scratch); free(scores);
    return rc;
}

/* src/model/sample.zig:11-17 */
uint32_t orc_greedy(const float *logits, size_t n) {
    uint32_t best = 0;
    for (size_t i = 1; i < n; i++)
        if (logits[i] > logits[best]) best = (uint32_t)i;
    return best;
}

/* rope.zig:14-31 and :56-75 */
void orc_rope(float *vec, size_t len, size_t pos, float theta, int neox) {
    const size_t half = len / 2;
    for (size_t i = 0; i < half; i++) {
        const float freq = 1.0f / powf(theta, (float)(2 * i) / (float)len);
        const float angle = (float)pos * freq;
        const float c = cosf(angle), s = sinf(angle);
        const size_t i0 = neox ? i : 2 * i, i1 = neox ? i + half : 2 * i + 1;
        const float x0 = vec[i0], x1 = vec[i1];
        vec[i0] = x0 * c - x1 * s;
        vec[i1] = x0 * s + x1 * c;
    }
}

/* attn.zig:13-42 */
void orc_sdp_attn(float *out, const float *q, const float *ks, const float *vs, size_t seq_len,
                  size_t head_dim, float scale) {
    float *scores = (float *)malloc(seq_len * 4);
    for (size_t i = 0; i < seq_len; i++) {
        float dot = 0.0f;
        for (size_t j = 0; j < head_dim; j++) dot += q[j] * ks[i * head_dim + j];
        scores[i] = dot * scale;
    }
    orc_softmax(scores, seq_len);
    memset(out, 0, head_dim * 4);
    for (size_t i = 0; i < seq_len; i++)
        for (size_t j = 0; j < head_dim; j++) out[j] += scores[i] * vs[i * head_dim + j];
    free(scores);
}

/* forward.zig:229-316 (see oracle.h) */
int orc_model_step(const orc_model *m, float *k_cache, float *v_cache, size_t kv_cap, uint32_t token,
                   size_t pos, float *logits, orc_pool *pool) {
    const size_t d = m->d_model, hd = m->head_dim, nq = m->n_heads * hd, nkv = m->n_kv_heads * hd;
    const size_t ff = m->d_ffn, seq = pos + 1;
    if (pos >= kv_cap || token >= m->vocab) return -1;
    size_t max_cols = d > nq ? d : nq;
    if (ff > max_cols) max_cols = ff;
    const size_t nthr = (size_t)orc_pool_threads(pool);
    float *scratch = (float *)malloc((nthr ? nthr : 1) * max_cols * 4);
    float *x = (float *)malloc(d * 4), *xb = (float *)malloc(d * 4), *q = (float *)malloc(nq * 4);
    float *kn = (float *)malloc(nkv * 4), *vn = (float *)malloc(nkv * 4), *att = (float *)malloc(nq * 4);
    float *ks = (float *)malloc(seq * hd * 4), *vs = (float *)malloc(seq * hd * 4);
    float *proj = (float *)malloc(d * 4), *g = (float *)malloc((ff ? ff : 1) * 4);
    float *u = (float *)malloc((ff ? ff : 1) * 4), *fo = (float *)malloc(d * 4);
    const float scale = 1.0f / sqrtf((float)hd);
    int rc = orc_dequant_row(m->token_emb + (size_t)token * orc_row_bytes(m->emb_type, d), x, d, m->emb_type);
    for (size_t l = 0; l < m->n_layers && rc == 0; l++) {
        const orc_layer *L = &m->layers[l];
        float *kc = k_cache + l * kv_cap * nkv, *vc = v_cache + l * kv_cap * nkv;
        orc_rmsnorm(xb, x, L->attn_norm, d, m->eps);
        rc |= orc_quant_matvec_par(q, L->wq, L->wq_type, xb, nq, d, scratch, pool);
        rc |= orc_quant_matvec_par(kn, L->wk, L->wk_type, xb, nkv, d, scratch, pool);
        rc |= orc_quant_matvec_par(vn, L->wv, L->wv_type, xb, nkv, d, scratch, pool);
        if (L->q_bias) for (size_t i = 0; i < nq; i++) q[i] += L->q_bias[i];
        if (L->k_bias) for (size_t i = 0; i < nkv; i++) kn[i] += L->k_bias[i];
        if (L->v_bias) for (size_t i = 0; i < nkv; i++) vn[i] += L->v_bias[i];
        if (L->q_norm) for (size_t h = 0; h < m->n_heads; h++) orc_rmsnorm(q + h * hd, q + h * hd, L->q_norm, hd, m->eps);
        if (L->k_norm) for (size_t h = 0; h < m->n_kv_heads; h++) orc_rmsnorm(kn + h * hd, kn + h * hd, L->k_norm, hd, m->eps);
        for (size_t h = 0; h < m->n_heads; h++) orc_rope(q + h * hd, hd, pos, m->rope_theta, m->rope_neox);
        for (size_t h = 0; h < m->n_kv_heads; h++) orc_rope(kn + h * hd, hd, pos, m->rope_theta, m->rope_neox);
        if (m->kv_f16)  /* an f16 cache returns the stored values rounded to nearest even */
            for (size_t i = 0; i < nkv; i++) {
                kn[i] = orc_f16_to_f32(orc_f32_to_f16(kn[i]));
                vn[i] = orc_f16_to_f32(orc_f32_to_f16(vn[i]));
            }
        memcpy(kc + pos * nkv, kn, nkv * 4);
        memcpy(vc + pos * nkv, vn, nkv * 4);
        for (size_t h = 0; h < m->n_heads; h++) {
            const size_t kvh = h / (m->n_heads / m->n_kv_heads);
            for (size_t s = 0; s < seq; s++) {
                memcpy(ks + s * hd, kc + s * nkv + kvh * hd, hd * 4);
                memcpy(vs + s * hd, vc + s * nkv + kvh * hd, hd * 4);
            }
            orc_sdp_attn(att + h * hd, q + h * hd, ks, vs, seq, hd, scale);
        }
        rc |= orc_quant_matvec_par(proj, L->wo, L->wo_type, att, d, nq, scratch, pool);
        for (size_t i = 0; i < d; i++) x[i] += proj[i];
        orc_rmsnorm(xb, x, L->ffn_norm, d, m->eps);
        if (L->router) {
            rc |= orc_moe_layer(fo, xb, 1, d, L->router, m->n_experts, m->k, m->norm_topk, NULL, L->e_gate, L->e_up,
                                L->e_gate_type, L->e_down, L->e_down_type, m->d_expert, 0, pool, NULL, NULL);
        } else {
            rc |= orc_quant_matvec_par(g, L->w_gate, L->ffn_gate_type, xb, ff, d, scratch, pool);
            rc |= orc_quant_matvec_par(u, L->w_up, L->ffn_gate_type, xb, ff, d, scratch, pool);
            for (size_t i = 0; i < ff; i++) g[i] = orc_silu(g[i]) * u[i];
            rc |= orc_quant_matvec_par(fo, L->w_down, L->ffn_down_type, g, d, ff, scratch, pool);
        }
        for (size_t i = 0; i < d; i++) x[i] += fo[i];
    }
    if (rc == 0) {
        orc_rmsnorm(xb, x, m->out_norm, d, m->eps);
        rc |= orc_quant_matvec_par(logits, m->lm_head, m->lm_type, xb, m->vocab, d, scratch, pool);
    }
    free(scratch); free(x); free(xb); free(q); free(kn); free(vn); free(att); free(ks); free(vs);
    free(proj); free(g); free(u); free(fo);
    return rc ? -1 : 0;
}

/* gemma4/forward.zig:37-567, CPU branches (see oracle.h) */
int orc_gemma_step(const orc_gemma *m, float *k_cache, float *v_cache, size_t global_cap, uint32_t token,
                   size_t pos, float *logits, orc_pool *pool) {
    const size_t d = m->d_model, seq = pos + 1, hdg = m->head_dim_global;
    if (token >= m->vocab) return -1;
    size_t max_hd = m->head_dim_swa > hdg ? m->head_dim_swa : hdg, max_nkv = 0;
    for (size_t l = 0; l < m->n_layers; l++) {
        const size_t hd = m->layers[l].is_swa ? m->head_dim_swa : hdg;
        if (m->layers[l].n_kv_heads * hd > max_nkv) max_nkv = m->layers[l].n_kv_heads * hd;
    }
    const size_t max_nq = m->n_heads * max_hd;
    size_t max_cols = d > max_nq ? d : max_nq;
    if (m->d_ffn > max_cols) max_cols = m->d_ffn;
    const size_t nthr = (size_t)orc_pool_threads(pool);
    float *scratch = (float *)malloc((nthr ? nthr : 1) * max_cols * 4);
    float *x = (float *)malloc(d * 4), *xb = (float *)malloc(d * 4), *attn_buf = (float *)malloc(d * 4);
    float *ffn = (float *)malloc(d * 4), *moe = (float *)malloc(d * 4), *moe_in = (float *)malloc(d * 4);
    float *router_in = (float *)malloc(d * 4), *scores = (float *)malloc(m->n_experts * 4);
    float *q = (float *)malloc(max_nq * 4), *kk = (float *)malloc(max_nkv * 4), *vv = (float *)malloc(max_nkv * 4);
    float *att = (float *)malloc(max_nq * 4);
    const size_t max_win = seq > m->sliding_window ? seq : m->sliding_window;
    float *ks = (float *)malloc(max_win * max_hd * 4), *vs = (float *)malloc(max_win * max_hd * 4);
    float *g = (float *)malloc(m->d_ffn * 4), *u = (float *)malloc(m->d_ffn * 4);
    float *eg = (float *)malloc(m->d_expert * 4), *eu = (float *)malloc(m->d_expert * 4), *ed = (float *)malloc(d * 4);
    float *freqs = (float *)malloc((hdg / 2) * 4);
    uint32_t top_idx[16];
    int rc = 0;
    if (m->k > 16) rc = -1;
    for (size_t i = 0; i < hdg / 2; i++)  /* loader.zig:225-233 fallback */
        freqs[i] = m->rope_freqs ? m->rope_freqs[i] : 1.0f / powf(1000000.0f, (float)(2 * i) / (float)hdg);
    if (rc == 0) rc = orc_dequant_row(m->token_emb + (size_t)token * orc_row_bytes(m->emb_type, d), x, d, m->emb_type);
    const float emb_scale = sqrtf((float)d);  /* forward.zig:117-120 */
    for (size_t i = 0; i < d; i++) x[i] *= emb_scale;
    size_t kv_off = 0;
    for (size_t l = 0; l < m->n_layers && rc == 0; l++) {
        const orc_gemma_layer *L = &m->layers[l];
        const size_t hd = L->is_swa ? m->head_dim_swa : hdg, nq = m->n_heads * hd, nkv = L->n_kv_heads * hd;
        const size_t cap = L->is_swa ? m->sliding_window : global_cap;
        float *kc = k_cache + kv_off, *vc = v_cache + kv_off;
        kv_off += cap * nkv;
        const size_t slot = pos % cap;
        const size_t win = L->is_swa ? (seq < m->sliding_window ? seq : m->sliding_window) : seq;
        orc_rmsnorm(xb, x, L->attn_norm, d, m->eps);
        rc |= orc_quant_matvec_par(q, L->wq, L->wq_type, xb, nq, d, scratch, pool);
        rc |= orc_quant_matvec_par(kk, L->wk, L->wk_type, xb, nkv, d, scratch, pool);
        if (L->wv)
            rc |= orc_quant_matvec_par(vv, L->wv, L->wv_type, xb, nkv, d, scratch, pool);
        else
            memcpy(vv, kk, nkv * 4);
        for (size_t h = 0; h < m->n_heads; h++) orc_rmsnorm(q + h * hd, q + h * hd, L->q_norm, hd, m->eps);
        for (size_t h = 0; h < L->n_kv_heads; h++) orc_rmsnorm(kk + h * hd, kk + h * hd, L->k_norm, hd, m->eps);
        for (size_t h = 0; h < L->n_kv_heads; h++) orc_rmsnorm_raw(vv + h * hd, vv + h * hd, hd, m->eps);
        if (L->is_swa) {
            for (size_t h = 0; h < m->n_heads; h++) orc_rope(q + h * hd, hd, pos, m->rope_theta_swa, 1);
            for (size_t h = 0; h < L->n_kv_heads; h++) orc_rope(kk + h * hd, hd, pos, m->rope_theta_swa, 1);
        } else {  /* rope.zig:78-94, applyRopeFreqsNeox */
            float *vecs[2] = {q, kk};
            const size_t nh[2] = {m->n_heads, L->n_kv_heads};
            for (int w = 0; w < 2; w++)
                for (size_t h = 0; h < nh[w]; h++) {
                    float *v = vecs[w] + h * hd;
                    const size_t half = hd / 2;
                    for (size_t i = 0; i < half; i++) {
                        const float angle = (float)pos * freqs[i];
                        const float c = cosf(angle), sn = sinf(angle);
                        const float x0 = v[i], x1 = v[i + half];
                        v[i] = x0 * c - x1 * sn;
                        v[i + half] = x0 * sn + x1 * c;
                    }
                }
        }
        memcpy(kc + slot * nkv, kk, nkv * 4);
        memcpy(vc + slot * nkv, vv, nkv * 4);
        for (size_t h = 0; h < m->n_heads; h++) {  /* forward.zig:306-327 */
            const size_t kvh = h / (m->n_heads / L->n_kv_heads);
            for (size_t wi = 0; wi < win; wi++) {
                const size_t s2 = ((seq - win) + wi) % cap;
                memcpy(ks + wi * hd, kc + s2 * nkv + kvh * hd, hd * 4);
                memcpy(vs + wi * hd, vc + s2 * nkv + kvh * hd, hd * 4);
            }
            orc_sdp_attn(att + h * hd, q + h * hd, ks, vs, win, hd, 1.0f);
        }
        rc |= orc_quant_matvec_par(attn_buf, L->wo, L->wo_type, att, d, nq, scratch, pool);
        orc_rmsnorm(attn_buf, attn_buf, L->post_attention_norm, d, m->eps);
        for (size_t i = 0; i < d; i++) x[i] += attn_buf[i];
        /* dense GeGLU FFN (:390-396) */
        orc_rmsnorm(xb, x, L->ffn_norm, d, m->eps);
        rc |= orc_quant_matvec_par(g, L->w_gate, L->gate_type, xb, m->d_ffn, d, scratch, pool);
        rc |= orc_quant_matvec_par(u, L->w_up, L->up_type, xb, m->d_ffn, d, scratch, pool);
        for (size_t i = 0; i < m->d_ffn; i++) g[i] = orc_gelu(g[i]) * u[i];
        rc |= orc_quant_matvec_par(ffn, L->w_down, L->down_type, g, d, m->d_ffn, scratch, pool);
        orc_rmsnorm(ffn, ffn, L->post_ffw_norm_1, d, m->eps);
        /* MoE (:401-494): math.zig:51-82 then routerTopKSoftmax and the expert loop */
        {
            float ss = 0.0f;
            for (size_t i = 0; i < d; i++) ss += x[i] * x[i];
            const float rms_inv = 1.0f / sqrtf(ss / (float)d + m->eps);
            const float raw_base = rms_inv * (1.0f / sqrtf((float)d));
            for (size_t i = 0; i < d; i++) {
                moe_in[i] = x[i] * rms_inv * L->pre_ffw_norm_2[i];
                router_in[i] = x[i] * raw_base * L->router_scale[i];
            }
        }
        orc_router_topk_softmax(scores, top_idx, m->k, L->router_w, m->n_experts, d, router_in, pool);
        memset(moe, 0, d * 4);
        const size_t gu_rb = orc_row_bytes(L->gu_type, d), dn_rb = orc_row_bytes(L->dn_type, m->d_expert);
        for (size_t i = 0; i < m->k; i++) {
            const uint32_t e = top_idx[i];
            const uint8_t *gd = L->gate_up_exps + (size_t)e * 2 * m->d_expert * gu_rb;
            rc |= orc_quant_matvec_par(eg, gd, L->gu_type, moe_in, m->d_expert, d, scratch, pool);
            rc |= orc_quant_matvec_par(eu, gd + m->d_expert * gu_rb, L->gu_type, moe_in, m->d_expert, d, scratch, pool);
            for (size_t r = 0; r < m->d_expert; r++) eg[r] = orc_gelu(eg[r]) * eu[r];
            rc |= orc_quant_matvec_par(ed, L->down_exps + (size_t)e * d * dn_rb, L->dn_type, eg, d, m->d_expert,
                                       scratch, pool);
            const float es = L->down_exps_scale[e] * scores[e];
            for (size_t r = 0; r < d; r++) moe[r] += es * ed[r];
        }
        orc_rmsnorm(moe, moe, L->post_ffw_norm_2, d, m->eps);
        for (size_t i = 0; i < d; i++) ffn[i] += moe[i];
        orc_rmsnorm(ffn, ffn, L->post_ffw_norm, d, m->eps);
        for (size_t i = 0; i < d; i++) x[i] += ffn[i];
        if (L->layer_output_scale != 1.0f)
            for (size_t i = 0; i < d; i++) x[i] *= L->layer_output_scale;
    }
    if (rc == 0) {
        orc_rmsnorm(xb, x, m->out_norm, d, m->eps);
        rc |= orc_quant_matvec_par(logits, m->lm_head, m->lm_type, xb, m->vocab, d, scratch, pool);
        if (m->logit_softcap != 0.0f)
            for (size_t i = 0; i < m->vocab; i++) logits[i] = tanhf(logits[i] / m->logit_softcap) * m->logit_softcap;
    }
    free(scratch); free(x); free(xb); free(attn_buf); free(ffn); free(moe); free(moe_in); free(router_in);
    free(scores); free(q); free(kk); free(vv); free(att); free(ks); free(vs); free(g); free(u); free(eg); free(eu);
    free(ed); free(freqs);
    return rc ? -1 : 0;
}

/* ── sampling (sample.zig:27-183) ─────────────────────────────────────────── */

static uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

/* SplitMix64 (Vigna), the seeding of std.Random.Xoshiro256 */
void orc_rng_seed(orc_rng *r, uint64_t seed) {
    uint64_t st = seed;
    for (int i = 0; i < 4; i++) {
        st += 0x9e3779b97f4a7c15ull;
        uint64_t z = st;
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        r->s[i] = z ^ (z >> 31);
    }
}

/* xoshiro256++ (Blackman & Vigna) */
static uint64_t rng_next(orc_rng *r) {
    uint64_t *s = r->s;
    const uint64_t res = rotl64(s[0] + s[3], 23) + s[0];
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
    return res;
}

static int clz64(uint64_t v) { return v ? __builtin_clzll(v) : 64; }

/* Random.float(f32): 23 random mantissa bits, an exponentially distributed
 * exponent from the leading zeros of the rest */
float orc_rng_float(orc_rng *r) {
    const uint64_t rnd = rng_next(r);
    int lz = clz64(rnd);
    if (lz >= 41) {
        lz = 41 + clz64(rng_next(r));
        if (lz == 41 + 64) lz += __builtin_clz((uint32_t)rng_next(r) | 0x7FFu);
    }
    const uint32_t bits = ((uint32_t)(126 - lz) << 23) | ((uint32_t)rnd & 0x7FFFFFu);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

typedef struct { uint32_t idx; float val; } orc_cand;

static int cmp_desc_f32(const void *a, const void *b) {
    const float x = *(const float *)a, y = *(const float *)b;
    return x > y ? -1 : x < y ? 1 : 0;
}

static const float *g_sort_probs;
static int cmp_idx_desc(const void *a, const void *b) {
    const size_t i = *(const size_t *)a, j = *(const size_t *)b;
    const float x = g_sort_probs[i], y = g_sort_probs[j];
    if (x > y) return -1;
    if (x < y) return 1;
    return i < j ? -1 : i > j ? 1 : 0;
}

uint32_t orc_sample(float *logits, size_t n, float temperature, uint32_t top_k, float top_p, orc_rng *rng) {
    if (temperature == 0.0f) return orc_greedy(logits, n);
    if (temperature != 1.0f) {
        const float inv_t = 1.0f / temperature;
        for (size_t i = 0; i < n; i++) logits[i] *= inv_t;
    }
    if (top_k > 0 && top_k < n && top_k <= 256) {  /* sampleTopK, sample.zig:82-145 */
        orc_cand c[256];
        size_t filled = 0;
        const size_t k = top_k;
        float max_logit = logits[0], exp_sum = 0.0f;
        for (size_t i = 0; i < n; i++) {
            const float logit = logits[i];
            if (logit > max_logit) {
                exp_sum = exp_sum * expf(max_logit - logit) + 1.0f;
                max_logit = logit;
            } else {
                exp_sum += expf(logit - max_logit);
            }
            if (filled < k) {
                size_t pos = filled++;
                while (pos > 0 && logit > logits[c[pos - 1].idx]) { c[pos] = c[pos - 1]; pos--; }
                c[pos].idx = (uint32_t)i;
                c[pos].val = logit;
            } else if (logit > logits[c[k - 1].idx]) {
                size_t pos = k - 1;
                while (pos > 0 && logit > logits[c[pos - 1].idx]) { c[pos] = c[pos - 1]; pos--; }
                c[pos].idx = (uint32_t)i;
                c[pos].val = logit;
            }
        }
        for (size_t i = 0; i < k; i++) c[i].val = expf(c[i].val - max_logit) / exp_sum;
        size_t kept = k;
        if (top_p < 1.0f) {
            float cum = 0.0f;
            for (size_t i = 0; i < k; i++) {
                cum += c[i].val;
                if (cum >= top_p) { kept = i + 1; break; }
            }
        }
        float kept_sum = 0.0f;
        for (size_t i = 0; i < kept; i++) kept_sum += c[i].val;
        if (kept_sum <= 0.0f) return c[0].idx;
        const float r = orc_rng_float(rng) * kept_sum;
        float cum = 0.0f;
        for (size_t i = 0; i < kept; i++) {
            cum += c[i].val;
            if (r <= cum) return c[i].idx;
        }
        return c[kept - 1].idx;
    }
    orc_softmax(logits, n);
    if (top_k > 0 && top_k < n) {  /* applyTopK, sample.zig:147-155 */
        float *tmp = (float *)malloc(n * 4);
        memcpy(tmp, logits, n * 4);
        qsort(tmp, n, 4, cmp_desc_f32);
        const float thr = tmp[(top_k < n ? top_k : n) - 1];
        for (size_t i = 0; i < n; i++)
            if (logits[i] < thr) logits[i] = 0.0f;
        free(tmp);
    }
    if (top_p < 1.0f) {  /* applyTopP, sample.zig:157-178 */
        size_t *idx = (size_t *)malloc(n * sizeof(size_t));
        for (size_t i = 0; i < n; i++) idx[i] = i;
        g_sort_probs = logits;
        qsort(idx, n, sizeof(size_t), cmp_idx_desc);
        float cum = 0.0f;
        int cutoff = 0;
        for (size_t j = 0; j < n; j++) {
            if (cutoff) {
                logits[idx[j]] = 0.0f;
            } else {
                cum += logits[idx[j]];
                if (cum >= top_p) cutoff = 1;
            }
        }
        free(idx);
    }
    float sum = 0.0f;  /* renormalize, sample.zig:180-187 */
    for (size_t i = 0; i < n; i++) sum += logits[i];
    if (sum > 0.0f) {
        const float inv = 1.0f / sum;
        for (size_t i = 0; i < n; i++) logits[i] *= inv;
    }
    const float r = orc_rng_float(rng);
    float cum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        cum += logits[i];
        if (r <= cum) return (uint32_t)i;
    }
    return (uint32_t)(n - 1);
}
