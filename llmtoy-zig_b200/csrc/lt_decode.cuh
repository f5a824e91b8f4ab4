// lt_decode.cuh — GGUF block decoders that take dot products against
// quantised activations held in shared memory.
//
// Activations.  Each 16-element group of an activation row is stored as
// x ~= s * (hi + lo / 254) with s = amax / 32767: hi = round(x / s) as int16
// and lo = round of the remainder in 1/254 steps as int8 -- about 2^-24 of the
// block's range, f32-like.  Products with the quant values (4-8 bit integers)
// accumulate exactly in int32: hi via dp2a (2 elements per instruction), lo
// via dp4a (4 per instruction).  The only rounding left is the f32 scale
// arithmetic.  (A single int16 term loses too much when expert outputs
// cancel in the weighted combine: measured 3e-4 relative error.)
//
// Shared-memory layout per token t and item i (256 columns): hi at
// xq + t*tok_hi + i*528, lo at xl + t*tok_lo + i*272; the 16 padding bytes
// per item put threads that decode different items in different banks.  Per
// 16-group: scale xs and the f32 sum of the original values xsum16 (used for
// the Q4_K minimum and the Q6_K -32 offset terms, applied in f32).
#pragma once

#include "lt_common.cuh"

namespace lt {

constexpr int kXHiPitch = 528;  // 256 int16 + 16 bytes of padding
constexpr int kXLoPitch = 272;  // 256 int8 + 16 bytes of padding
constexpr float kLoScale = 1.0f / 254.0f;

struct XS {
    uint8_t *xq;    // hi terms
    uint8_t *xl;    // lo terms
    float *xs;      // [t][item*16 + group] scale
    float *xsum16;  // [t][item*16 + group] sum of x over 16 elements
    int nitems;
    int tok_hi;  // nitems * 528
    int tok_lo;  // nitems * 272
    int tok_g;   // nitems * 16
};

__host__ __device__ inline size_t xs_bytes(int ntok, int nitems) {
    return (size_t)ntok * nitems * (kXHiPitch + kXLoPitch + 16 * 4 + 16 * 4);
}

LT_DEVINL XS xs_carve(uint8_t *p, int ntok, int nitems) {
    XS x;
    x.nitems = nitems;
    x.tok_hi = nitems * kXHiPitch;
    x.tok_lo = nitems * kXLoPitch;
    x.tok_g = nitems * 16;
    x.xq = p;
    p += (size_t)ntok * x.tok_hi;
    x.xl = p;
    p += (size_t)ntok * x.tok_lo;
    x.xs = reinterpret_cast<float *>(p);
    p += (size_t)ntok * nitems * 16 * 4;
    x.xsum16 = reinterpret_cast<float *>(p);
    return x;
}

// 32 consecutive activation values: hi terms as 16 int16 pairs, lo terms as
// 8 words of 4 int8.
LT_DEVINL void load_x32(const XS &X, int t, int item, int elem0, uint32_t (&hi)[16], uint32_t (&lo)[8]) {
    const uint8_t *ph = X.xq + (size_t)t * X.tok_hi + item * kXHiPitch + 2 * elem0;
    const uint8_t *pl = X.xl + (size_t)t * X.tok_lo + item * kXLoPitch + elem0;
#pragma unroll
    for (int v = 0; v < 4; v++) {
        const uint4 h4 = lds128(ph + 16 * v);
        hi[4 * v] = h4.x; hi[4 * v + 1] = h4.y; hi[4 * v + 2] = h4.z; hi[4 * v + 3] = h4.w;
    }
#pragma unroll
    for (int v = 0; v < 2; v++) {
        const uint4 l4 = lds128(pl + 16 * v);
        lo[4 * v] = l4.x; lo[4 * v + 1] = l4.y; lo[4 * v + 2] = l4.z; lo[4 * v + 3] = l4.w;
    }
}

// sums over 32 elements of q * x_hi and q * x_lo for quant bytes q[8] (4 per
// word, unsigned), kept per 16-element half (each half has its own scale).
LT_DEVINL void dot32_u(const uint32_t (&q)[8], const uint32_t (&xh)[16], const uint32_t (&xl)[8], int (&hi)[2],
                       int (&lo)[2]) {
    int h0 = 0, h1 = 0, l0 = 0, l1 = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        h0 = dp2a_hi_su((int)xh[2 * k + 1], q[k], dp2a_lo_su((int)xh[2 * k], q[k], h0));
        h1 = dp2a_hi_su((int)xh[2 * k + 9], q[k + 4], dp2a_lo_su((int)xh[2 * k + 8], q[k + 4], h1));
        l0 = dp4a_su((int)xl[k], q[k], l0);
        l1 = dp4a_su((int)xl[k + 4], q[k + 4], l1);
    }
    hi[0] = h0; hi[1] = h1;
    lo[0] = l0; lo[1] = l1;
}

// Same with signed quant bytes (Q8_0).
LT_DEVINL void dot32_s(const uint32_t (&q)[8], const uint32_t (&xh)[16], const uint32_t (&xl)[8], int (&hi)[2],
                       int (&lo)[2]) {
    int h0 = 0, h1 = 0, l0 = 0, l1 = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        h0 = dp2a_hi_ss((int)xh[2 * k + 1], q[k], dp2a_lo_ss((int)xh[2 * k], q[k], h0));
        h1 = dp2a_hi_ss((int)xh[2 * k + 9], q[k + 4], dp2a_lo_ss((int)xh[2 * k + 8], q[k + 4], h1));
        l0 = dp4a_ss((int)xl[k], q[k], l0);
        l1 = dp4a_ss((int)xl[k + 4], q[k + 4], l1);
    }
    hi[0] = h0; hi[1] = h1;
    lo[0] = l0; lo[1] = l1;
}

LT_DEVINL float qx(int hi, int lo) { return (float)hi + (float)lo * kLoScale; }

// ── Q4_K superblock: [f16 d][f16 dmin][12 B 6-bit scales/mins][128 B nibbles] ──
template <int NT>
LT_DEVINL void dot_q4k(const uint8_t *sbp, int item, const XS &X, int t0, int nt, float (&res)[NT]) {
    const uint4 hdr = lds128(sbp);
    const float d = f16_bits_to_f32(hdr.x), dmin = f16_bits_to_f32(hdr.x >> 16);
    // scale_min (src/quant/dequant.zig:291-300) for sub-blocks 0-3 and 4-7, one byte each
    const uint32_t sc_lo = hdr.y & 0x3F3F3F3Fu, mn_lo = hdr.z & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
    const uint32_t mn_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint32_t scw = c < 2 ? sc_lo : sc_hi, mnw = c < 2 ? mn_lo : mn_hi;
        const int j0 = (2 * c) & 3, j1 = (2 * c + 1) & 3;
        const float dA = d * byte_to_f32(scw, j0), mA = dmin * byte_to_f32(mnw, j0);
        const float dB = d * byte_to_f32(scw, j1), mB = dmin * byte_to_f32(mnw, j1);
        const uint4 qa = lds128(sbp + 16 + 32 * c), qb = lds128(sbp + 32 + 32 * c);
        const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        uint32_t lo[8], hi[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            lo[k] = w[k] & 0x0F0F0F0Fu;          // elements 64c + 4k.. (sub-block 2c)
            hi[k] = (w[k] >> 4) & 0x0F0F0F0Fu;   // elements 64c + 32 + 4k.. (sub-block 2c+1)
        }
#pragma unroll
        for (int tt = 0; tt < NT; tt++) {
            if (tt < nt) {
                const int t = t0 + tt;
                uint32_t ah[16], al[8], bh[16], bl[8];
                load_x32(X, t, item, 64 * c, ah, al);
                load_x32(X, t, item, 64 * c + 32, bh, bl);
                int aH[2], aL[2], bH[2], bL[2];
                dot32_u(lo, ah, al, aH, aL);
                dot32_u(hi, bh, bl, bH, bL);
                const float *xs = X.xs + t * X.tok_g + item * 16 + 4 * c;
                const float *x16 = X.xsum16 + t * X.tok_g + item * 16 + 4 * c;
                res[tt] += dA * (xs[0] * qx(aH[0], aL[0]) + xs[1] * qx(aH[1], aL[1])) - mA * (x16[0] + x16[1]);
                res[tt] += dB * (xs[2] * qx(bH[0], bL[0]) + xs[3] * qx(bH[1], bL[1])) - mB * (x16[2] + x16[3]);
            }
        }
    }
}

// 4 bytes starting at static byte offset O of a word array.
template <int O>
LT_DEVINL uint32_t word_at(const uint32_t *w) {
    if constexpr ((O & 3) == 0) {
        return w[O >> 2];
    } else {
        return __byte_perm(w[O >> 2], w[(O >> 2) + 1],
                           (uint32_t)(((O & 3) + 3) << 12 | ((O & 3) + 2) << 8 | ((O & 3) + 1) << 4 | (O & 3)));
    }
}

template <int B, int NT>
LT_DEVINL void dot_q8_block(const uint32_t *w, int item, const XS &X, int t0, int nt, float (&res)[NT]) {
    const float d = f16_bits_to_f32(word_at<34 * B>(w) & 0xffffu);
    uint32_t q[8];
    q[0] = word_at<34 * B + 2>(w);
    q[1] = word_at<34 * B + 6>(w);
    q[2] = word_at<34 * B + 10>(w);
    q[3] = word_at<34 * B + 14>(w);
    q[4] = word_at<34 * B + 18>(w);
    q[5] = word_at<34 * B + 22>(w);
    q[6] = word_at<34 * B + 26>(w);
    q[7] = word_at<34 * B + 30>(w);
#pragma unroll
    for (int tt = 0; tt < NT; tt++) {
        if (tt < nt) {
            const int t = t0 + tt;
            uint32_t xh[16], xl[8];
            load_x32(X, t, item, 32 * B, xh, xl);
            int h[2], l[2];
            dot32_s(q, xh, xl, h, l);
            const float *xs = X.xs + t * X.tok_g + item * 16 + 2 * B;
            res[tt] += d * (xs[0] * qx(h[0], l[0]) + xs[1] * qx(h[1], l[1]));
        }
    }
}

// Q8_0 group of eight 34-byte blocks (272 B, 16-byte aligned); nb < 8 only
// for the last group of a row whose block count is not a multiple of 8.
template <int NT>
LT_DEVINL void dot_q8_0(const uint8_t *gp, int item, int nb, const XS &X, int t0, int nt, float (&res)[NT]) {
    uint32_t w[68];
#pragma unroll
    for (int i = 0; i < 17; i++) {
        const uint4 v = lds128(gp + 16 * i);
        w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
    }
    dot_q8_block<0>(w, item, X, t0, nt, res);
    if (nb > 1) dot_q8_block<1>(w, item, X, t0, nt, res);
    if (nb > 2) dot_q8_block<2>(w, item, X, t0, nt, res);
    if (nb > 3) dot_q8_block<3>(w, item, X, t0, nt, res);
    if (nb > 4) dot_q8_block<4>(w, item, X, t0, nt, res);
    if (nb > 5) dot_q8_block<5>(w, item, X, t0, nt, res);
    if (nb > 6) dot_q8_block<6>(w, item, X, t0, nt, res);
    if (nb > 7) dot_q8_block<7>(w, item, X, t0, nt, res);
}

// Q6_K superblock (210 B, only 2-byte aligned): [ql 128][qh 64][i8 sc 16][f16 d].
// Words are read 4-byte aligned and realigned with one PRMT each.
template <int NT>
LT_DEVINL void dot_q6k(const uint8_t *sbp, int item, const XS &X, int t0, int nt, float (&res)[NT]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(sbp);
    const uint8_t *pa = reinterpret_cast<const uint8_t *>(a & ~(uintptr_t)3);
    const uint32_t sel = (a & 2) ? 0x5432u : 0x3210u;
    uint32_t rs[6];
#pragma unroll
    for (int i = 0; i < 6; i++) rs[i] = lds32(pa + 4 * (48 + i));
    uint32_t scw[4];
#pragma unroll
    for (int i = 0; i < 4; i++) scw[i] = __byte_perm(rs[i], rs[i + 1], sel);
    const float d = f16_bits_to_f32(__byte_perm(rs[4], rs[5], sel) & 0xffffu);
#pragma unroll
    for (int n = 0; n < 2; n++) {
        uint32_t rq[17], rh[9];
#pragma unroll
        for (int i = 0; i < 17; i++) rq[i] = lds32(pa + 4 * (16 * n + i));
#pragma unroll
        for (int i = 0; i < 9; i++) rh[i] = lds32(pa + 4 * (32 + 8 * n + i));
        uint32_t qv[4][8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const uint32_t qlA = __byte_perm(rq[k], rq[k + 1], sel);
            const uint32_t qlB = __byte_perm(rq[8 + k], rq[9 + k], sel);
            const uint32_t h = __byte_perm(rh[k], rh[k + 1], sel);
            qv[0][k] = (qlA & 0x0F0F0F0Fu) | ((h << 4) & 0x30303030u);          // 128n + l
            qv[1][k] = (qlB & 0x0F0F0F0Fu) | ((h << 2) & 0x30303030u);          // 128n + 32 + l
            qv[2][k] = ((qlA >> 4) & 0x0F0F0F0Fu) | (h & 0x30303030u);          // 128n + 64 + l
            qv[3][k] = ((qlB >> 4) & 0x0F0F0F0Fu) | ((h >> 2) & 0x30303030u);   // 128n + 96 + l
        }
#pragma unroll
        for (int kind = 0; kind < 4; kind++) {
            // i8 scales for l in [0,16) and [16,32): sc[8n + is + 2*kind]
            const int s0 = 8 * n + 2 * kind, s1 = s0 + 1;
            const float ds0 = d * (float)(int8_t)((scw[s0 >> 2] >> (8 * (s0 & 3))) & 0xffu);
            const float ds1 = d * (float)(int8_t)((scw[s1 >> 2] >> (8 * (s1 & 3))) & 0xffu);
#pragma unroll
            for (int tt = 0; tt < NT; tt++) {
                if (tt < nt) {
                    const int t = t0 + tt;
                    uint32_t xh[16], xl[8];
                    load_x32(X, t, item, 128 * n + 32 * kind, xh, xl);
                    // the two 16-element halves carry different scales
                    int h0 = 0, l0 = 0, h1 = 0, l1 = 0;
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        h0 = dp2a_hi_su((int)xh[2 * k + 1], qv[kind][k], dp2a_lo_su((int)xh[2 * k], qv[kind][k], h0));
                        l0 = dp4a_su((int)xl[k], qv[kind][k], l0);
                        h1 = dp2a_hi_su((int)xh[9 + 2 * k], qv[kind][4 + k],
                                        dp2a_lo_su((int)xh[8 + 2 * k], qv[kind][4 + k], h1));
                        l1 = dp4a_su((int)xl[4 + k], qv[kind][4 + k], l1);
                    }
                    const int g = 8 * n + 2 * kind;  // 16-group index inside the item
                    const float *x16 = X.xsum16 + t * X.tok_g + item * 16;
                    const float *xs = X.xs + t * X.tok_g + item * 16;
                    // sum (q - 32) x = s * sum q*xq - 32 * sum x
                    res[tt] += ds0 * (xs[g] * qx(h0, l0) - 32.0f * x16[g]);
                    res[tt] += ds1 * (xs[g + 1] * qx(h1, l1) - 32.0f * x16[g + 1]);
                }
            }
        }
    }
}

// ── 32-element block formats with a fifth bit (Q5_0, Q5_1) or a table (IQ4_NL).
// An item is eight consecutive blocks (176 / 192 / 144 bytes, so it starts
// 16-byte aligned); it is read as words and each block's fields are taken at
// static byte offsets.

// Bits 0..3 of v to bit 4 of bytes 0..3.
LT_DEVINL uint32_t hbit4(uint32_t v) {
    return ((v & 1u) | ((v & 2u) << 7) | ((v & 4u) << 14) | ((v & 8u) << 21)) << 4;
}

// The 32 five-bit values of a Q5_0 / Q5_1 block (nibbles qs[0..16): low
// nibble = element j, high nibble = element j + 16; bit e of qh is element
// e's fifth bit), elements 4k..4k+3 in q[k].
LT_DEVINL void q5_values(const uint32_t (&qs)[4], uint32_t qh, uint32_t (&q)[8]) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
        q[k] = (qs[k] & 0x0F0F0F0Fu) | hbit4(qh >> (4 * k));
        q[k + 4] = ((qs[k] >> 4) & 0x0F0F0F0Fu) | hbit4(qh >> (16 + 4 * k));
    }
}

// FMT 0: Q5_0 (22 B: d, qh, qs; value d * (q - 16), dequant.zig:201-217)
// FMT 1: Q5_1 (24 B: d, m, qh, qs; value d * q + m, dequant.zig:469-487)
// FMT 2: IQ4_NL (18 B: d, qs; value d * table[nibble], dequant.zig:623-640)
template <int FMT, int B, int NT>
LT_DEVINL void dot_b32_block(const uint32_t *w, int item, const XS &X, int t0, int nt, float (&res)[NT]) {
    constexpr int BB = FMT == 0 ? 22 : FMT == 1 ? 24 : 18;
    constexpr int O = BB * B;
    const uint32_t w0 = word_at<O>(w);
    const float d = f16_bits_to_f32(w0 & 0xffffu);
    uint32_t q[8];
    if constexpr (FMT == 2) {
        const uint32_t qs[4] = {word_at<O + 2>(w), word_at<O + 6>(w), word_at<O + 10>(w), word_at<O + 14>(w)};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            q[k] = iq4nl_lookup4(qs[k] & 0x0F0F0F0Fu);
            q[k + 4] = iq4nl_lookup4((qs[k] >> 4) & 0x0F0F0F0Fu);
        }
    } else {
        constexpr int OH = FMT == 0 ? O + 2 : O + 4, OQ = OH + 4;
        const uint32_t qs[4] = {word_at<OQ>(w), word_at<OQ + 4>(w), word_at<OQ + 8>(w), word_at<OQ + 12>(w)};
        q5_values(qs, word_at<OH>(w), q);
    }
#pragma unroll
    for (int tt = 0; tt < NT; tt++) {
        if (tt < nt) {
            const int t = t0 + tt;
            uint32_t xh[16], xl[8];
            load_x32(X, t, item, 32 * B, xh, xl);
            int h[2], l[2];
            const float *xs = X.xs + t * X.tok_g + item * 16 + 2 * B;
            const float *x16 = X.xsum16 + t * X.tok_g + item * 16 + 2 * B;
            if constexpr (FMT == 2) {
                dot32_s(q, xh, xl, h, l);
                res[tt] += d * (xs[0] * qx(h[0], l[0]) + xs[1] * qx(h[1], l[1]));
            } else {
                dot32_u(q, xh, xl, h, l);
                if constexpr (FMT == 0) {  // sum (q - 16) x = s * sum q*xq - 16 * sum x
                    res[tt] += d * ((xs[0] * qx(h[0], l[0]) - 16.0f * x16[0]) + (xs[1] * qx(h[1], l[1]) - 16.0f * x16[1]));
                } else {
                    const float m = f16_bits_to_f32(w0 >> 16);
                    res[tt] += d * (xs[0] * qx(h[0], l[0]) + xs[1] * qx(h[1], l[1])) + m * (x16[0] + x16[1]);
                }
            }
        }
    }
}

template <int FMT, int NT>
LT_DEVINL void dot_b32(const uint8_t *gp, int item, int nb, const XS &X, int t0, int nt, float (&res)[NT]) {
    constexpr int NW = (FMT == 0 ? 176 : FMT == 1 ? 192 : 144) / 4;
    uint32_t w[NW];
#pragma unroll
    for (int i = 0; i < NW / 4; i++) {
        const uint4 v = lds128(gp + 16 * i);
        w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
    }
    dot_b32_block<FMT, 0>(w, item, X, t0, nt, res);
    if (nb > 1) dot_b32_block<FMT, 1>(w, item, X, t0, nt, res);
    if (nb > 2) dot_b32_block<FMT, 2>(w, item, X, t0, nt, res);
    if (nb > 3) dot_b32_block<FMT, 3>(w, item, X, t0, nt, res);
    if (nb > 4) dot_b32_block<FMT, 4>(w, item, X, t0, nt, res);
    if (nb > 5) dot_b32_block<FMT, 5>(w, item, X, t0, nt, res);
    if (nb > 6) dot_b32_block<FMT, 6>(w, item, X, t0, nt, res);
    if (nb > 7) dot_b32_block<FMT, 7>(w, item, X, t0, nt, res);
}

// ── Q5_K superblock (176 B): Q4_K's header and nibbles plus qh[32], whose bit
// 2c (2c + 1) is the fifth bit of chunk c's low (high) nibbles
// (dequant.zig:324-367).
template <int NT>
LT_DEVINL void dot_q5k(const uint8_t *sbp, int item, const XS &X, int t0, int nt, float (&res)[NT]) {
    const uint4 hdr = lds128(sbp);
    const float d = f16_bits_to_f32(hdr.x), dmin = f16_bits_to_f32(hdr.x >> 16);
    const uint32_t sc_lo = hdr.y & 0x3F3F3F3Fu, mn_lo = hdr.z & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
    const uint32_t mn_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
    const uint4 h0 = lds128(sbp + 16), h1 = lds128(sbp + 32);
    const uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint32_t scw = c < 2 ? sc_lo : sc_hi, mnw = c < 2 ? mn_lo : mn_hi;
        const int j0 = (2 * c) & 3, j1 = (2 * c + 1) & 3;
        const float dA = d * byte_to_f32(scw, j0), mA = dmin * byte_to_f32(mnw, j0);
        const float dB = d * byte_to_f32(scw, j1), mB = dmin * byte_to_f32(mnw, j1);
        const uint4 qa = lds128(sbp + 48 + 32 * c), qb = lds128(sbp + 64 + 32 * c);
        const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        uint32_t lo[8], hi[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            lo[k] = (w[k] & 0x0F0F0F0Fu) | (((qh[k] >> (2 * c)) & 0x01010101u) << 4);
            hi[k] = ((w[k] >> 4) & 0x0F0F0F0Fu) | (((qh[k] >> (2 * c + 1)) & 0x01010101u) << 4);
        }
#pragma unroll
        for (int tt = 0; tt < NT; tt++) {
            if (tt < nt) {
                const int t = t0 + tt;
                uint32_t ah[16], al[8], bh[16], bl[8];
                load_x32(X, t, item, 64 * c, ah, al);
                load_x32(X, t, item, 64 * c + 32, bh, bl);
                int aH[2], aL[2], bH[2], bL[2];
                dot32_u(lo, ah, al, aH, aL);
                dot32_u(hi, bh, bl, bH, bL);
                const float *xs = X.xs + t * X.tok_g + item * 16 + 4 * c;
                const float *x16 = X.xsum16 + t * X.tok_g + item * 16 + 4 * c;
                res[tt] += dA * (xs[0] * qx(aH[0], aL[0]) + xs[1] * qx(aH[1], aL[1])) - mA * (x16[0] + x16[1]);
                res[tt] += dB * (xs[2] * qx(bH[0], bL[0]) + xs[3] * qx(bH[1], bL[1])) - mB * (x16[2] + x16[3]);
            }
        }
    }
}

// ── Q3_K superblock (110 B, only 2-byte aligned): [hmask 32][qs 64][scales 12][f16 d].
// Unit (h, j) = elements 128h + 32j + [0, 32): two low bits (qs byte
// 32h + e >> 2j), the third from hmask byte e bit 4h + j, value
// (low | third << 2) - 4; 16-element groups carry 6-bit scales minus 32
// (dequant.zig:388-464).
template <int NT>
LT_DEVINL void dot_q3k(const uint8_t *sbp, int item, const XS &X, int t0, int nt, float (&res)[NT]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(sbp);
    const uint8_t *pa = reinterpret_cast<const uint8_t *>(a & ~(uintptr_t)3);
    const uint32_t sel = (a & 2) ? 0x5432u : 0x3210u;
    uint32_t r[29];
#pragma unroll
    for (int i = 0; i < 29; i++) r[i] = lds32(pa + 4 * i);
    auto W = [&](int i) { return __byte_perm(r[i], r[i + 1], sel); };
    const uint32_t a0 = W(24), a1 = W(25), tmp = W(26);
    uint32_t scw[4];
    scw[0] = (a0 & 0x0F0F0F0Fu) | ((tmp & 0x03030303u) << 4);
    scw[1] = (a1 & 0x0F0F0F0Fu) | (((tmp >> 2) & 0x03030303u) << 4);
    scw[2] = ((a0 >> 4) & 0x0F0F0F0Fu) | (((tmp >> 4) & 0x03030303u) << 4);
    scw[3] = ((a1 >> 4) & 0x0F0F0F0Fu) | (((tmp >> 6) & 0x03030303u) << 4);
    const float d = f16_bits_to_f32(W(27) & 0xffffu);
    uint32_t hm[8];
#pragma unroll
    for (int m = 0; m < 8; m++) hm[m] = W(m);
#pragma unroll
    for (int h = 0; h < 2; h++) {
        uint32_t qs[8];
#pragma unroll
        for (int m = 0; m < 8; m++) qs[m] = W(8 + 8 * h + m);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint32_t q[8];
#pragma unroll
            for (int m = 0; m < 8; m++)
                q[m] = ((qs[m] >> (2 * j)) & 0x03030303u) | (((hm[m] >> (4 * h + j)) & 0x01010101u) << 2);
            const int g = 8 * h + 2 * j;  // scale index = 16-group index inside the item
            const float dl0 = d * ((float)((scw[g >> 2] >> (8 * (g & 3))) & 0xffu) - 32.0f);
            const float dl1 = d * ((float)((scw[(g + 1) >> 2] >> (8 * ((g + 1) & 3))) & 0xffu) - 32.0f);
#pragma unroll
            for (int tt = 0; tt < NT; tt++) {
                if (tt < nt) {
                    const int t = t0 + tt;
                    uint32_t xh[16], xl[8];
                    load_x32(X, t, item, 128 * h + 32 * j, xh, xl);
                    int hh[2], ll[2];
                    dot32_u(q, xh, xl, hh, ll);
                    const float *xs = X.xs + t * X.tok_g + item * 16 + g;
                    const float *x16 = X.xsum16 + t * X.tok_g + item * 16 + g;
                    // sum (q - 4) x = s * sum q*xq - 4 * sum x
                    res[tt] += dl0 * (xs[0] * qx(hh[0], ll[0]) - 4.0f * x16[0]);
                    res[tt] += dl1 * (xs[1] * qx(hh[1], ll[1]) - 4.0f * x16[1]);
                }
            }
        }
    }
}

// Dot product of one item of a row held in shared memory.
template <uint32_t TYPE, int NT>
LT_DEVINL void dot_item(const uint8_t *rowp, int item, int nblocks_row, const XS &X, int t0, int nt,
                        float (&res)[NT]) {
    if constexpr (TYPE == T_Q4_K) {
        dot_q4k<NT>(rowp + 144 * item, item, X, t0, nt, res);
    } else if constexpr (TYPE == T_Q6_K) {
        dot_q6k<NT>(rowp + 210 * item, item, X, t0, nt, res);
    } else if constexpr (TYPE == T_Q5_K) {
        dot_q5k<NT>(rowp + 176 * item, item, X, t0, nt, res);
    } else if constexpr (TYPE == T_Q3_K) {
        dot_q3k<NT>(rowp + 110 * item, item, X, t0, nt, res);
    } else if constexpr (TYPE == T_Q5_0 || TYPE == T_Q5_1 || TYPE == T_IQ4_NL) {
        constexpr int FMT = TYPE == T_Q5_0 ? 0 : TYPE == T_Q5_1 ? 1 : 2;
        const int nb = min(8, nblocks_row - 8 * item);
        dot_b32<FMT, NT>(rowp + (FMT == 0 ? 176 : FMT == 1 ? 192 : 144) * item, item, nb, X, t0, nt, res);
    } else {
        const int nb = min(8, nblocks_row - 8 * item);
        dot_q8_0<NT>(rowp + 272 * item, item, nb, X, t0, nt, res);
    }
}

}  // namespace lt
