// lt_rowdot.cuh — row dot products in 64-column chunks with the activation
// chunk held in registers.
//
// The single-token kernel streams many weight rows against one activation
// vector.  Decoding a whole superblock per lane (lt_decode.cuh) re-reads
// 768 bytes of quantised activations from shared memory for every row, which
// makes shared-memory bandwidth, not HBM, the limit.  Here a lane owns one
// 64-column chunk of the activation (hi, lo, scales, sums: 56 registers),
// loads it once, and walks the rows: per row it reads only that chunk's
// weight bytes.  The integer dot products and the scale arithmetic are the
// same as lt_decode.cuh's (two-term int16 + int8 activations, dp2a/dp4a,
// 16-group scales).
#pragma once

#include "lt_decode.cuh"

namespace lt {

// A lane's 64 activation values: element 2i, 2i+1 in hi[i] (int16 pair),
// elements 4i..4i+3 in lo[i] (int8), per 16-group scale and sum.
struct XChunk {
    uint32_t hi[32];
    uint32_t lo[16];
    float s[4];
    float sum[4];
};

// The chunk taken by lane l of n lanes that cover n consecutive chunks.  The
// four chunks of a 256-column item sit 128 bytes apart in X (the same banks),
// items 528 bytes apart (different banks), so consecutive lanes take chunks
// of different items: an 8-lane wavefront of 16-byte loads then falls in 8
// bank groups instead of 2 (n % 4 == 0; otherwise lane l takes chunk l).
LT_DEVINL uint32_t spread_chunk(uint32_t l, uint32_t n) {
    if (n % 4 != 0) return l;
    const uint32_t q = n / 4;
    return (l % q) * 4 + l / q;
}

// Chunk cb (columns [64 cb, 64 cb + 64)) of row t of the padded layout X.
LT_DEVINL void xchunk_load(const XS &X, int t, int cb, XChunk &x) {
    const int e0 = 64 * cb;
    const uint8_t *ph = X.xq + (size_t)t * X.tok_hi + (e0 >> 8) * kXHiPitch + 2 * (e0 & 255);
    const uint8_t *pl = X.xl + (size_t)t * X.tok_lo + (e0 >> 8) * kXLoPitch + (e0 & 255);
#pragma unroll
    for (int v = 0; v < 8; v++) {
        const uint4 h4 = lds128(ph + 16 * v);
        x.hi[4 * v] = h4.x; x.hi[4 * v + 1] = h4.y; x.hi[4 * v + 2] = h4.z; x.hi[4 * v + 3] = h4.w;
    }
#pragma unroll
    for (int v = 0; v < 4; v++) {
        const uint4 l4 = lds128(pl + 16 * v);
        x.lo[4 * v] = l4.x; x.lo[4 * v + 1] = l4.y; x.lo[4 * v + 2] = l4.z; x.lo[4 * v + 3] = l4.w;
    }
    const float4 s4 = *reinterpret_cast<const float4 *>(X.xs + t * X.tok_g + e0 / 16);
    const float4 m4 = *reinterpret_cast<const float4 *>(X.xsum16 + t * X.tok_g + e0 / 16);
    x.s[0] = s4.x; x.s[1] = s4.y; x.s[2] = s4.z; x.s[3] = s4.w;
    x.sum[0] = m4.x; x.sum[1] = m4.y; x.sum[2] = m4.z; x.sum[3] = m4.w;
}

// sum over 32 elements (offset O*32 in the chunk) of q * x_hi and q * x_lo,
// per 16-element half; q unsigned (4 per word).
template <int O>
LT_DEVINL void chunk_dot32_u(const uint32_t (&q)[8], const XChunk &x, int (&hi)[2], int (&lo)[2]) {
    int h0 = 0, h1 = 0, l0 = 0, l1 = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        h0 = dp2a_hi_su((int)x.hi[16 * O + 2 * k + 1], q[k], dp2a_lo_su((int)x.hi[16 * O + 2 * k], q[k], h0));
        h1 = dp2a_hi_su((int)x.hi[16 * O + 2 * k + 9], q[k + 4], dp2a_lo_su((int)x.hi[16 * O + 2 * k + 8], q[k + 4], h1));
        l0 = dp4a_su((int)x.lo[8 * O + k], q[k], l0);
        l1 = dp4a_su((int)x.lo[8 * O + k + 4], q[k + 4], l1);
    }
    hi[0] = h0; hi[1] = h1;
    lo[0] = l0; lo[1] = l1;
}

// Same with signed quant bytes (Q8_0).
template <int O>
LT_DEVINL void chunk_dot32_s(const uint32_t (&q)[8], const XChunk &x, int (&hi)[2], int (&lo)[2]) {
    int h0 = 0, h1 = 0, l0 = 0, l1 = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        h0 = dp2a_hi_ss((int)x.hi[16 * O + 2 * k + 1], q[k], dp2a_lo_ss((int)x.hi[16 * O + 2 * k], q[k], h0));
        h1 = dp2a_hi_ss((int)x.hi[16 * O + 2 * k + 9], q[k + 4], dp2a_lo_ss((int)x.hi[16 * O + 2 * k + 8], q[k + 4], h1));
        l0 = dp4a_ss((int)x.lo[8 * O + k], q[k], l0);
        l1 = dp4a_ss((int)x.lo[8 * O + k + 4], q[k + 4], l1);
    }
    hi[0] = h0; hi[1] = h1;
    lo[0] = l0; lo[1] = l1;
}

// ── Q4_K: chunk cb = pair c = cb % 4 of sub-blocks (2c, 2c+1) of superblock cb / 4
LT_DEVINL float dot64_q4k(const uint8_t *row, int cb, const XChunk &x) {
    const uint8_t *sb = row + 144 * (cb >> 2);
    const int c = cb & 3;
    const uint4 hdr = lds128(sb);
    const float d = f16_bits_to_f32(hdr.x), dmin = f16_bits_to_f32(hdr.x >> 16);
    // scale_min (src/quant/dequant.zig:291-300): sub-blocks 0-3 in the low
    // 6 bits of bytes 0-7, 4-7 split across bytes 8-11 and the top bits
    uint32_t scw, mnw;
    if (c < 2) {
        scw = hdr.y & 0x3F3F3F3Fu;
        mnw = hdr.z & 0x3F3F3F3Fu;
    } else {
        scw = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
        mnw = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
    }
    const int j0 = (2 * c) & 3;
    const float dA = d * byte_to_f32(scw, j0), mA = dmin * byte_to_f32(mnw, j0);
    const float dB = d * byte_to_f32(scw, j0 + 1), mB = dmin * byte_to_f32(mnw, j0 + 1);
    const uint4 qa = lds128(sb + 16 + 32 * c), qb = lds128(sb + 32 + 32 * c);
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        lo[k] = w[k] & 0x0F0F0F0Fu;         // sub-block 2c: chunk elements 0..31
        hi[k] = (w[k] >> 4) & 0x0F0F0F0Fu;  // sub-block 2c+1: chunk elements 32..63
    }
    int aH[2], aL[2], bH[2], bL[2];
    chunk_dot32_u<0>(lo, x, aH, aL);
    chunk_dot32_u<1>(hi, x, bH, bL);
    const float ra = dA * (x.s[0] * qx(aH[0], aL[0]) + x.s[1] * qx(aH[1], aL[1])) - mA * (x.sum[0] + x.sum[1]);
    const float rb = dB * (x.s[2] * qx(bH[0], bL[0]) + x.s[3] * qx(bH[1], bL[1])) - mB * (x.sum[2] + x.sum[3]);
    return ra + rb;
}

// ── Q6_K (210 B superblocks, 2-byte aligned): chunk cb = quarter qq = cb % 4
// of superblock cb / 4: half n = qq / 2, kinds 2u and 2u+1 (u = qq % 2), i.e.
// elements 128n + 64u + [0, 64) (dequant.zig:235-262).
LT_DEVINL float dot64_q6k(const uint8_t *row, int cb, const XChunk &x) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(row + 210 * (cb >> 2));
    const uint8_t *pa = reinterpret_cast<const uint8_t *>(a & ~(uintptr_t)3);
    const uint32_t sel = (a & 2) ? 0x5432u : 0x3210u;
    const int qq = cb & 3, n = qq >> 1, u = qq & 1;
    uint32_t rq[17], rh[9], rs[6];
#pragma unroll
    for (int i = 0; i < 17; i++) rq[i] = lds32(pa + 4 * (16 * n + i));
#pragma unroll
    for (int i = 0; i < 9; i++) rh[i] = lds32(pa + 4 * (32 + 8 * n + i));
#pragma unroll
    for (int i = 0; i < 6; i++) rs[i] = lds32(pa + 4 * (48 + i));
    const float d = f16_bits_to_f32(__byte_perm(rs[4], rs[5], sel) & 0xffffu);
    // i8 scales sc[8n + 4u + 0..3]: kind 2u (l < 16, l >= 16), kind 2u+1 (same)
    const uint32_t s01 = __byte_perm(rs[0], rs[1], sel), s23 = __byte_perm(rs[1], rs[2], sel);
    const uint32_t s45 = __byte_perm(rs[2], rs[3], sel), s67 = __byte_perm(rs[3], rs[4], sel);
    const uint32_t scw = n == 0 ? (u == 0 ? s01 : s23) : (u == 0 ? s45 : s67);
    const float ds0 = d * (float)(int8_t)(scw & 0xffu), ds1 = d * (float)(int8_t)((scw >> 8) & 0xffu);
    const float ds2 = d * (float)(int8_t)((scw >> 16) & 0xffu), ds3 = d * (float)(int8_t)(scw >> 24);
    uint32_t qA[8], qB[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const uint32_t qlA = __byte_perm(rq[k], rq[k + 1], sel);
        const uint32_t qlB = __byte_perm(rq[8 + k], rq[9 + k], sel);
        const uint32_t h = __byte_perm(rh[k], rh[k + 1], sel);
        if (u == 0) {
            qA[k] = (qlA & 0x0F0F0F0Fu) | ((h << 4) & 0x30303030u);  // kind 0: 128n + l
            qB[k] = (qlB & 0x0F0F0F0Fu) | ((h << 2) & 0x30303030u);  // kind 1: 128n + 32 + l
        } else {
            qA[k] = ((qlA >> 4) & 0x0F0F0F0Fu) | (h & 0x30303030u);         // kind 2: 128n + 64 + l
            qB[k] = ((qlB >> 4) & 0x0F0F0F0Fu) | ((h >> 2) & 0x30303030u);  // kind 3: 128n + 96 + l
        }
    }
    int aH[2], aL[2], bH[2], bL[2];
    chunk_dot32_u<0>(qA, x, aH, aL);
    chunk_dot32_u<1>(qB, x, bH, bL);
    // sum (q - 32) x = s * sum q*xq - 32 * sum x, per 16-group
    const float r0 = ds0 * (x.s[0] * qx(aH[0], aL[0]) - 32.0f * x.sum[0]);
    const float r1 = ds1 * (x.s[1] * qx(aH[1], aL[1]) - 32.0f * x.sum[1]);
    const float r2 = ds2 * (x.s[2] * qx(bH[0], bL[0]) - 32.0f * x.sum[2]);
    const float r3 = ds3 * (x.s[3] * qx(bH[1], bL[1]) - 32.0f * x.sum[3]);
    return (r0 + r1) + (r2 + r3);
}

// ── Q8_0: chunk cb = blocks 2cb and 2cb+1 (68 bytes at a 4-byte boundary);
// the second block only if it exists (nb = blocks in the row).
LT_DEVINL float dot64_q8_0(const uint8_t *row, int cb, int nb, const XChunk &x) {
    const uint8_t *p = row + 68 * cb;
    uint32_t w[17];
#pragma unroll
    for (int i = 0; i < 17; i++) w[i] = lds32(p + 4 * i);
    const float d0 = f16_bits_to_f32(w[0] & 0xffffu);
    uint32_t q0[8];
    q0[0] = word_at<2>(w); q0[1] = word_at<6>(w); q0[2] = word_at<10>(w); q0[3] = word_at<14>(w);
    q0[4] = word_at<18>(w); q0[5] = word_at<22>(w); q0[6] = word_at<26>(w); q0[7] = word_at<30>(w);
    int h[2], l[2];
    chunk_dot32_s<0>(q0, x, h, l);
    float r = d0 * (x.s[0] * qx(h[0], l[0]) + x.s[1] * qx(h[1], l[1]));
    if (2 * cb + 1 < nb) {
        const float d1 = f16_bits_to_f32(w[8] >> 16);
        uint32_t q1[8];
#pragma unroll
        for (int k = 0; k < 8; k++) q1[k] = w[9 + k];
        chunk_dot32_s<1>(q1, x, h, l);
        r += d1 * (x.s[2] * qx(h[0], l[0]) + x.s[3] * qx(h[1], l[1]));
    }
    return r;
}

template <uint32_t TYPE>
LT_DEVINL float dot64(const uint8_t *row, int cb, int nblocks, const XChunk &x) {
    if constexpr (TYPE == T_Q4_K) {
        return dot64_q4k(row, cb, x);
    } else if constexpr (TYPE == T_Q6_K) {
        return dot64_q6k(row, cb, x);
    } else {
        return dot64_q8_0(row, cb, nblocks, x);
    }
}

}  // namespace lt
