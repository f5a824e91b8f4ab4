// lt_attn_common.cuh — device helpers of the single-token attention kernels
// (lt_attn_block.cu, lt_stack.cu): block reductions over 16 warps, loads of
// activations other CTAs of the launch wrote, quantised row dots against a
// shared-memory weight tile, per-head norm + RoPE, and the online-softmax
// attention of one query head over a split of the cached positions.
#pragma once

#include "lt_qact.cuh"
#include "lt_rowdot.cuh"

namespace lt {

constexpr int kAbWarps = 16;
constexpr int kAbThreads = kAbWarps * 32;

LT_DEVINL float ab_block_sum(float v, float *red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kAbWarps; i++) s += red[i];
    return s;
}

// x[0, n) (f32, shared) -> quantised rows of X (16 warps, 32-blocks).
LT_DEVINL void ab_quantise(const XS &X, const float *xf, uint32_t n, int warp, int lane) {
#pragma unroll 1
    for (uint32_t b = warp; b < (n + 31) / 32; b += kAbWarps) {
        const uint32_t e = 32 * b + lane;
        qact_block_to_xs(X, 0, (int)b, e < n ? xf[e] : 0.0f, lane);
    }
}

// The same from x before the RMSNorm: quantises x[e] * rms_inv * w[e] (the
// normalised value the norm loop would have stored, with the same rounding).
LT_DEVINL void ab_quantise_norm(const XS &X, const float *xf, uint32_t n, float rms_inv, const float *w, int warp,
                                int lane) {
#pragma unroll 1
    for (uint32_t b = warp; b < (n + 31) / 32; b += kAbWarps) {
        const uint32_t e = 32 * b + lane;
        qact_block_to_xs(X, 0, (int)b, e < n ? xf[e] * rms_inv * w[e] : 0.0f, lane);
    }
}

// n f32 values from global (written by other CTAs of this launch) into
// shared memory, float4 at a time with every load issued before any store.
LT_DEVINL void ab_load(float *dst, const float *src, uint32_t n) {
    const uint32_t n4 = n / 4;
    for (uint32_t i0 = threadIdx.x; i0 < n4; i0 += 4 * kAbThreads) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint32_t i = i0 + u * kAbThreads;
            if (i < n4) v[u] = __ldcg(reinterpret_cast<const float4 *>(src) + i);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint32_t i = i0 + u * kAbThreads;
            if (i < n4) reinterpret_cast<float4 *>(dst)[i] = v[u];
        }
    }
    for (uint32_t i = 4 * n4 + threadIdx.x; i < n; i += kAbThreads) dst[i] = __ldcg(src + i);
}

// A quantised activation row (lt_qact.cuh layout, written by other CTAs of
// this launch) into the shared layout X, loads through L2.
LT_DEVINL void ab_load_qact(const XS &X, const uint8_t *row, uint32_t cols) {
    const uint32_t nhi = cols / 8, nlo = cols / 16, ng = cols / 16;
    for (uint32_t i = threadIdx.x; i < nhi + nlo; i += kAbThreads) {
        if (i < nhi) {
            const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(row) + i);
            const uint32_t e0 = 8 * i;
            *reinterpret_cast<uint4 *>(X.xq + (e0 >> 8) * kXHiPitch + 2 * (e0 & 255)) = v;
        } else {
            const uint32_t c = i - nhi;
            const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(row + (size_t)cols * 2) + c);
            const uint32_t e0 = 16 * c;
            *reinterpret_cast<uint4 *>(X.xl + (e0 >> 8) * kXLoPitch + (e0 & 255)) = v;
        }
    }
    const float *sc = reinterpret_cast<const float *>(row + (size_t)cols * 3);
    for (uint32_t i = threadIdx.x; i < 2 * ng; i += kAbThreads) {
        const float v = __ldcg(sc + i);
        if (i < ng)
            X.xs[i] = v;
        else
            X.xsum16[i - ng] = v;
    }
}

// rows [0, nrows) of a shared tile (pitch) against X: y[r] per row.  Lanes
// own 64-column chunks (spread_chunk within each group of 32), loaded once per chunk;
// warp w takes rows 4w .. 4w+3 (then 64 further): each activation chunk a
// warp loads serves four rows, so few warps load it.
template <uint32_t T, int R = 4>
LT_DEVINL void ab_rows(const uint8_t *tile, uint64_t pitch, uint32_t nrows, uint32_t cols, uint32_t nb, const XS &X,
                       int warp, int lane, float *y) {
    const uint32_t nch = (cols + 63) / 64;
    for (uint32_t r0 = warp * R; r0 < nrows; r0 += kAbWarps * R) {
        float acc[R];
#pragma unroll
        for (int i = 0; i < R; i++) acc[i] = 0.0f;
        for (uint32_t g = 0; g < nch; g += 32) {
            const uint32_t n = min(32u, nch - g);
            if ((uint32_t)lane < n) {
                const uint32_t cb = g + spread_chunk((uint32_t)lane, n);
                XChunk xc;
                xchunk_load(X, 0, (int)cb, xc);
#pragma unroll
                for (int i = 0; i < R; i++) {
                    const uint32_t r = r0 + i;
                    if (r < nrows) acc[i] += dot64<T>(tile + (size_t)r * pitch, (int)cb, (int)nb, xc);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < R; i++) {
            const uint32_t r = r0 + i;
            const float v = warp_sum(acc[i]);
            if (lane == 0 && r < nrows) y[r] = v;
        }
    }
}

// ab_rows with as few rows per warp as fill the 16 warps (a warp's rows share
// its activation chunk loads but run on one warp; every row's sum order is the
// same for any split).
template <uint32_t T>
LT_DEVINL void ab_rows_fit(const uint8_t *tile, uint64_t pitch, uint32_t nrows, uint32_t cols, uint32_t nb,
                           const XS &X, int warp, int lane, float *y) {
    if (nrows <= (uint32_t)kAbWarps)
        ab_rows<T, 1>(tile, pitch, nrows, cols, nb, X, warp, lane, y);
    else if (nrows <= 2u * kAbWarps)
        ab_rows<T, 2>(tile, pitch, nrows, cols, nb, X, warp, lane, y);
    else if (nrows <= 3u * kAbWarps)
        ab_rows<T, 3>(tile, pitch, nrows, cols, nb, X, warp, lane, y);
    else
        ab_rows<T, 4>(tile, pitch, nrows, cols, nb, X, warp, lane, y);
}

// ab_rows_fit for a tile of type T, or (T == 0) of the run-time type `type`.
template <uint32_t T>
LT_DEVINL void ab_rows_any(uint32_t type, const uint8_t *tile, uint64_t pitch, uint32_t nrows, uint32_t cols,
                           uint32_t nb, const XS &X, int warp, int lane, float *y) {
    if constexpr (T != 0) {
        ab_rows_fit<T>(tile, pitch, nrows, cols, nb, X, warp, lane, y);
    } else {
        switch (type) {
        case T_Q8_0: ab_rows_fit<T_Q8_0>(tile, pitch, nrows, cols, nb, X, warp, lane, y); break;
        case T_Q4_K: ab_rows_fit<T_Q4_K>(tile, pitch, nrows, cols, nb, X, warp, lane, y); break;
        case T_Q6_K: ab_rows_fit<T_Q6_K>(tile, pitch, nrows, cols, nb, X, warp, lane, y); break;
        default: break;
        }
    }
}

LT_DEVINL float ab_rinv(float ss, uint32_t n, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
}

// Per-head RMSNorm (optional weights) and RoPE of the query head hq and the
// key head hk (hd values each, shared memory), both at once: threads
// [0, hd) work on q, [hd, 2 hd) on k.
LT_DEVINL void ab_norm_rope2(float *hq, const float *qn, float *hk, const float *kn, const AttnGeom &g, uint32_t pos,
                             float *red) {
    const uint32_t hd = g.hd, half = hd / 2, tid = threadIdx.x;
    const int warp = (int)(tid >> 5), lane = (int)(tid & 31);
    const bool isq = tid < hd, isk = tid >= hd && tid < 2 * hd;
    float *v = isq ? hq : hk;
    const float *nw = isq ? qn : kn;
    const uint32_t e = isq ? tid : tid - hd;
    float ss = 0.0f;
    if ((isq || isk) && nw) ss = __fmul_rn(v[e], v[e]);
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if ((isq || isk) && nw) {
        const uint32_t w0 = isq ? 0 : hd / 32;
        float t = 0.0f;
        for (uint32_t w = 0; w < hd / 32; w++) t = __fadd_rn(t, red[w0 + w]);
        const float rms_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)hd), g.eps)));
        v[e] = __fmul_rn(__fmul_rn(v[e], rms_inv), nw[e]);
    }
    __syncthreads();
    // rope: threads [0, half) rotate q's pairs, [half, hd) k's
    float r0 = 0.0f, r1 = 0.0f;
    uint32_t i0 = 0, i1 = 0;
    float *rv = tid < half ? hq : hk;
    const bool act = tid < hd;
    if (act) {
        const uint32_t i = tid < half ? tid : tid - half;
        const float ang = __fmul_rn((float)pos, __fdiv_rn(1.0f, powf(g.theta, __fdiv_rn((float)(2 * i), (float)hd))));
        float sn, cs;
        sincosf(ang, &sn, &cs);
        i0 = g.rope_neox ? i : 2 * i;
        i1 = g.rope_neox ? i + half : 2 * i + 1;
        const float x0 = rv[i0], x1 = rv[i1];
        r0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        r1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
    }
    __syncthreads();
    if (act) {
        rv[i0] = r0;
        rv[i1] = r1;
    }
    __syncthreads();
}

// Online-softmax attention of one query head over the split's positions of
// the window (src/ops/attn.zig:13-42): warp w takes positions s*16 + w,
// + 16 S, ...; lane owns head dims [lane*PER, lane*PER + PER) and loads them
// as one vector per position.  The next batch of NB positions is in flight
// while the current one is scored; the current position (the last of the
// window) comes from shared memory, older ones from the cache (f16 or f32).
template <int HD, bool F16>
LT_DEVINL void ab_attend(const void *kcache, const void *vcache, const AttnGeom &g, uint32_t s, uint32_t S, uint32_t win, uint32_t first, size_t kvoff,
                         uint32_t nkv, const float *hq, const float *hk, const float *hv, int warp, int lane,
                         float &m, float &l, float (&o)[HD / 32]) {
    constexpr int PER = HD / 32;
    constexpr int W = F16 ? PER / 2 : PER;  // 32-bit words of a lane's slice of one vector
    constexpr int NB = 8 / W > 0 ? 8 / W : 1;  // two batches of K and V words: 32 registers
    const size_t esz = F16 ? 2 : 4;
    const uint8_t *kc = static_cast<const uint8_t *>(kcache), *vc = static_cast<const uint8_t *>(vcache);
    float qv[PER];
#pragma unroll
    for (int i = 0; i < PER; i++) {
        qv[i] = hq[lane * PER + i];
        o[i] = 0.0f;
    }
    const uint32_t stride = S * kAbWarps, last = win - 1;  // position `last` is this step's
    auto load = [&](uint32_t j0, uint32_t (&kr)[NB][W], uint32_t (&vr)[NB][W]) {
#pragma unroll
        for (int b = 0; b < NB; b++) {
            const uint32_t j = j0 + b * stride;
            if (j < last) {
                const size_t off = (((size_t)((first + j) % g.cap) * nkv + kvoff) + (size_t)lane * PER) * esz;
#pragma unroll
                for (int w4 = 0; w4 < W; w4 += 4) {
                    if constexpr (W >= 4) {
                        const uint4 kk = __ldg(reinterpret_cast<const uint4 *>(kc + off) + w4 / 4);
                        const uint4 vv = __ldg(reinterpret_cast<const uint4 *>(vc + off) + w4 / 4);
                        kr[b][w4] = kk.x; kr[b][w4 + 1] = kk.y; kr[b][w4 + 2] = kk.z; kr[b][w4 + 3] = kk.w;
                        vr[b][w4] = vv.x; vr[b][w4 + 1] = vv.y; vr[b][w4 + 2] = vv.z; vr[b][w4 + 3] = vv.w;
                    } else if constexpr (W == 2) {
                        const uint2 kk = __ldg(reinterpret_cast<const uint2 *>(kc + off));
                        const uint2 vv = __ldg(reinterpret_cast<const uint2 *>(vc + off));
                        kr[b][0] = kk.x; kr[b][1] = kk.y;
                        vr[b][0] = vv.x; vr[b][1] = vv.y;
                    } else {
                        kr[b][0] = __ldg(reinterpret_cast<const uint32_t *>(kc + off));
                        vr[b][0] = __ldg(reinterpret_cast<const uint32_t *>(vc + off));
                    }
                }
            }
        }
    };
    auto val = [&](const uint32_t (&r)[W], int i) -> float {
        if constexpr (F16)
            return f16_bits_to_f32((r[i >> 1] >> (16 * (i & 1))) & 0xffffu);
        else
            return __uint_as_float(r[i]);
    };
    auto update = [&](float sc, const float *vals) {
        const float mn = fmaxf(m, sc);
        const float al = expf(m - mn), p = expf(sc - mn);
        l = l * al + p;
#pragma unroll
        for (int i = 0; i < PER; i++) o[i] = fmaf(p, vals[i], o[i] * al);
        m = mn;
    };
    uint32_t ka[NB][W], va[NB][W], kb[NB][W], vb[NB][W];
    uint32_t j0 = s * kAbWarps + warp;
    if (j0 < last) load(j0, ka, va);
    for (; j0 < last; j0 += NB * stride) {
        const uint32_t jn = j0 + NB * stride;
        if (jn < last) load(jn, kb, vb);
        float dot[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) {
            dot[b] = 0.0f;
#pragma unroll
            for (int i = 0; i < PER; i++) dot[b] = fmaf(qv[i], val(ka[b], i), dot[b]);
        }
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1)
#pragma unroll
            for (int b = 0; b < NB; b++) dot[b] += __shfl_xor_sync(0xffffffffu, dot[b], o2);
#pragma unroll
        for (int b = 0; b < NB; b++) {
            if (j0 + b * stride < last) {
                float vals[PER];
#pragma unroll
                for (int i = 0; i < PER; i++) vals[i] = val(va[b], i);
                update(dot[b] * g.scale, vals);
            }
        }
#pragma unroll
        for (int b = 0; b < NB; b++)
#pragma unroll
            for (int w = 0; w < W; w++) {
                ka[b][w] = kb[b][w];
                va[b][w] = vb[b][w];
            }
    }
    // this step's position: the warp whose sequence it ends
    if (last % stride == s * kAbWarps + (uint32_t)warp) {
        float dot = 0.0f, vals[PER];
#pragma unroll
        for (int i = 0; i < PER; i++) {
            dot = fmaf(qv[i], hk[lane * PER + i], dot);
            vals[i] = hv[lane * PER + i];
        }
        dot = warp_sum(dot);
        update(dot * g.scale, vals);
    }
}


}  // namespace lt
