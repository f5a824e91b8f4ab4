// lt_qact.cuh — quantised activation rows in global memory ("qact").
//
// An activation row of `cols` f32 values (cols % 32 == 0) is stored once, by
// the kernel that produces it, as
//     [int16 hi x cols][int8 lo x cols][f32 scale x cols/16][f32 sum16 x cols/16]
// at a 16-byte row pitch: x ~= scale * (hi + lo/254) per 16-group, sum16 =
// f32 sum of the original values per 16-group (lt_decode.cuh explains the
// split).  A 16-group is the smallest unit a producer writes, so producers
// that split a row between CTAs at 16-column boundaries quantise independently.
// Consumers copy rows into the padded shared-memory layout of lt_decode.cuh
// instead of each CTA re-quantising.
#pragma once

#include "lt_decode.cuh"
#include "lt_launch.cuh"

namespace lt {

__host__ __device__ inline size_t qact_pitch(uint64_t cols) {
    return align16((size_t)cols * 3 + (cols / 16) * 8);
}

// Quantise one value per lane of a warp; each half-warp is one 16-group.
// Returns the hi/lo terms of this lane and the group's scale and sum.
LT_DEVINL void qact_quant(float v, int &qh, int &ql, float &s, float &sum) {
    float amax = fabsf(v);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    qh = 0;
    ql = 0;
    s = 0.0f;
    if (amax > 0.0f) {
        // any scale works as long as the remainder is taken against it
        s = amax * (1.0f / 32767.0f);
        const float inv = __frcp_rn(s);
        qh = max(-32767, min(32767, __float2int_rn(v * inv)));
        const float r = fmaf(-(float)qh, s, v);  // remainder, |r| <~ s/2
        ql = max(-127, min(127, __float2int_rn(r * inv * 254.0f)));
    }
    sum = v;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
}

// Quantise columns [32b, 32b+32) of a row into global qact row qrow; the
// calling warp holds one value per lane.
LT_DEVINL void qact_store_block(uint8_t *qrow, int cols, int b, float v, int lane) {
    int qh, ql;
    float s, sum;
    qact_quant(v, qh, ql, s, sum);
    reinterpret_cast<int16_t *>(qrow)[32 * b + lane] = (int16_t)qh;
    reinterpret_cast<int8_t *>(qrow + (size_t)cols * 2)[32 * b + lane] = (int8_t)ql;
    float *sc = reinterpret_cast<float *>(qrow + (size_t)cols * 3);
    if ((lane & 15) == 0) {
        sc[2 * b + (lane >> 4)] = s;
        sc[cols / 16 + 2 * b + (lane >> 4)] = sum;
    }
}

// Same quantisation straight into the padded layout X (row t), in shared or
// global memory.  Lanes with own == false (a whole half-warp, that is a whole
// 16-group, at a time) take part in the shuffles but write nothing.
LT_DEVINL void qact_block_to_xs(const XS &X, int t, int b, float v, int lane, bool own = true) {
    int qh, ql;
    float s, sum;
    qact_quant(v, qh, ql, s, sum);
    if (!own) return;
    const int e = 32 * b + lane;
    *reinterpret_cast<int16_t *>(X.xq + (size_t)t * X.tok_hi + (e >> 8) * kXHiPitch + 2 * (e & 255)) = (int16_t)qh;
    *reinterpret_cast<int8_t *>(X.xl + (size_t)t * X.tok_lo + (e >> 8) * kXLoPitch + (e & 255)) = (int8_t)ql;
    if ((lane & 15) == 0) {
        X.xs[t * X.tok_g + e / 16] = s;
        X.xsum16[t * X.tok_g + e / 16] = sum;
    }
}

// Copy nt qact rows (row pointers in shared memory) into the padded layout X.
LT_DEVINL void qact_to_smem(const XS &X, const uint8_t *const *rows, int nt, int cols) {
    const int nhi = cols / 8, nlo = cols / 16;  // 16-byte chunks of the hi and lo arrays
    const int per_tok = nhi + nlo;
    const int tid = threadIdx.x, nthr = blockDim.x;
    for (int i = tid; i < nt * per_tok; i += nthr) {
        const int t = i / per_tok, r = i - t * per_tok;
        if (r < nhi) {
            const uint4 v = reinterpret_cast<const uint4 *>(rows[t])[r];
            const int e0 = 8 * r;
            *reinterpret_cast<uint4 *>(X.xq + (size_t)t * X.tok_hi + (e0 >> 8) * kXHiPitch + 2 * (e0 & 255)) = v;
        } else {
            const int c = r - nhi;
            const uint4 v = reinterpret_cast<const uint4 *>(rows[t] + (size_t)cols * 2)[c];
            const int e0 = 16 * c;
            *reinterpret_cast<uint4 *>(X.xl + (size_t)t * X.tok_lo + (e0 >> 8) * kXLoPitch + (e0 & 255)) = v;
        }
    }
    const int ng = cols / 16;  // scales, then sums
    for (int i = tid; i < nt * 2 * ng; i += nthr) {
        const int t = i / (2 * ng), r = i - t * 2 * ng;
        const float v = reinterpret_cast<const float *>(rows[t] + (size_t)cols * 3)[r];
        if (r < ng)
            X.xs[t * X.tok_g + r] = v;
        else
            X.xsum16[t * X.tok_g + (r - ng)] = v;
    }
}

}  // namespace lt
