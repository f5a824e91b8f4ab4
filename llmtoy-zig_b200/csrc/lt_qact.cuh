// lt_qact.cuh — quantised activation rows in global memory ("qact").
//
// An activation row of `cols` f32 values (cols % 32 == 0) is stored once, by
// the kernel that produces it, as
//     [int16 hi x cols][int8 lo x cols][f32 scale x cols/32][f32 sum16 x cols/16]
// at a 16-byte row pitch: x ~= scale * (hi + lo/254) per 32-block, sum16 =
// f32 sum of the original values per 16 (lt_decode.cuh explains the split).
// Consumers copy rows into the padded shared-memory layout of lt_decode.cuh
// instead of each CTA re-quantising.
#pragma once

#include "lt_decode.cuh"
#include "lt_launch.cuh"

namespace lt {

__host__ __device__ inline size_t qact_pitch(uint64_t cols) {
    return align16((size_t)cols * 3 + (cols / 32) * 4 + (cols / 16) * 4);
}

// Quantise the 32-block b of a row; the calling warp holds one value per lane.
LT_DEVINL void qact_store_block(uint8_t *qrow, int cols, int b, float v, int lane) {
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int qh = 0, ql = 0;
    float s = 0.0f;
    if (amax > 0.0f) {
        const float inv = 32767.0f / amax;
        s = amax / 32767.0f;
        qh = max(-32767, min(32767, __float2int_rn(v * inv)));
        const float r = fmaf(-(float)qh, s, v);  // remainder, |r| <~ s/2
        ql = max(-127, min(127, __float2int_rn(r * inv * 254.0f)));
    }
    reinterpret_cast<int16_t *>(qrow)[32 * b + lane] = (int16_t)qh;
    reinterpret_cast<int8_t *>(qrow + (size_t)cols * 2)[32 * b + lane] = (int8_t)ql;
    float sum = v;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    float *sc = reinterpret_cast<float *>(qrow + (size_t)cols * 3);
    if (lane == 0) sc[b] = s;
    if ((lane & 15) == 0) sc[cols / 32 + 2 * b + (lane >> 4)] = sum;
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
    const int nsc = cols / 32, nsum = cols / 16;
    for (int i = tid; i < nt * (nsc + nsum); i += nthr) {
        const int t = i / (nsc + nsum), r = i - t * (nsc + nsum);
        const float v = reinterpret_cast<const float *>(rows[t] + (size_t)cols * 3)[r];
        if (r < nsc)
            X.xs[t * X.tok_blk + r] = v;
        else
            X.xsum16[t * X.tok_blk * 2 + (r - nsc)] = v;
    }
}

}  // namespace lt
