// lt_router.cuh — router arithmetic shared by the router kernel and the
// persistent decode kernel, so both produce the same logits, expert ids and
// weights bit for bit.
//
// Logits follow dotf32's exact evaluation order (src/ops/math.zig:96-116):
// lane l owns the chain over elements l, l+32, ... (acc_{l/8}[l%8] in the
// reference), then (a0+a1)+(a2+a3), the 8-wide tail, the ordered 8-lane
// reduction and the scalar tail.  Given the same input vector the logits, and
// so the selected ids, equal the CPU path bit for bit.
//
// Selection (topKWithSoftmaxStats, src/model/gemma4/forward.zig:598-629) is
// an insertion sort with a strict '>': the result is ordered by descending
// score and, among equal scores, by ascending index.  Here every expert
// computes its rank in that order directly from a 64-bit key; experts of
// rank < k are the selection.  NaN logits rank below every number (the CPU
// order is not defined for them).
#pragma once

#include "lt_common.cuh"
#include "lt_internal.h"

namespace lt {

constexpr int kRouterChunk = 64;  // weights per lane kept in registers (2048 columns)

// One expert logit in dotf32 order.  w0 holds this lane's weights for the
// first 2048 columns (prefetched); xs is the token row in shared memory.
LT_DEVINL float router_logit(const float *wrow, const float *xs, uint32_t cols, int lane,
                             const float (&w0)[kRouterChunk]) {
    const uint32_t n32 = cols & ~31u;
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < kRouterChunk; j++)
        if (32u * j < n32) acc = __fadd_rn(acc, __fmul_rn(w0[j], xs[32 * j + lane]));
    for (uint32_t base = 32u * kRouterChunk; base < n32; base += 32u * kRouterChunk) {
        float wv[kRouterChunk];
#pragma unroll
        for (int j = 0; j < kRouterChunk; j++) wv[j] = base + 32u * j < n32 ? __ldg(wrow + base + 32 * j + lane) : 0.f;
#pragma unroll
        for (int j = 0; j < kRouterChunk; j++)
            if (base + 32u * j < n32) acc = __fadd_rn(acc, __fmul_rn(wv[j], xs[base + 32 * j + lane]));
    }
    uint32_t i = n32;
    // acc = (acc0 + acc1) + (acc2 + acc3), lane l < 8 holds lane l of the 8-vector
    const float a1 = __shfl_sync(0xffffffffu, acc, (lane + 8) & 31);
    const float a2 = __shfl_sync(0xffffffffu, acc, (lane + 16) & 31);
    const float a3 = __shfl_sync(0xffffffffu, acc, (lane + 24) & 31);
    float v = __fadd_rn(__fadd_rn(acc, a1), __fadd_rn(a2, a3));
    for (; i + 8 <= cols; i += 8)
        if (lane < 8) v = __fadd_rn(v, __fmul_rn(__ldg(wrow + i + lane), xs[i + lane]));
    // @reduce(.Add): ((((-0 + v0) + v1) + ...) + v7)
    float sum = -0.0f;
#pragma unroll
    for (int l = 0; l < 8; l++) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, v, l));
    for (; i < cols; i++) sum = __fadd_rn(sum, __fmul_rn(__ldg(wrow + i), xs[i]));
    return sum;
}

// The same logit with the router row in shared memory (staged by TMA): a
// rolled loop, so the code stays small (the persistent kernels run it once
// per launch, from a cold instruction cache).
LT_DEVINL float router_logit_sm(const float *wsm, const float *xs, uint32_t cols, int lane) {
    const uint32_t n32 = cols & ~31u;
    float acc = 0.0f;
#pragma unroll 8
    for (uint32_t j = 0; j < n32 / 32; j++) acc = __fadd_rn(acc, __fmul_rn(wsm[32 * j + lane], xs[32 * j + lane]));
    uint32_t i = n32;
    const float a1 = __shfl_sync(0xffffffffu, acc, (lane + 8) & 31);
    const float a2 = __shfl_sync(0xffffffffu, acc, (lane + 16) & 31);
    const float a3 = __shfl_sync(0xffffffffu, acc, (lane + 24) & 31);
    float v = __fadd_rn(__fadd_rn(acc, a1), __fadd_rn(a2, a3));
    for (; i + 8 <= cols; i += 8)
        if (lane < 8) v = __fadd_rn(v, __fmul_rn(wsm[i + lane], xs[i + lane]));
    float sum = -0.0f;
#pragma unroll
    for (int l = 0; l < 8; l++) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, v, l));
    for (; i < cols; i++) sum = __fadd_rn(sum, __fmul_rn(wsm[i], xs[i]));
    return sum;
}

// Load this lane's first-chunk router weights for expert row wrow.
LT_DEVINL void router_prefetch(const float *wrow, uint32_t cols, int lane, bool valid, float (&w0)[kRouterChunk]) {
    const uint32_t n32 = cols & ~31u;
#pragma unroll
    for (int j = 0; j < kRouterChunk; j++) w0[j] = (valid && 32u * j < n32) ? __ldg(wrow + 32 * j + lane) : 0.0f;
}

// Sort key of expert i with logit v: larger key = earlier in the selection.
// High word: an order-preserving map of v (-0 as +0, NaN below -inf); low
// word: ~i, so equal values order by ascending index.  Keys are distinct.
LT_DEVINL uint64_t router_key(float v, uint32_t i) {
    uint32_t u = __float_as_uint(v);
    const uint32_t m = u & 0x7fffffffu;
    uint32_t ord;
    if (m > 0x7f800000u)
        ord = 0;  // NaN
    else if (m == 0)
        ord = 0x80000000u;  // +0 and -0
    else
        ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((uint64_t)ord << 32) | (uint32_t)~i;
}

// Selection by rank: keys[0, E) in shared memory (keys[E] = 0 when E is odd),
// sel[r] = the expert of rank r for r < k.  Thread i < E ranks expert i.
LT_DEVINL void router_rank_keys(const uint64_t *keys, uint32_t E, uint32_t k, uint32_t *sel, int tid, int nthr) {
    const uint32_t E2 = (E + 1) & ~1u;
    for (uint32_t i = tid; i < E; i += nthr) {
        const uint64_t ki = keys[i];
        uint32_t r = 0;
#pragma unroll 8
        for (uint32_t j = 0; j < E2; j += 2) {
            const ulonglong2 kk = *reinterpret_cast<const ulonglong2 *>(keys + j);
            r += (kk.x > ki) + (kk.y > ki);
        }
        if (r < k) sel[r] = i;
    }
}

// The same with P threads per expert (threads [0, P*E), P <= 4), each
// counting over a quarter of the keys; cnt is [4][E] shared scratch.  Called
// by the whole block: contains a __syncthreads.
LT_DEVINL void router_rank_keys_split(const uint64_t *keys, uint32_t E, uint32_t k, uint32_t *sel, uint32_t P,
                                      uint32_t *cnt, int tid) {
    const uint32_t E2 = (E + 1) & ~1u;
    const uint32_t span = ((E2 + 2 * P - 1) / (2 * P)) * 2;  // even
    if ((uint32_t)tid < P * E) {
        const uint32_t i = (uint32_t)tid % E, p = (uint32_t)tid / E;
        const uint32_t j0 = p * span, j1 = min(E2, j0 + span);
        const uint64_t ki = keys[i];
        uint32_t r = 0;
#pragma unroll 8
        for (uint32_t j = j0; j < j1; j += 2) {
            const ulonglong2 kk = *reinterpret_cast<const ulonglong2 *>(keys + j);
            r += (kk.x > ki) + (kk.y > ki);
        }
        cnt[p * E + i] = r;
    }
    __syncthreads();
    if ((uint32_t)tid < E) {
        uint32_t r = 0;
        for (uint32_t p = 0; p < P; p++) r += cnt[p * E + tid];
        if (r < k) sel[r] = (uint32_t)tid;
    }
}

// Softmax statistics over all E logits, one warp: lane l sums exp(v - max)
// over experts l, l+32, ... in that order, then a butterfly reduction.
LT_DEVINL void router_softmax_stats(const float *lg, uint32_t E, int lane, float &mx, float &es) {
    float v[kRouterMaxE / 32];
    mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kRouterMaxE / 32; j++) {
        const uint32_t ee = lane + 32 * j;
        v[j] = ee < E ? lg[ee] : -INFINITY;
        mx = fmaxf(mx, v[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    es = 0.0f;
#pragma unroll
    for (int j = 0; j < kRouterMaxE / 32; j++)
        if (lane + 32 * j < E) es += expf(v[j] - mx);
    es = warp_sum(es);
}

// Weights of the selected experts, in selection order (one thread):
// softmax probability, renormalised over the selection if norm_topk, times
// the per-expert scale if given (forward.zig:463-479).
LT_DEVINL void router_weights(const float *lg, const uint32_t *sel, uint32_t k, float mx, float es, int norm_topk,
                              const float *escale, float *w) {
    float sum = 0.0f;
    for (uint32_t i = 0; i < k; i++) {
        w[i] = expf(lg[sel[i]] - mx) / es;
        if (norm_topk) sum += w[i];
    }
    for (uint32_t i = 0; i < k; i++) {
        float v = norm_topk ? w[i] / sum : w[i];
        if (escale) v = escale[sel[i]] * v;
        w[i] = v;
    }
}

}  // namespace lt
