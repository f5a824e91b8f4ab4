// lt_sample.cu — sampling beyond greedy as the last op of a decode step
// (src/model/sample.zig:27-183): temperature, the top-k fast path (k <= 256,
// sampleTopK :82-145) with optional top-p, and the full path (softmax, top-k
// threshold :147-155, top-p cut :157-178, renormalise :180-187, multinomial).
// The random stream is std.Random.DefaultPrng (xoshiro256++ seeded by
// SplitMix64) with Random.float(f32), restated from the published
// algorithms; its four words live on the device and advance only when a
// token is actually sampled (not on prompt positions).
//
// One CTA of 1024 threads per launch.  The top-k candidates are found by a
// radix select on order-preserving keys and compacted in index order, so ties
// resolve as the reference's insertion (earlier index first); the sums that
// the reference accumulates sequentially (the softmax denominator, the
// running cumulative sum) are block reductions here, which can move a draw
// that lands within rounding of a bucket edge.
#include "lt_launch.cuh"
#include "lt_router.cuh"

namespace lt {

constexpr int kSmpThreads = 1024;
constexpr int kSmpMaxK = 256;

struct SampleArgs {
    const float *logits;
    uint32_t n;
    float temperature, top_p;
    uint32_t top_k;
    unsigned long long *rng;  // 4 words
    uint32_t *tokens, *pos;
    const uint32_t *n_prompt;
    float *probs;  // [n] scratch (full path)
};

LT_DEVINL uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

LT_DEVINL uint64_t xoshiro_next(uint64_t (&s)[4]) {
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

// Random.float(f32): 23 mantissa bits, exponent from the leading zeros of the rest.
LT_DEVINL float rng_float(uint64_t (&s)[4]) {
    const uint64_t rnd = xoshiro_next(s);
    int lz = __clzll((long long)rnd);
    if (lz >= 41) {
        lz = 41 + __clzll((long long)xoshiro_next(s));
        if (lz == 41 + 64) lz += __clz((int)((uint32_t)xoshiro_next(s) | 0x7FFu));
    }
    return __uint_as_float(((uint32_t)(126 - lz) << 23) | ((uint32_t)rnd & 0x7FFFFFu));
}

// Order-preserving key of a float (larger float -> larger key; NaN lowest).
LT_DEVINL uint32_t fkey(float v) { return (uint32_t)(router_key(v, 0) >> 32); }

LT_DEVINL float smp_max(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = red[0];
    for (int i = 1; i < kSmpThreads / 32; i++) m = fmaxf(m, red[i]);
    return m;
}

LT_DEVINL float smp_sum(float v, float *red) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.0f;
    for (int i = 0; i < kSmpThreads / 32; i++) s += red[i];
    return s;
}

// Exclusive scan of one value per thread (block-wide, deterministic order).
LT_DEVINL uint32_t smp_scan_u32(uint32_t v, uint32_t *wsum, uint32_t &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    __syncthreads();
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    uint32_t base = 0, tot = 0;
    for (int w = 0; w < kSmpThreads / 32; w++) {
        if (w < warp) base += wsum[w];
        tot += wsum[w];
    }
    total = tot;
    return base + incl - v;
}

LT_DEVINL float smp_scan_f32(float v, float *wsum, float &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    __syncthreads();
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    float base = 0.0f, tot = 0.0f;
    for (int w = 0; w < kSmpThreads / 32; w++) {
        if (w < warp) base += wsum[w];
        tot += wsum[w];
    }
    total = tot;
    return base + incl - v;
}

// The k-th largest key among keys(i), i < n (k >= 1): returns it and how
// many elements equal to it belong to the top k.
template <class KeyFn>
LT_DEVINL uint32_t radix_select(uint32_t n, uint32_t k, KeyFn key, uint32_t *hist, uint32_t *s_sel, uint32_t &need) {
    uint32_t prefix = 0, mask = 0, kk = k;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (uint32_t i = threadIdx.x; i < 256; i += kSmpThreads) hist[i] = 0;
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < n; i += kSmpThreads) {
            const uint32_t kv = key(i);
            if ((kv & mask) == prefix) atomicAdd(&hist[(kv >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t cum = 0, d = 255;
            for (;; d--) {
                if (cum + hist[d] >= kk || d == 0) break;
                cum += hist[d];
            }
            s_sel[0] = d;
            s_sel[1] = kk - cum;
        }
        __syncthreads();
        prefix |= s_sel[0] << shift;
        mask |= 255u << shift;
        kk = s_sel[1];
        __syncthreads();
    }
    need = kk;
    return prefix;
}

__global__ void __launch_bounds__(kSmpThreads) k_sample(SampleArgs a) {
    __shared__ float red[kSmpThreads / 32];
    __shared__ uint32_t wsum[kSmpThreads / 32];
    __shared__ float wsumf[kSmpThreads / 32];
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_sel[4];
    __shared__ uint64_t ckey[kSmpMaxK];
    __shared__ uint32_t s_pick;
    pdl_wait();
    const uint32_t tid = threadIdx.x, n = a.n;
    const uint32_t p = *a.pos;
    if (p + 1 < *a.n_prompt) {  // a prompt position: nothing sampled, the stream does not move
        __syncthreads();
        if (tid == 0) *a.pos = p + 1;
        return;
    }
    const float *lg = a.logits;
    uint32_t pick = 0;
    if (a.temperature == 0.0f) {  // greedy: first index of the maximum
        float bv = -INFINITY;
        uint32_t bi = 0xffffffffu;
        for (uint32_t i = tid; i < n; i += kSmpThreads) {
            const float v = lg[i];
            if (v == v && (bi == 0xffffffffu || v > bv)) {
                bv = v;
                bi = i;
            }
        }
        const float m = smp_max(bi == 0xffffffffu ? -INFINITY : bv, red);
        if (tid == 0) s_pick = 0xffffffffu;
        __syncthreads();
        if (bi != 0xffffffffu && bv == m) atomicMin(&s_pick, bi);
        __syncthreads();
        pick = s_pick == 0xffffffffu ? 0 : s_pick;
    } else {
        const float inv_t = a.temperature != 1.0f ? __fdiv_rn(1.0f, a.temperature) : 1.0f;
        auto L = [&](uint32_t i) { return a.temperature != 1.0f ? __fmul_rn(lg[i], inv_t) : lg[i]; };
        float mx = -INFINITY;
        for (uint32_t i = tid; i < n; i += kSmpThreads) mx = fmaxf(mx, L(i));
        const float M = smp_max(mx, red);
        const bool fast = a.top_k > 0 && a.top_k < n && a.top_k <= (uint32_t)kSmpMaxK;
        uint64_t st[4];
        if (tid == 0)
            for (int i = 0; i < 4; i++) st[i] = a.rng[i];
        if (fast) {
            float es = 0.0f;
            for (uint32_t i = tid; i < n; i += kSmpThreads) es += expf(L(i) - M);
            const float S = smp_sum(es, red);
            const uint32_t k = a.top_k;
            uint32_t need = 0;
            const uint32_t T = radix_select(n, k, [&](uint32_t i) { return fkey(L(i)); }, hist, s_sel, need);
            // candidates in index order: every key > T, the first `need` keys == T
            const uint32_t C = (n + kSmpThreads - 1) / kSmpThreads, i0 = tid * C, i1 = min(n, i0 + C);
            uint32_t cg = 0, ce = 0;
            for (uint32_t i = i0; i < i1; i++) {
                const uint32_t kv = fkey(L(i));
                cg += kv > T;
                ce += kv == T;
            }
            uint32_t tg = 0, te = 0;
            uint32_t og = smp_scan_u32(cg, wsum, tg);
            uint32_t oe = smp_scan_u32(ce, wsum, te);
            for (uint32_t i = tid; i < (uint32_t)kSmpMaxK; i += kSmpThreads) ckey[i] = 0;
            __syncthreads();
            for (uint32_t i = i0; i < i1; i++) {
                const float v = L(i);
                const uint32_t kv = fkey(v);
                if (kv > T) ckey[og++] = router_key(v, i);
                else if (kv == T && oe < need) ckey[tg + oe++] = router_key(v, i);
                else if (kv == T) oe++;
            }
            __syncthreads();
            // bitonic sort of the candidate keys, descending (value desc, index asc)
            for (uint32_t size = 2; size <= (uint32_t)kSmpMaxK; size <<= 1) {
                for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
                    if (tid < (uint32_t)kSmpMaxK) {
                        const uint32_t j = tid ^ stride;
                        if (j > tid) {
                            const bool desc = (tid & size) == 0;
                            const uint64_t x = ckey[tid], y = ckey[j];
                            if (desc ? x < y : x > y) {
                                ckey[tid] = y;
                                ckey[j] = x;
                            }
                        }
                    }
                    __syncthreads();
                }
            }
            if (tid == 0) {  // sampleTopK's tail (sample.zig:124-145)
                float pr[kSmpMaxK];
                uint32_t id[kSmpMaxK];
                for (uint32_t c = 0; c < k; c++) {
                    id[c] = ~(uint32_t)ckey[c];
                    pr[c] = __fdiv_rn(expf(L(id[c]) - M), S);
                }
                uint32_t kept = k;
                if (a.top_p < 1.0f) {
                    float cum = 0.0f;
                    for (uint32_t c = 0; c < k; c++) {
                        cum = __fadd_rn(cum, pr[c]);
                        if (cum >= a.top_p) {
                            kept = c + 1;
                            break;
                        }
                    }
                }
                float ks = 0.0f;
                for (uint32_t c = 0; c < kept; c++) ks = __fadd_rn(ks, pr[c]);
                if (ks <= 0.0f) {
                    pick = id[0];
                } else {
                    uint64_t s4[4] = {st[0], st[1], st[2], st[3]};
                    const float r = __fmul_rn(rng_float(s4), ks);
                    for (int i = 0; i < 4; i++) st[i] = s4[i];
                    pick = id[kept - 1];
                    float cum = 0.0f;
                    for (uint32_t c = 0; c < kept; c++) {
                        cum = __fadd_rn(cum, pr[c]);
                        if (r <= cum) {
                            pick = id[c];
                            break;
                        }
                    }
                }
            }
        } else {
            // full path: softmax into the scratch probabilities
            float es = 0.0f;
            for (uint32_t i = tid; i < n; i += kSmpThreads) {
                const float e = expf(L(i) - M);
                a.probs[i] = e;
                es += e;
            }
            const float S = smp_sum(es, red);
            for (uint32_t i = tid; i < n; i += kSmpThreads) a.probs[i] = __fdiv_rn(a.probs[i], S);
            __syncthreads();
            float *pb = a.probs;
            if (a.top_k > 0 && a.top_k < n) {  // zero everything below the k-th largest probability
                uint32_t need = 0;
                const uint32_t T = radix_select(n, a.top_k, [&](uint32_t i) { return __float_as_uint(__ldcg(pb + i)); },
                                                hist, s_sel, need);
                const float thr = __uint_as_float(T);
                for (uint32_t i = tid; i < n; i += kSmpThreads)
                    if (pb[i] < thr) pb[i] = 0.0f;
                __syncthreads();
            }
            if (a.top_p < 1.0f) {
                // the largest probabilities whose running sum first reaches top_p: find the
                // threshold key digit by digit with per-digit sums, then take
                // the needed elements at the threshold in index order
                __shared__ float hsum[256];
                uint32_t prefix = 0, mask = 0;
                float above = 0.0f;  // sum of the probabilities above the current prefix range
                for (int shift = 24; shift >= 0; shift -= 8) {
                    for (uint32_t i = tid; i < 256; i += kSmpThreads) hsum[i] = 0.0f;
                    __syncthreads();
                    for (uint32_t i = tid; i < n; i += kSmpThreads) {
                        const float v = pb[i];
                        const uint32_t kv = __float_as_uint(v);
                        if (v > 0.0f && (kv & mask) == prefix) atomicAdd(&hsum[(kv >> shift) & 255u], v);
                    }
                    __syncthreads();
                    if (tid == 0) {
                        float cum = above;
                        uint32_t d = 255;
                        for (;; d--) {
                            if ((hsum[d] > 0.0f && cum + hsum[d] >= a.top_p) || d == 0) break;
                            cum += hsum[d];
                        }
                        s_sel[0] = d;
                        wsumf[0] = cum;
                    }
                    __syncthreads();
                    prefix |= s_sel[0] << shift;
                    mask |= 255u << shift;
                    above = wsumf[0];
                    __syncthreads();
                }
                const float tval = __uint_as_float(prefix);
                // keep every p > tval; of the p == tval, as many as reach top_p, in index order
                const uint32_t C = (n + kSmpThreads - 1) / kSmpThreads, i0 = tid * C, i1 = min(n, i0 + C);
                uint32_t ce = 0;
                for (uint32_t i = i0; i < i1; i++) ce += pb[i] == tval && tval > 0.0f;
                uint32_t te = 0;
                uint32_t oe = smp_scan_u32(ce, wsum, te);
                uint32_t m = te;
                if (tval > 0.0f) {
                    m = 0;
                    float cum = above;
                    while (m < te) {
                        cum = __fadd_rn(cum, tval);
                        m++;
                        if (cum >= a.top_p) break;
                    }
                }
                for (uint32_t i = i0; i < i1; i++) {
                    const float v = pb[i];
                    if (v < tval) pb[i] = 0.0f;
                    else if (v == tval && tval > 0.0f) {
                        if (oe >= m) pb[i] = 0.0f;
                        oe++;
                    }
                }
                __syncthreads();
            }
            // renormalise, then the multinomial draw over the index order
            float ps = 0.0f;
            for (uint32_t i = tid; i < n; i += kSmpThreads) ps += pb[i];
            const float sum = smp_sum(ps, red);
            const float inv = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 1.0f;
            const uint32_t C = (n + kSmpThreads - 1) / kSmpThreads, i0 = tid * C, i1 = min(n, i0 + C);
            float cs = 0.0f;
            for (uint32_t i = i0; i < i1; i++) {
                const float v = sum > 0.0f ? __fmul_rn(pb[i], inv) : pb[i];
                pb[i] = v;
                cs = __fadd_rn(cs, v);
            }
            float tot = 0.0f;
            const float base = smp_scan_f32(cs, wsumf, tot);
            __shared__ float s_r;
            if (tid == 0) {
                uint64_t s4[4] = {st[0], st[1], st[2], st[3]};
                s_r = rng_float(s4);
                for (int i = 0; i < 4; i++) st[i] = s4[i];
                s_pick = 0xffffffffu;
            }
            __syncthreads();
            const float r = s_r;
            if (i1 > i0 && r <= __fadd_rn(base, cs)) {
                float cum = base;
                for (uint32_t i = i0; i < i1; i++) {
                    cum = __fadd_rn(cum, pb[i]);
                    if (r <= cum) {
                        atomicMin(&s_pick, i);
                        break;
                    }
                }
            }
            __syncthreads();
            pick = s_pick == 0xffffffffu ? n - 1 : s_pick;
        }
        if (tid == 0)
            for (int i = 0; i < 4; i++) a.rng[i] = st[i];
    }
    if (tid == 0) {
        a.tokens[p + 1] = pick;
        *a.pos = p + 1;
    }
}

cudaError_t launch_sample(const LaunchCfg &c, const float *logits, uint32_t n, float temperature, uint32_t top_k,
                          float top_p, unsigned long long *rng, uint32_t *tokens, uint32_t *pos,
                          const uint32_t *n_prompt, float *probs) {
    SampleArgs a{logits, n, temperature, top_p, top_k, rng, tokens, pos, n_prompt, probs};
    return launch_k(c, "sample", k_sample, dim3(1), dim3(kSmpThreads), 0, a);
}

}  // namespace lt
