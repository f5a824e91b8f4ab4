// lt_attn.cu — decode-time attention of the model forward loops.
//
//   attn_prep:   per-head Q/K RMSNorm (optional weights), RoPE on Q and K,
//                and the KV-cache append of this position's K and V
//                (src/model/forward.zig:281-292; the per-head norms of
//                src/model/gemma4/forward.zig:267-269; src/ops/rope.zig:14-75)
//   attn_decode: single-query attention of every head over the cached
//                positions (src/ops/attn.zig:13-42, GQA head mapping of
//                forward.zig:294-296, the sliding window of
//                gemma4/forward.zig:315-319)
//
// The position comes from a device word, so one captured graph serves every
// decode step; the KV cache is a ring of `cap` positions per layer,
// [cap][n_kv * head_dim] for K and for V (the reference's KvCache layout), f32
// or f16 elements (the reference's GPU cache keeps f16).
#include "lt_launch.cuh"

namespace lt {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnMaxHd = 256;

LT_DEVINL float block_sum128(float v, float *red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kAttnWarps; i++) s += red[i];
    return s;
}

// rope.zig:21-24: freq_i = 1 / theta^(2i / len), each step rounded in f32.
LT_DEVINL float rope_freq(float theta, uint32_t i, uint32_t len) {
    const float e = __fdiv_rn((float)(2 * i), (float)len);
    return __fdiv_rn(1.0f, powf(theta, e));
}

// One block per head vector: blocks [0, n_heads) the query heads, blocks
// [n_heads, n_heads + n_kv) the key heads (which also append their value
// head).  Thread i < hd/2 rotates pair i.
__global__ void __launch_bounds__(kAttnThreads) k_attn_prep(AttnGeom g, float *qkv, const float *q_norm,
                                                            const float *k_norm, const uint32_t *pos_p, void *kc,
                                                            void *vc) {
    __shared__ float v[kAttnMaxHd];
    __shared__ float red[kAttnWarps];
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t hd = g.hd, half = hd / 2;
    const uint32_t b = blockIdx.x;
    const bool is_q = b < g.n_heads;
    const uint32_t kh = is_q ? 0 : b - g.n_heads;
    const uint32_t nq = g.n_heads * hd, nkv = g.n_kv * hd;
    float *src = is_q ? qkv + (size_t)b * hd : qkv + nq + (size_t)kh * hd;
    const float *nw = is_q ? q_norm : k_norm;
    const uint32_t pos = *pos_p;
    for (uint32_t i = threadIdx.x; i < hd; i += kAttnThreads) v[i] = src[i];
    if (nw) {  // math.zig:20-26 over the head
        float ss = 0.0f;
        for (uint32_t i = threadIdx.x; i < hd; i += kAttnThreads) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
        ss = block_sum128(ss, red);
        const float rms_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), g.eps)));
        for (uint32_t i = threadIdx.x; i < hd; i += kAttnThreads) v[i] = __fmul_rn(__fmul_rn(v[i], rms_inv), nw[i]);
    }
    __syncthreads();
    const size_t slot = (size_t)(pos % g.cap) * nkv + (size_t)kh * hd;  // K and V heads in the caches
    const float fpos = (float)pos;
    for (uint32_t i = threadIdx.x; i < half; i += kAttnThreads) {
        const float ang = __fmul_rn(fpos, rope_freq(g.theta, i, hd));
        float s, c;
        sincosf(ang, &s, &c);
        const uint32_t i0 = g.rope_neox ? i : 2 * i, i1 = g.rope_neox ? i + half : 2 * i + 1;
        const float x0 = v[i0], x1 = v[i1];
        const float r0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        const float r1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        if (is_q) {
            src[i0] = r0;
            src[i1] = r1;
        } else {
            kv_st(kc, slot + i0, r0, g.kv_f16);
            kv_st(kc, slot + i1, r1, g.kv_f16);
        }
    }
    if (!is_q) {
        const float *vs = qkv + nq + nkv + (size_t)kh * hd;
        if (g.v_norm) {  // rmsnormRaw (math.zig:43-48) of the V head
            __syncthreads();
            float ss = 0.0f;
            for (uint32_t i = threadIdx.x; i < hd; i += kAttnThreads) ss = __fadd_rn(ss, __fmul_rn(vs[i], vs[i]));
            ss = block_sum128(ss, red);
            const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), g.eps)));
            for (uint32_t i = threadIdx.x; i < hd; i += kAttnThreads) kv_st(vc, slot + i, __fmul_rn(vs[i], r), g.kv_f16);
        } else {
            for (uint32_t i = threadIdx.x; i < hd; i += kAttnThreads) kv_st(vc, slot + i, vs[i], g.kv_f16);
        }
    }
}

// Attention: grid (n_heads, nsplit).  Split s of head h handles the window
// positions j = s*4 + w + 4*nsplit*m (warp w), online softmax per warp, then
// per CTA; the last CTA of a head merges the splits (partials in scratch,
// one counter per head, reset by the merger).  Each lane holds hd/32 dims.
template <int HD>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(AttnGeom g, const float *q, const void *kc,
                                                              const void *vc, const uint32_t *pos_p, float *out,
                                                              float *part, uint32_t *counters) {
    constexpr int PER = HD / 32;
    __shared__ float s_m[kAttnWarps], s_l[kAttnWarps];
    __shared__ float s_o[kAttnWarps][HD];
    __shared__ int s_last;
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t h = blockIdx.x, split = blockIdx.y, nsplit = gridDim.y;
    const uint32_t kh = h / (g.n_heads / g.n_kv);
    const uint32_t nkv = g.n_kv * HD;
    const uint32_t pos = *pos_p, seq = pos + 1;
    const uint32_t win = g.window ? min(seq, g.window) : seq;
    const uint32_t first = seq - win;

    float qv[PER];
#pragma unroll
    for (int i = 0; i < PER; i++) qv[i] = q[(size_t)h * HD + lane + 32 * i];
    float m = -INFINITY, l = 0.0f, o[PER];
#pragma unroll
    for (int i = 0; i < PER; i++) o[i] = 0.0f;
    const uint32_t stride = kAttnWarps * nsplit;
    for (uint32_t j = split * kAttnWarps + warp; j < win; j += stride) {
        const uint32_t slot = (first + j) % g.cap;
        const size_t row = (size_t)slot * nkv + (size_t)kh * HD;
        float kv[PER], vv[PER];
#pragma unroll
        for (int i = 0; i < PER; i++) {
            kv[i] = kv_ld(kc, row + lane + 32 * i, g.kv_f16);
            vv[i] = kv_ld(vc, row + lane + 32 * i, g.kv_f16);
        }
        float dot = 0.0f;
#pragma unroll
        for (int i = 0; i < PER; i++) dot = fmaf(qv[i], kv[i], dot);
        dot = warp_sum(dot);
        const float sc = dot * g.scale;
        const float mn = fmaxf(m, sc);
        const float a = expf(m - mn), p = expf(sc - mn);
        l = l * a + p;
#pragma unroll
        for (int i = 0; i < PER; i++) o[i] = fmaf(p, vv[i], o[i] * a);
        m = mn;
    }
    if (lane == 0) {
        s_m[warp] = m;
        s_l[warp] = l;
    }
#pragma unroll
    for (int i = 0; i < PER; i++) s_o[warp][lane + 32 * i] = o[i];
    __syncthreads();
    // merge the warps; thread t < HD owns output dim t
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, s_m[w]);
    float L = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; w++) L += s_m[w] == -INFINITY ? 0.0f : s_l[w] * expf(s_m[w] - M);
    float *pp = part + ((size_t)h * nsplit + split) * (HD + 2);
    for (uint32_t t = threadIdx.x; t < HD; t += kAttnThreads) {
        float acc = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; w++)
            if (s_m[w] != -INFINITY) acc += s_o[w][t] * expf(s_m[w] - M);
        pp[2 + t] = acc;
    }
    if (threadIdx.x == 0) {
        pp[0] = M;
        pp[1] = L;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&counters[h], 1u) == nsplit - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float *hp = part + (size_t)h * nsplit * (HD + 2);
    float GM = -INFINITY;
    for (uint32_t s = 0; s < nsplit; s++) GM = fmaxf(GM, __ldcg(hp + s * (HD + 2)));
    float GL = 0.0f;
    for (uint32_t s = 0; s < nsplit; s++) {
        const float ms = __ldcg(hp + s * (HD + 2));
        if (ms != -INFINITY) GL += __ldcg(hp + s * (HD + 2) + 1) * expf(ms - GM);
    }
    for (uint32_t t = threadIdx.x; t < HD; t += kAttnThreads) {
        float acc = 0.0f;
        for (uint32_t s = 0; s < nsplit; s++) {
            const float ms = __ldcg(hp + s * (HD + 2));
            if (ms != -INFINITY) acc += __ldcg(hp + s * (HD + 2) + 2 + t) * expf(ms - GM);
        }
        out[(size_t)h * HD + t] = acc / GL;
    }
    if (threadIdx.x == 0) counters[h] = 0;
}

uint32_t attn_splits(const AttnGeom &g, int num_sms) {
    const uint32_t want = (uint32_t)((num_sms + g.n_heads - 1) / g.n_heads);
    return max(1u, min(want, 64u));
}

size_t attn_scratch_floats(const AttnGeom &g, int num_sms) {
    return (size_t)g.n_heads * attn_splits(g, num_sms) * (g.hd + 2);
}

cudaError_t launch_attn_prep(const LaunchCfg &c, const AttnGeom &g, float *qkv, const float *q_norm,
                             const float *k_norm, const uint32_t *pos, void *kc, void *vc) {
    return launch_k(c, "attn_prep", k_attn_prep, dim3(g.n_heads + g.n_kv), dim3(kAttnThreads), 0, g, qkv, q_norm,
                    k_norm, pos, kc, vc);
}

cudaError_t launch_attn_decode(const LaunchCfg &c, const AttnGeom &g, const float *q, const void *kc,
                               const void *vc, const uint32_t *pos, float *out, float *part, uint32_t *counters) {
    const dim3 grid(g.n_heads, attn_splits(g, c.num_sms));
    switch (g.hd) {
    case 64: return launch_k(c, "attn_decode", k_attn_decode<64>, grid, dim3(kAttnThreads), 0, g, q, kc, vc, pos, out, part, counters);
    case 128: return launch_k(c, "attn_decode", k_attn_decode<128>, grid, dim3(kAttnThreads), 0, g, q, kc, vc, pos, out, part, counters);
    case 256: return launch_k(c, "attn_decode", k_attn_decode<256>, grid, dim3(kAttnThreads), 0, g, q, kc, vc, pos, out, part, counters);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace lt
