// lt_attn_block.cu — the attention half of a decoder layer for one token in
// one persistent kernel (one CTA per SM, two grid-wide hand-offs):
//
//   phase Q  every CTA stages x, normalises it (math.zig:20-26) and
//            quantises it; CTA c computes its share of the Q/K/V rows (bias
//            added, forward.zig:272-287) from weight rows it copied into
//            shared memory by TMA before waiting for the previous kernel.
//                                                      -> grid barrier
//   phase A  work item (query head h, split s): per-head Q/K RMSNorm and
//            RoPE (rope.zig, gemma4/forward.zig:267-268), the K/V append of
//            this position (by split 0 of the group's first head), and
//            online-softmax attention over the split's positions; the
//            current position's K/V come from registers, older ones from the
//            cache.  The last split of a head to finish merges the head.
//                                                      -> grid barrier
//   phase O  every CTA quantises the attention vector and computes its wo
//            rows plus the residual: out = x + wo . att (forward.zig:304-305).
//
// The weights are static, so both tiles (this CTA's Q/K/V rows and wo rows)
// stream in while the previous kernel finishes; an optional L2 prefetch
// range (the next kernel's weights) is issued at the same time.
#include "lt_qact.cuh"
#include "lt_rowdot.cuh"

namespace lt {

constexpr int kAbWarps = 16;
constexpr int kAbThreads = kAbWarps * 32;

// Layout of the context's attention sync block.
constexpr size_t kAbEpoch = 0, kAbB1 = 8, kAbB2 = 16;

struct AttnBlockArgs {
    AttnGeom g;
    uint32_t d;
    const float *x, *norm_w;
    float eps;
    const uint8_t *wqkv;
    uint64_t qpitch;
    uint32_t qrows, qnb;  // rows (nq + 2 nkv), 32-blocks per row (d / 32)
    const float *bias;    // nullable [qrows]
    const float *q_norm, *k_norm;
    const uint32_t *pos;
    float *kc, *vc;
    const uint8_t *wo;
    uint64_t opitch;
    uint32_t onb;  // 32-blocks per wo row (nq / 32)
    float *out;
    float *qkv, *part, *att;  // global scratch
    uint32_t *head_ctr;       // [n_heads], zero between launches
    uint8_t *sync;
    const uint8_t *pf[2];
    uint64_t pf_bytes[2];
    int *dev_err;
    uint32_t splits, maxq, maxo;
};

struct AbLayout {
    size_t bars, misc, wq, wo, xs, as, xf, nw, xres, head, total;
};

__host__ __device__ inline AbLayout ab_layout(const AttnBlockArgs &a) {
    AbLayout L;
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off += (b + 127) & ~(size_t)127;
        return o;
    };
    const uint32_t nq = a.g.n_heads * a.g.hd;
    L.bars = take(64);
    L.misc = take(256);
    L.wq = take((size_t)a.maxq * a.qpitch + 128);  // + slack: a Q8_0 chunk reads up to 34 bytes past a row
    L.wo = take((size_t)a.maxo * a.opitch + 128);
    L.xs = take(xs_bytes(1, (int)((a.d + 255) / 256)));
    L.as = take(xs_bytes(1, (int)((nq + 255) / 256)));
    L.xf = take((size_t)(a.d > nq ? a.d : nq) * 4);
    L.nw = take((size_t)a.d * 4);
    L.xres = take((size_t)a.maxo * 4);
    // per-item head vectors q, k, v and the warps' softmax partials
    L.head = take((size_t)(3 * a.g.hd + kAbWarps * (a.g.hd + 2)) * 4);
    L.total = off;
    return L;
}

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
    for (uint32_t b = warp; b < (n + 31) / 32; b += kAbWarps) {
        const uint32_t e = 32 * b + lane;
        qact_block_to_xs(X, 0, (int)b, e < n ? xf[e] : 0.0f, lane);
    }
}

// rows [0, nrows) of a shared tile (pitch) against X: y[r] per row, lanes own
// 64-column chunks (cb = lane, lane + 32, ...), warp w takes rows w, w+16, ...
template <uint32_t T>
LT_DEVINL void ab_rows(const uint8_t *tile, uint64_t pitch, uint32_t nrows, uint32_t cols, uint32_t nb, const XS &X,
                       int warp, int lane, float *y) {
    const uint32_t nch = (cols + 63) / 64;
    for (uint32_t r = warp; r < nrows; r += kAbWarps) {
        float acc = 0.0f;
        for (uint32_t cb = lane; cb < nch; cb += 32) {
            XChunk xc;
            xchunk_load(X, 0, (int)cb, xc);
            acc += dot64<T>(tile + (size_t)r * pitch, (int)cb, (int)nb, xc);
        }
        acc = warp_sum(acc);
        if (lane == 0) y[r] = acc;
    }
}

// Per-head RMSNorm (optional weights) and RoPE of hd values in shared memory.
LT_DEVINL void ab_norm_rope(float *v, const float *nw, const AttnGeom &g, uint32_t pos, float *red) {
    const uint32_t hd = g.hd, half = hd / 2;
    if (nw) {
        float ss = 0.0f;
        for (uint32_t i = threadIdx.x; i < hd; i += kAbThreads) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
        ss = ab_block_sum(ss, red);
        const float rms_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), g.eps)));
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < hd; i += kAbThreads) v[i] = __fmul_rn(__fmul_rn(v[i], rms_inv), nw[i]);
    }
    __syncthreads();
    float r0 = 0.0f, r1 = 0.0f;
    uint32_t i0 = 0, i1 = 0;
    const bool act = threadIdx.x < half;
    if (act) {
        const uint32_t i = threadIdx.x;
        const float ang = __fmul_rn((float)pos, __fdiv_rn(1.0f, powf(g.theta, __fdiv_rn((float)(2 * i), (float)hd))));
        float s, c;
        sincosf(ang, &s, &c);
        i0 = g.rope_neox ? i : 2 * i;
        i1 = g.rope_neox ? i + half : 2 * i + 1;
        const float x0 = v[i0], x1 = v[i1];
        r0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        r1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    __syncthreads();
    if (act) {
        v[i0] = r0;
        v[i1] = r1;
    }
    __syncthreads();
}

template <uint32_t QT, uint32_t OT, int HD>
__global__ void __launch_bounds__(kAbThreads, 1) k_attn_block(AttnBlockArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int PER = HD / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t G = gridDim.x, c = blockIdx.x;
    const AbLayout L = ab_layout(a);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    float *red = reinterpret_cast<float *>(smem + L.misc);            // [16]
    uint64_t *s_epoch = reinterpret_cast<uint64_t *>(smem + L.misc + 64);
    int *s_flag = reinterpret_cast<int *>(smem + L.misc + 72);
    uint8_t *wq = smem + L.wq, *wo = smem + L.wo;
    const XS Xx = xs_carve(smem + L.xs, 1, (int)((a.d + 255) / 256));
    const uint32_t nq = a.g.n_heads * HD, nkv = a.g.n_kv * HD;
    const XS Xa = xs_carve(smem + L.as, 1, (int)((nq + 255) / 256));
    float *xf = reinterpret_cast<float *>(smem + L.xf);
    float *nw = reinterpret_cast<float *>(smem + L.nw);
    float *xres = reinterpret_cast<float *>(smem + L.xres);
    float *hq = reinterpret_cast<float *>(smem + L.head), *hk = hq + HD, *hv = hk + HD;
    float *wpart = hv + HD;  // [16][HD + 2]: m, l, o[HD]
    unsigned long long *ctr_epoch = reinterpret_cast<unsigned long long *>(a.sync + kAbEpoch);
    unsigned long long *ctr1 = reinterpret_cast<unsigned long long *>(a.sync + kAbB1);
    unsigned long long *ctr2 = reinterpret_cast<unsigned long long *>(a.sync + kAbB2);

    const uint32_t q0 = (uint32_t)((uint64_t)c * a.qrows / G), q1 = (uint32_t)((uint64_t)(c + 1) * a.qrows / G);
    const uint32_t o0 = (uint32_t)((uint64_t)c * a.d / G), o1 = (uint32_t)((uint64_t)(c + 1) * a.d / G);
    const uint32_t nqr = q1 - q0, nor = o1 - o0;

    // static inputs first: both weight tiles, the norm weights, the L2 prefetch
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_barrier_init();
        if (nqr) {
            mbar_arrive_expect_tx(&bars[0], (uint32_t)(nqr * a.qpitch));
            tma_load_1d(wq, a.wqkv + (uint64_t)q0 * a.qpitch, (uint32_t)(nqr * a.qpitch), &bars[0]);
        }
        if (nor) {
            mbar_arrive_expect_tx(&bars[1], (uint32_t)(nor * a.opitch));
            tma_load_1d(wo, a.wo + (uint64_t)o0 * a.opitch, (uint32_t)(nor * a.opitch), &bars[1]);
        }
    }
    if (tid < 2 && a.pf[tid]) prefetch_l2_share(a.pf[tid], a.pf_bytes[tid], c, G);
    for (uint32_t i = tid; i < a.d; i += kAbThreads) nw[i] = __ldg(a.norm_w + i);
    pdl_launch_dependents();
    pdl_wait();

    // ── phase Q ──────────────────────────────────────────────────────────────
    if (tid == 0) *s_epoch = grid_epoch(ctr_epoch, G);
    const uint32_t pos = *a.pos;
    for (uint32_t i = tid; i < a.d; i += kAbThreads) xf[i] = __ldcg(a.x + i);
    __syncthreads();
    for (uint32_t r = tid; r < nor; r += kAbThreads) xres[r] = xf[o0 + r];
    {
        float ss = 0.0f;
        for (uint32_t i = tid; i < a.d; i += kAbThreads) ss += xf[i] * xf[i];
        ss = ab_block_sum(ss, red);
        const float rms_inv = 1.0f / sqrtf(ss / (float)a.d + a.eps);
        for (uint32_t i = tid; i < a.d; i += kAbThreads) xf[i] = xf[i] * rms_inv * nw[i];
    }
    __syncthreads();
    ab_quantise(Xx, xf, a.d, warp, lane);
    __syncthreads();
    const uint64_t epoch = *s_epoch;
    float *yq = xf;  // the normalised x is quantised already
    if (nqr && tile_wait(&bars[0], a.dev_err)) ab_rows<QT>(wq, a.qpitch, nqr, a.d, a.qnb, Xx, warp, lane, yq);
    __syncthreads();
    for (uint32_t r = tid; r < nqr; r += kAbThreads)
        a.qkv[q0 + r] = a.bias ? __fadd_rn(yq[r], a.bias[q0 + r]) : yq[r];
    grid_arrive(ctr1);
    grid_wait(ctr1, epoch, a.dev_err, kWaitLimitNs);

    // ── phase A ──────────────────────────────────────────────────────────────
    const uint32_t S = a.splits, group = a.g.n_heads / a.g.n_kv;
    const uint32_t seq = pos + 1, win = a.g.window ? min(seq, a.g.window) : seq, first = seq - win;
    for (uint32_t item = c; item < a.g.n_heads * S; item += G) {
        const uint32_t h = item / S, s = item - h * S, kh = h / group;
        for (uint32_t i = tid; i < HD; i += kAbThreads) {
            hq[i] = __ldcg(a.qkv + h * HD + i);
            hk[i] = __ldcg(a.qkv + nq + kh * HD + i);
            hv[i] = __ldcg(a.qkv + nq + nkv + kh * HD + i);
        }
        __syncthreads();
        ab_norm_rope(hq, a.q_norm, a.g, pos, red);
        ab_norm_rope(hk, a.k_norm, a.g, pos, red);
        if (s == 0 && h % group == 0) {  // this position's K/V into the cache
            const size_t slot = (size_t)(pos % a.g.cap) * nkv + (size_t)kh * HD;
            for (uint32_t i = tid; i < HD; i += kAbThreads) {
                a.kc[slot + i] = hk[i];
                a.vc[slot + i] = hv[i];
            }
        }
        float qv[PER], o[PER];
#pragma unroll
        for (int i = 0; i < PER; i++) {
            qv[i] = hq[lane + 32 * i];
            o[i] = 0.0f;
        }
        float m = -INFINITY, l = 0.0f;
        for (uint32_t j = s * kAbWarps + warp; j < win; j += S * kAbWarps) {
            float kv[PER], vv[PER];
            if (j == win - 1) {  // the current position
#pragma unroll
                for (int i = 0; i < PER; i++) {
                    kv[i] = hk[lane + 32 * i];
                    vv[i] = hv[lane + 32 * i];
                }
            } else {
                const size_t slot = (size_t)((first + j) % a.g.cap) * nkv + (size_t)kh * HD;
#pragma unroll
                for (int i = 0; i < PER; i++) {
                    kv[i] = a.kc[slot + lane + 32 * i];
                    vv[i] = a.vc[slot + lane + 32 * i];
                }
            }
            float dot = 0.0f;
#pragma unroll
            for (int i = 0; i < PER; i++) dot = fmaf(qv[i], kv[i], dot);
            dot = warp_sum(dot);
            const float sc = dot * a.g.scale;
            const float mn = fmaxf(m, sc);
            const float al = expf(m - mn), p = expf(sc - mn);
            l = l * al + p;
#pragma unroll
            for (int i = 0; i < PER; i++) o[i] = fmaf(p, vv[i], o[i] * al);
            m = mn;
        }
        float *wp = wpart + warp * (HD + 2);
        if (lane == 0) {
            wp[0] = m;
            wp[1] = l;
        }
#pragma unroll
        for (int i = 0; i < PER; i++) wp[2 + lane + 32 * i] = o[i];
        __syncthreads();
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAbWarps; w++) M = fmaxf(M, wpart[w * (HD + 2)]);
        float *pp = a.part + ((size_t)h * S + s) * (HD + 2);
        for (uint32_t t = tid; t < HD; t += kAbThreads) {
            float acc = 0.0f;
#pragma unroll
            for (int w = 0; w < kAbWarps; w++) {
                const float mw = wpart[w * (HD + 2)];
                if (mw != -INFINITY) acc += wpart[w * (HD + 2) + 2 + t] * expf(mw - M);
            }
            pp[2 + t] = acc;
        }
        if (tid == 0) {
            float Lsum = 0.0f;
            for (int w = 0; w < kAbWarps; w++) {
                const float mw = wpart[w * (HD + 2)];
                if (mw != -INFINITY) Lsum += wpart[w * (HD + 2) + 1] * expf(mw - M);
            }
            pp[0] = M;
            pp[1] = Lsum;
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) *s_flag = atomicAdd(&a.head_ctr[h], 1u) == S - 1;
        __syncthreads();
        if (*s_flag) {  // the last split of head h merges it
            __threadfence();
            const float *hp = a.part + (size_t)h * S * (HD + 2);
            float GM = -INFINITY;
            for (uint32_t k = 0; k < S; k++) GM = fmaxf(GM, __ldcg(hp + k * (HD + 2)));
            float GL = 0.0f;
            for (uint32_t k = 0; k < S; k++) {
                const float mk = __ldcg(hp + k * (HD + 2));
                if (mk != -INFINITY) GL += __ldcg(hp + k * (HD + 2) + 1) * expf(mk - GM);
            }
            for (uint32_t t = tid; t < HD; t += kAbThreads) {
                float acc = 0.0f;
                for (uint32_t k = 0; k < S; k++) {
                    const float mk = __ldcg(hp + k * (HD + 2));
                    if (mk != -INFINITY) acc += __ldcg(hp + k * (HD + 2) + 2 + t) * expf(mk - GM);
                }
                a.att[h * HD + t] = acc / GL;
            }
            if (tid == 0) a.head_ctr[h] = 0;
        }
        __syncthreads();
    }
    grid_arrive(ctr2);
    grid_wait(ctr2, epoch, a.dev_err, kWaitLimitNs);

    // ── phase O ──────────────────────────────────────────────────────────────
    for (uint32_t i = tid; i < nq; i += kAbThreads) xf[i] = __ldcg(a.att + i);
    __syncthreads();
    ab_quantise(Xa, xf, nq, warp, lane);
    __syncthreads();
    float *yo = xf;  // the attention vector is quantised already
    if (nor && tile_wait(&bars[1], a.dev_err)) ab_rows<OT>(wo, a.opitch, nor, nq, a.onb, Xa, warp, lane, yo);
    __syncthreads();
    for (uint32_t r = tid; r < nor; r += kAbThreads) a.out[o0 + r] = __fadd_rn(xres[r], yo[r]);
}

bool attn_block_supported(const AttnGeom &g, const DevMat &wqkv, const DevMat &wo, uint32_t d) {
    auto ok_type = [](uint32_t t) { return t == T_Q8_0 || t == T_Q4_K || t == T_Q6_K; };
    if (!ok_type(wqkv.type) || !ok_type(wo.type)) return false;
    if (g.hd != 64 && g.hd != 128 && g.hd != 256) return false;
    if (wqkv.cols != d || wqkv.rows != (uint64_t)(g.n_heads + 2 * g.n_kv) * g.hd) return false;
    if (wo.rows != d || wo.cols != (uint64_t)g.n_heads * g.hd) return false;
    return d % 32 == 0 && d <= 8192 && wo.cols <= 16384;
}

static AttnBlockArgs ab_args(const AttnGeom &g, int num_sms, uint32_t d, const DevMat &wqkv, const DevMat &wo) {
    AttnBlockArgs a{};
    a.g = g;
    a.d = d;
    a.qpitch = wqkv.pitch;
    a.qrows = (uint32_t)wqkv.rows;
    a.qnb = (uint32_t)(wqkv.cols / 32);
    a.opitch = wo.pitch;
    a.onb = (uint32_t)(wo.cols / 32);
    const uint32_t G = (uint32_t)num_sms;
    a.splits = max(1u, G / g.n_heads);
    a.maxq = (a.qrows + G - 1) / G;
    a.maxo = (d + G - 1) / G;
    return a;
}

size_t attn_block_smem(const AttnGeom &g, int num_sms, uint32_t d, const DevMat &wqkv, const DevMat &wo) {
    return ab_layout(ab_args(g, num_sms, d, wqkv, wo)).total;
}

size_t attn_block_scratch_floats(const AttnGeom &g, int num_sms, uint32_t d, const DevMat &wqkv, const DevMat &wo) {
    const AttnBlockArgs a = ab_args(g, num_sms, d, wqkv, wo);
    return (size_t)a.qrows + (size_t)g.n_heads * a.splits * (g.hd + 2) + (size_t)g.n_heads * g.hd + 64;
}

template <uint32_t QT, uint32_t OT>
static cudaError_t launch_ab_t(const LaunchCfg &c, const AttnBlockArgs &a, size_t smem) {
    switch (a.g.hd) {
    case 64: return launch_k(c, "attn_block", k_attn_block<QT, OT, 64>, dim3(c.num_sms), dim3(kAbThreads), smem, a);
    case 128: return launch_k(c, "attn_block", k_attn_block<QT, OT, 128>, dim3(c.num_sms), dim3(kAbThreads), smem, a);
    case 256: return launch_k(c, "attn_block", k_attn_block<QT, OT, 256>, dim3(c.num_sms), dim3(kAbThreads), smem, a);
    default: return cudaErrorInvalidValue;
    }
}

template <uint32_t QT>
static cudaError_t launch_ab_q(const LaunchCfg &c, const AttnBlockArgs &a, size_t smem, uint32_t ot) {
    switch (ot) {
    case T_Q8_0: return launch_ab_t<QT, T_Q8_0>(c, a, smem);
    case T_Q4_K: return launch_ab_t<QT, T_Q4_K>(c, a, smem);
    case T_Q6_K: return launch_ab_t<QT, T_Q6_K>(c, a, smem);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_attn_block(const LaunchCfg &c, const AttnBlockParams &p) {
    AttnBlockArgs a = ab_args(p.g, c.num_sms, p.d, p.wqkv, p.wo);
    a.x = p.x;
    a.norm_w = p.norm_w;
    a.eps = p.eps;
    a.wqkv = p.wqkv.data;
    a.bias = p.bias;
    a.q_norm = p.q_norm;
    a.k_norm = p.k_norm;
    a.pos = p.pos;
    a.kc = p.kc;
    a.vc = p.vc;
    a.wo = p.wo.data;
    a.out = p.out;
    float *sc = p.scratch;
    a.qkv = sc;
    a.part = sc + ((a.qrows + 31) & ~31u);
    a.att = a.part + (((size_t)p.g.n_heads * a.splits * (p.g.hd + 2) + 31) & ~(size_t)31);
    a.head_ctr = p.head_ctr;
    a.sync = p.sync;
    for (int i = 0; i < 2; i++) {
        a.pf[i] = p.pf[i];
        a.pf_bytes[i] = p.pf_bytes[i];
    }
    a.dev_err = c.dev_err;
    const size_t smem = ab_layout(a).total;
    if (smem > kDecodeSmemLimit) return cudaErrorInvalidValue;
    switch (p.wqkv.type) {
    case T_Q8_0: return launch_ab_q<T_Q8_0>(c, a, smem, p.wo.type);
    case T_Q4_K: return launch_ab_q<T_Q4_K>(c, a, smem, p.wo.type);
    case T_Q6_K: return launch_ab_q<T_Q6_K>(c, a, smem, p.wo.type);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace lt
