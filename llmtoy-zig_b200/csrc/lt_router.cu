// lt_router.cu — MoE router: routerTopKSoftmax (src/model/gemma4/forward.zig:
// 648-668) with the pre-FFN RMSNorm (src/ops/math.zig:20-26) and the
// activation quantisation for the expert kernels fused in.
//
// Each warp computes one expert's logit (router_logit, lt_router.cuh: dotf32's
// exact order).  The last CTA of each token group selects the top-k and the
// softmax weights (lt_router.cuh).
#include "lt_qact.cuh"
#include "lt_router.cuh"

namespace lt {

constexpr int kRouterWarps = 8;  // experts per CTA
constexpr int kRouterTok = 4;    // tokens per CTA (one warp each for the top-k)
constexpr int kRouterNormThreads = 128;  // RMSNorm reduction width (the decode kernel uses the same)

uint32_t router_token_groups(uint32_t ntok) { return (ntok + kRouterTok - 1) / kRouterTok; }

struct RouterArgs {
    const float *W;  // [E][w_ld]
    uint32_t E, cols, w_ld;
    const float *x;       // [ntok][cols]
    const float *norm_w;  // nullable: route rmsnorm(x) * norm_w instead of x
    float eps;
    uint32_t ntok, k;
    int norm_topk;
    const float *escale;
    uint32_t *ids;
    float *wout;
    float *logits;  // [ntok][E] scratch
    uint32_t *counters;
    uint8_t *xq;  // nullable: qact rows of the (normalised) input for the experts
    uint64_t xq_pitch;
    float *xn;  // nullable: f32 rows of the (normalised) input, written by the CTAs of blockIdx.x == 0
};

__global__ void __launch_bounds__(kRouterWarps * 32) k_router(RouterArgs a) {
    extern __shared__ __align__(16) float xsm[];  // [kRouterTok][cols] x, then [cols] norm weights
    __shared__ int s_last;
    __shared__ float s_ss[kRouterWarps][kRouterTok];
    __shared__ float s_rms[kRouterTok];
    __shared__ uint32_t s_sel[kRouterTok][16];
    __shared__ float s_mx[kRouterTok], s_es[kRouterTok];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t e = blockIdx.x * kRouterWarps + warp;
    const uint32_t t0 = blockIdx.y * kRouterTok;
    const uint32_t nt = min((uint32_t)kRouterTok, a.ntok - t0);
    const uint32_t cols = a.cols, n32 = cols & ~31u;
    float *nwsm = xsm + kRouterTok * cols;
    // router and norm weights are static: fetch them while the producer of x finishes
    float w0[kRouterChunk];
#pragma unroll
    for (int j = 0; j < kRouterChunk; j++)
        w0[j] = (e < a.E && 32u * j < n32) ? __ldg(a.W + (size_t)e * a.w_ld + 32 * j + lane) : 0.0f;
    if (a.norm_w) {
        if ((cols & 3) == 0 && (reinterpret_cast<uintptr_t>(a.norm_w) & 15) == 0) {
#pragma unroll 8
            for (uint32_t i = threadIdx.x; i < cols / 4; i += blockDim.x)
                reinterpret_cast<float4 *>(nwsm)[i] = __ldg(reinterpret_cast<const float4 *>(a.norm_w) + i);
        } else {
#pragma unroll 8
            for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) nwsm[i] = __ldg(a.norm_w + i);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    {
        const float *xt = a.x + (size_t)t0 * cols;
        const uint32_t n = nt * cols;
        if ((cols & 3) == 0 && (reinterpret_cast<uintptr_t>(xt) & 15) == 0) {
#pragma unroll 8
            for (uint32_t i = threadIdx.x; i < n / 4; i += blockDim.x)
                reinterpret_cast<float4 *>(xsm)[i] = reinterpret_cast<const float4 *>(xt)[i];
        } else {
#pragma unroll 8
            for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) xsm[i] = xt[i];
        }
    }
    __syncthreads();
    if (a.norm_w) {  // rmsnorm(out, x, w, eps): x * (1/sqrt(ss/n + eps)) * w
        float ss[kRouterTok];
#pragma unroll
        for (int tt = 0; tt < kRouterTok; tt++) {
            ss[tt] = 0.0f;
            if (tt < (int)nt && threadIdx.x < kRouterNormThreads)
                for (uint32_t i = threadIdx.x; i < cols; i += kRouterNormThreads)
                    ss[tt] += xsm[tt * cols + i] * xsm[tt * cols + i];
            ss[tt] = warp_sum(ss[tt]);
        }
        if (lane == 0 && warp < kRouterNormThreads / 32)
#pragma unroll
            for (int tt = 0; tt < kRouterTok; tt++) s_ss[warp][tt] = ss[tt];
        __syncthreads();
        if (threadIdx.x < nt) {
            float s = 0.0f;
            for (int w = 0; w < kRouterNormThreads / 32; w++) s += s_ss[w][threadIdx.x];
            s_rms[threadIdx.x] = 1.0f / sqrtf(s / (float)cols + a.eps);
        }
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < nt * cols; i += blockDim.x) {
            const uint32_t tt = i / cols, c = i - tt * cols;
            xsm[i] = xsm[i] * s_rms[tt] * nwsm[c];
        }
        __syncthreads();
    }
    if (a.xn && blockIdx.x == 0)
        for (uint32_t i = threadIdx.x; i < nt * cols; i += blockDim.x) a.xn[(size_t)t0 * cols + i] = xsm[i];
    if (a.xq) {  // quantise this CTA's share of the 32-blocks for the expert kernels
        const uint32_t nblk = cols / 32;
        for (uint32_t task = blockIdx.x * kRouterWarps + warp; task < nt * nblk; task += gridDim.x * kRouterWarps) {
            const uint32_t tt = task / nblk, b = task - tt * nblk;
            qact_store_block(a.xq + (size_t)(t0 + tt) * a.xq_pitch, (int)cols, (int)b, xsm[tt * cols + 32 * b + lane],
                             lane);
        }
    }
    if (e < a.E) {
        for (uint32_t tt = 0; tt < nt; tt++) {
            const float v = router_logit(a.W + (size_t)e * a.w_ld, xsm + tt * cols, cols, lane, w0);
            if (lane == 0) a.logits[(size_t)(t0 + tt) * a.E + e] = v;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t ticket = atomicAdd(&a.counters[blockIdx.y], 1u);
        s_last = ticket == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // top-k + softmax weights per token (lt_router.cuh); x is no longer needed,
    // its shared memory holds the logits and sort keys
    float(*s_lg)[kRouterMaxE] = reinterpret_cast<float(*)[kRouterMaxE]>(xsm);
    uint64_t(*s_key)[kRouterMaxE + 2] =
        reinterpret_cast<uint64_t(*)[kRouterMaxE + 2]>(xsm + kRouterTok * kRouterMaxE);
    for (uint32_t i = threadIdx.x; i < nt * a.E; i += blockDim.x) {
        const uint32_t tt = i / a.E, ee = i - tt * a.E;
        const float v = __ldcg(a.logits + (size_t)(t0 + tt) * a.E + ee);
        s_lg[tt][ee] = v;
        s_key[tt][ee] = router_key(v, ee);
    }
    if (threadIdx.x < nt) s_key[threadIdx.x][a.E] = 0;
    __syncthreads();
    for (uint32_t tt = 0; tt < nt; tt++) router_rank_keys(s_key[tt], a.E, a.k, s_sel[tt], threadIdx.x, blockDim.x);
    if (warp < (int)nt) {
        float mx, es;
        router_softmax_stats(s_lg[warp], a.E, lane, mx, es);
        if (lane == 0) {
            s_mx[warp] = mx;
            s_es[warp] = es;
        }
    }
    __syncthreads();
    if (threadIdx.x < nt) {
        const uint32_t tt = threadIdx.x;
        float w[16];
        router_weights(s_lg[tt], s_sel[tt], a.k, s_mx[tt], s_es[tt], a.norm_topk, a.escale, w);
        for (uint32_t i = 0; i < a.k; i++) {
            a.ids[(size_t)(t0 + tt) * a.k + i] = s_sel[tt][i];
            a.wout[(size_t)(t0 + tt) * a.k + i] = w[i];
        }
    }
    if (threadIdx.x == 0) a.counters[blockIdx.y] = 0;
}

// Token-major router for large batches: a CTA owns kRtTok tokens and computes
// all E logits for them, 8 experts at a time with each warp's router row in
// registers reused across the tokens, then ranks them itself.  Per token the
// arithmetic is the expert-major kernel's (the same norm reduction order, the
// same router_logit, ranking and weights), so the ids and weights are
// identical; the router weights are read once per kRtTok tokens instead of
// once per 4, and no logits go through global memory.
constexpr int kRtWarps = 8;
constexpr int kRtTok = 8;
constexpr uint32_t kRtMinTokens = 32;  // smaller batches: the expert-major kernel (more CTAs)
constexpr uint32_t kRtMaxCols = 4096;

// Shared-memory layout (byte offsets, 16-byte aligned): x rows, norm
// weights, logits, sort keys with an even row stride of at least E + 2 so
// that every row starts 16-byte aligned (router_rank_keys loads key pairs).
struct RtLayout {
    size_t nw, lg, keys, total;
    uint32_t kstride;
};
__host__ __device__ inline RtLayout rt_layout(uint32_t cols, uint32_t E) {
    auto al = [](size_t v) { return (v + 15) & ~(size_t)15; };
    RtLayout L;
    L.kstride = (E + 3) & ~1u;
    L.nw = al((size_t)kRtTok * cols * 4);
    L.lg = al(L.nw + (size_t)cols * 4);
    L.keys = al(L.lg + (size_t)kRtTok * E * 4);
    L.total = L.keys + (size_t)kRtTok * L.kstride * 8;
    return L;
}

__global__ void __launch_bounds__(kRtWarps * 32, 2) k_router_tok(RouterArgs a) {
    extern __shared__ __align__(16) float rsm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t cols = a.cols, E = a.E;
    const uint32_t t0 = blockIdx.x * kRtTok;
    const uint32_t nt = min((uint32_t)kRtTok, a.ntok - t0);
    const RtLayout Lr = rt_layout(cols, E);
    uint8_t *base = reinterpret_cast<uint8_t *>(rsm);
    float *xs = rsm;                                           // [kRtTok][cols]
    float *nwsm = reinterpret_cast<float *>(base + Lr.nw);     // [cols]
    float *lg = reinterpret_cast<float *>(base + Lr.lg);       // [kRtTok][E]
    uint64_t *keys = reinterpret_cast<uint64_t *>(base + Lr.keys);  // [kRtTok][Lr.kstride], 16-byte aligned rows
    __shared__ float s_ss[kRtWarps];
    __shared__ float s_rms[kRtTok];
    __shared__ uint32_t s_sel[kRtTok][16];
    __shared__ float s_mx[kRtTok], s_es[kRtTok];
    if (a.norm_w)
        for (uint32_t i = tid; i < cols; i += kRtWarps * 32) nwsm[i] = __ldg(a.norm_w + i);
    pdl_launch_dependents();
    pdl_wait();
    {
        const float *xt = a.x + (size_t)t0 * cols;
        const uint32_t n = nt * cols;
        if ((cols & 3) == 0 && (reinterpret_cast<uintptr_t>(xt) & 15) == 0) {
#pragma unroll 8
            for (uint32_t i = tid; i < n / 4; i += kRtWarps * 32)
                reinterpret_cast<float4 *>(xs)[i] = reinterpret_cast<const float4 *>(xt)[i];
        } else {
            for (uint32_t i = tid; i < n; i += kRtWarps * 32) xs[i] = xt[i];
        }
    }
    __syncthreads();
    if (a.norm_w) {
        // the expert-major kernel's order: per token, 128 threads stride the
        // columns, then their 4 warp sums in order; two tokens at a time here
        constexpr int G = kRtWarps * 32 / kRouterNormThreads;
        for (uint32_t base = 0; base < nt; base += G) {
            const uint32_t g = tid / kRouterNormThreads, tt = base + g, ti = tid % kRouterNormThreads;
            float ss = 0.0f;
            if (tt < nt)
                for (uint32_t i = ti; i < cols; i += kRouterNormThreads) ss += xs[tt * cols + i] * xs[tt * cols + i];
            ss = warp_sum(ss);
            if (lane == 0) s_ss[warp] = ss;
            __syncthreads();
            if (ti == 0 && tt < nt) {
                float sum = 0.0f;
                for (int w = 0; w < kRouterNormThreads / 32; w++) sum += s_ss[g * (kRouterNormThreads / 32) + w];
                s_rms[tt] = 1.0f / sqrtf(sum / (float)cols + a.eps);
            }
            __syncthreads();
        }
        for (uint32_t i = tid; i < nt * cols; i += kRtWarps * 32) {
            const uint32_t tt = i / cols, cc = i - tt * cols;
            xs[i] = xs[i] * s_rms[tt] * nwsm[cc];
        }
        __syncthreads();
    }
    if (a.xn)
        for (uint32_t i = tid; i < nt * cols; i += kRtWarps * 32) a.xn[(size_t)t0 * cols + i] = xs[i];
    if (a.xq) {
        const uint32_t nblk = cols / 32;
        for (uint32_t task = warp; task < nt * nblk; task += kRtWarps) {
            const uint32_t tt = task / nblk, b = task - tt * nblk;
            qact_store_block(a.xq + (size_t)(t0 + tt) * a.xq_pitch, (int)cols, (int)b, xs[tt * cols + 32 * b + lane],
                             lane);
        }
    }
    for (uint32_t e0 = 0; e0 < E; e0 += kRtWarps) {
        const uint32_t e = e0 + warp;
        if (e < E) {
            float w0[kRouterChunk];
            router_prefetch(a.W + (size_t)e * a.w_ld, cols, lane, true, w0);
            for (uint32_t tt = 0; tt < nt; tt++) {
                const float v = router_logit(a.W + (size_t)e * a.w_ld, xs + tt * cols, cols, lane, w0);
                if (lane == 0) lg[tt * E + e] = v;
            }
        }
    }
    __syncthreads();
    const uint32_t E2 = Lr.kstride;
    for (uint32_t i = tid; i < nt * E; i += kRtWarps * 32) {
        const uint32_t tt = i / E, ee = i - tt * E;
        keys[tt * E2 + ee] = router_key(lg[i], ee);
    }
    if ((uint32_t)tid < nt) keys[tid * E2 + E] = 0;
    __syncthreads();
    {  // rank: one group of kRouterNormThreads threads per token at a time
        constexpr int G = kRtWarps * 32 / kRouterNormThreads;
        const uint32_t g = tid / kRouterNormThreads, ti = tid % kRouterNormThreads;
        for (uint32_t base = 0; base < nt; base += G)
            if (base + g < nt)
                router_rank_keys(keys + (base + g) * E2, E, a.k, s_sel[base + g], (int)ti, kRouterNormThreads);
    }
    for (uint32_t tt = warp; tt < nt; tt += kRtWarps) {
        float mx, es;
        router_softmax_stats(lg + tt * E, E, lane, mx, es);
        if (lane == 0) {
            s_mx[tt] = mx;
            s_es[tt] = es;
        }
    }
    __syncthreads();
    if ((uint32_t)tid < nt) {
        const uint32_t tt = tid;
        float w[16];
        router_weights(lg + tt * E, s_sel[tt], a.k, s_mx[tt], s_es[tt], a.norm_topk, a.escale, w);
        for (uint32_t i = 0; i < a.k; i++) {
            a.ids[(size_t)(t0 + tt) * a.k + i] = s_sel[tt][i];
            a.wout[(size_t)(t0 + tt) * a.k + i] = w[i];
        }
    }
}

// Register-tiled token-major router for large batches.  dotf32's order makes
// each logit 32 independent chains (lane l sums w[l + 32j] * x[l + 32j] over
// j in order), combined in a fixed order at the end; every chain is an
// ordinary sequential accumulation, so a CTA can compute the logits of a
// tile of TC tokens x EC experts like a GEMM with K split into 32 residue
// classes: thread (warp, lane l) holds the chains of residue l for 8 tokens
// x 8 experts in registers, and each 32-column step costs 16 shared-memory
// loads for 64 multiply-adds (k_router_tok: one load per multiply-add, one
// chain per warp).  x and the router rows stream through two stages of
// 256 columns by cp.async; the chains are combined through shared memory in
// router_logit's order; the last of a token tile's expert-group CTAs ranks
// the tile's tokens with the shared ranking and weight code.  The norm, the
// quantised / f32 rows and every result equal k_router_tok's bit for bit.
constexpr int kRmTT = 8, kRmEE = 8;  // tokens x experts per thread
constexpr uint32_t kRmKC = 256;      // columns per stage (8 steps of 32)
constexpr int kRmNorm = 128;         // threads per token of the norm reduction (kRouterNormThreads)

template <int WT, int WE>
struct RmGeo {
    static constexpr int NT = WT * WE * 32;
    static constexpr int TC = WT * kRmTT, EC = WE * kRmEE;
    static constexpr size_t kStage = (size_t)(TC + EC + 1) * kRmKC;  // floats per stage: x, router rows, norm weights
    static constexpr size_t kSmem = 2 * kStage * 4;
};

namespace {
LT_DEVINL void rm_cp16(float *dst_smem, const float *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst_smem)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
LT_DEVINL void rm_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
LT_DEVINL void rm_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
}  // namespace

template <int WT, int WE>
__global__ void __launch_bounds__(WT *WE * 32, WT *WE <= 8 ? 2 : 1) k_router_mm(RouterArgs a) {
    using Gm = RmGeo<WT, WE>;
    constexpr int NT = Gm::NT, TC = Gm::TC, EC = Gm::EC;
    constexpr int NG = NT / kRmNorm;  // tokens normalised at once
    extern __shared__ __align__(16) float msm[];
    __shared__ float s_part[TC][kRmNorm / 32];
    __shared__ float s_rms[TC];
    __shared__ uint32_t s_sel[TC][16];
    __shared__ float s_mx[TC], s_es[TC];
    __shared__ int s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t cols = a.cols, E = a.E;
    const uint32_t e0 = blockIdx.x * EC, t0 = blockIdx.y * TC;
    const uint32_t nt = min((uint32_t)TC, a.ntok - t0);
    const uint32_t wt = (uint32_t)warp / WE, we = (uint32_t)warp % WE;
    const uint32_t nchunks = (cols + kRmKC - 1) / kRmKC;
    auto sx = [&](uint32_t st) { return msm + st * Gm::kStage; };
    auto sw = [&](uint32_t st) { return msm + st * Gm::kStage + (size_t)TC * kRmKC; };
    auto sn = [&](uint32_t st) { return msm + st * Gm::kStage + (size_t)(TC + EC) * kRmKC; };
    // chunk ch into stage ch & 1: x rows past the batch and router rows past E read as zeros
    auto issue = [&](uint32_t ch) {
        constexpr uint32_t Q = kRmKC / 4;  // 16-byte pieces of a full chunk row
        const uint32_t c0 = ch * kRmKC, q = min(kRmKC, cols - c0) / 4;
        float *xs = sx(ch & 1), *ws = sw(ch & 1);
#pragma unroll
        for (uint32_t i = tid; i < TC * Q; i += NT) {
            const uint32_t r = i / Q, p = i % Q;
            const bool ok = r < nt;
            if (p < q)
                rm_cp16(xs + r * kRmKC + 4 * p, a.x + (size_t)(t0 + (ok ? r : 0)) * cols + c0 + 4 * p, ok ? 16u : 0u);
        }
#pragma unroll
        for (uint32_t i = tid; i < EC * Q; i += NT) {
            const uint32_t r = i / Q, p = i % Q;
            const bool ok = e0 + r < E;
            if (p < q)
                rm_cp16(ws + r * kRmKC + 4 * p, a.W + (size_t)(ok ? e0 + r : 0) * a.w_ld + c0 + 4 * p, ok ? 16u : 0u);
        }
        if (a.norm_w && (uint32_t)tid < q) rm_cp16(sn(ch & 1) + 4 * tid, a.norm_w + c0 + 4 * tid, 16u);
        rm_commit();
    };
    pdl_launch_dependents();
    pdl_wait();
    issue(0);
    if (nchunks > 1) issue(1);
    if (a.norm_w) {
        // k_router_tok's reduction: per token, 128 threads stride the columns,
        // then their 4 warp sums in order (here every token of the tile at once)
        const uint32_t g = (uint32_t)tid / kRmNorm, ti = (uint32_t)tid % kRmNorm;
        constexpr int TPG = TC / NG;  // tokens per thread
        const float *xb = a.x + (size_t)t0 * cols;
        float ss[TPG];
#pragma unroll
        for (int k = 0; k < TPG; k++) ss[k] = 0.0f;
        for (uint32_t i0 = ti; i0 < cols; i0 += 4 * kRmNorm) {  // four strides' loads in flight, then the sums in order
            float v[4][TPG];
#pragma unroll
            for (int u = 0; u < 4; u++)
#pragma unroll
                for (int k = 0; k < TPG; k++) {
                    const uint32_t tt = g + (uint32_t)k * NG, i = i0 + (uint32_t)u * kRmNorm;
                    v[u][k] = tt < nt && i < cols ? __ldg(xb + (size_t)tt * cols + i) : 0.0f;
                }
#pragma unroll
            for (int u = 0; u < 4; u++)
#pragma unroll
                for (int k = 0; k < TPG; k++)
                    if (i0 + (uint32_t)u * kRmNorm < cols) ss[k] += v[u][k] * v[u][k];
        }
#pragma unroll
        for (int k = 0; k < TC / NG; k++) {
            const float s = warp_sum(ss[k]);
            if (lane == 0) s_part[g + k * NG][ti / 32] = s;
        }
        __syncthreads();
        if ((uint32_t)tid < nt) {
            float sum = 0.0f;
            for (int w = 0; w < kRmNorm / 32; w++) sum += s_part[tid][w];
            s_rms[tid] = 1.0f / sqrtf(sum / (float)cols + a.eps);
        }
    }
    float acc[kRmTT][kRmEE];
#pragma unroll
    for (int i = 0; i < kRmTT; i++)
#pragma unroll
        for (int j = 0; j < kRmEE; j++) acc[i][j] = 0.0f;
    for (uint32_t ch = 0; ch < nchunks; ch++) {
        if (ch + 1 < nchunks)
            rm_wait<1>();
        else
            rm_wait<0>();
        __syncthreads();
        float *xs = sx(ch & 1);
        const float *ws = sw(ch & 1);
        const uint32_t c0 = ch * kRmKC, cw = min(kRmKC, cols - c0);
        if (a.norm_w || (blockIdx.x == 0 && (a.xn || a.xq))) {
            constexpr uint32_t Q = kRmKC / 4;
            if (a.norm_w) {  // x * rms * w per element, four at a time
                const float4 *nws = reinterpret_cast<const float4 *>(sn(ch & 1));
#pragma unroll
                for (uint32_t i = tid; i < TC * Q; i += NT) {
                    const uint32_t tt = i / Q, p = i % Q;
                    if (tt < nt && 4 * p < cw) {
                        float4 *px = reinterpret_cast<float4 *>(xs + tt * kRmKC) + p;
                        float4 v = *px;
                        const float4 w4 = nws[p];
                        const float rs = s_rms[tt];
                        v.x = v.x * rs * w4.x;
                        v.y = v.y * rs * w4.y;
                        v.z = v.z * rs * w4.z;
                        v.w = v.w * rs * w4.w;
                        *px = v;
                    }
                }
                __syncthreads();
            }
            if (blockIdx.x == 0 && a.xn)
#pragma unroll
                for (uint32_t i = tid; i < TC * kRmKC; i += NT) {
                    const uint32_t tt = i / kRmKC, cc = i % kRmKC;
                    if (tt < nt && cc < cw) a.xn[(size_t)(t0 + tt) * cols + c0 + cc] = xs[tt * kRmKC + cc];
                }
            if (blockIdx.x == 0 && a.xq)
                for (uint32_t task = (uint32_t)warp; task < TC * (kRmKC / 32); task += NT / 32) {
                    const uint32_t tt = task / (kRmKC / 32), b = task % (kRmKC / 32);
                    if (tt < nt && 32 * b < cw)
                        qact_store_block(a.xq + (size_t)(t0 + tt) * a.xq_pitch, (int)cols, (int)(c0 / 32 + b),
                                         xs[tt * kRmKC + 32 * b + lane], lane);
                }
        }
        const float *xw = xs + (size_t)wt * kRmTT * kRmKC + lane;
        const float *ww = ws + (size_t)we * kRmEE * kRmKC + lane;
        auto step = [&](uint32_t j) {
            float xv[kRmTT], wv[kRmEE];
#pragma unroll
            for (int i = 0; i < kRmTT; i++) xv[i] = xw[i * kRmKC + 32 * j];
#pragma unroll
            for (int e = 0; e < kRmEE; e++) wv[e] = ww[e * kRmKC + 32 * j];
#pragma unroll
            for (int i = 0; i < kRmTT; i++)
#pragma unroll
                for (int e = 0; e < kRmEE; e++) acc[i][e] = __fadd_rn(acc[i][e], __fmul_rn(wv[e], xv[i]));
        };
        if (cw == kRmKC) {
#pragma unroll
            for (uint32_t j = 0; j < kRmKC / 32; j++) step(j);
        } else {
            for (uint32_t j = 0; j < cw / 32; j++) step(j);
        }
        __syncthreads();
        if (ch + 2 < nchunks) issue(ch + 2);
    }
    // combine each (token, expert)'s 32 chains in router_logit's order: lane l
    // of the 8-vector takes (c_l + c_{l+8}) + (c_{l+16} + c_{l+24}), then
    // ((-0 + v0) + v1) + ... + v7; the chains pass through shared memory
    {
        float *red = msm + (size_t)warp * 32 * 33;
#pragma unroll
        for (int half = 0; half < 2; half++) {
#pragma unroll
            for (int p = 0; p < 32; p++) red[p * 33 + lane] = acc[(32 * half + p) / kRmEE][(32 * half + p) % kRmEE];
            __syncwarp();
            const float *rr = red + lane * 33;
            float sum = -0.0f;
#pragma unroll
            for (int l = 0; l < 8; l++) sum = __fadd_rn(sum, __fadd_rn(__fadd_rn(rr[l], rr[l + 8]), __fadd_rn(rr[l + 16], rr[l + 24])));
            const uint32_t pp = 32u * half + lane, tt = wt * kRmTT + pp / kRmEE, e = e0 + we * kRmEE + pp % kRmEE;
            if (tt < nt && e < E) a.logits[(size_t)(t0 + tt) * E + e] = sum;
            __syncwarp();
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&a.counters[blockIdx.y], 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // the tile's tokens: logits and sort keys (even row stride, 16-byte aligned rows), ranks, weights
    const uint32_t E2 = (E + 3) & ~1u;
    float *lg = msm;                                                              // [TC][E]
    uint64_t *keys = reinterpret_cast<uint64_t *>(msm + (((size_t)TC * E + 3) & ~(size_t)3));  // [TC][E2]
    for (uint32_t i = tid; i < nt * E; i += NT) {
        const uint32_t tt = i / E, ee = i - tt * E;
        const float v = __ldcg(a.logits + (size_t)t0 * E + i);
        lg[i] = v;
        keys[tt * E2 + ee] = router_key(v, ee);
    }
    if ((uint32_t)tid < nt) keys[tid * E2 + E] = 0;
    __syncthreads();
    {
        const uint32_t g = (uint32_t)tid / kRmNorm, ti = (uint32_t)tid % kRmNorm;
        for (uint32_t base = 0; base < nt; base += NG)
            if (base + g < nt) router_rank_keys(keys + (base + g) * E2, E, a.k, s_sel[base + g], (int)ti, kRmNorm);
    }
    for (uint32_t tt = (uint32_t)warp; tt < nt; tt += NT / 32) {
        float mx, es;
        router_softmax_stats(lg + tt * E, E, lane, mx, es);
        if (lane == 0) {
            s_mx[tt] = mx;
            s_es[tt] = es;
        }
    }
    __syncthreads();
    if ((uint32_t)tid < nt) {
        const uint32_t tt = tid;
        float w[16];
        router_weights(lg + tt * E, s_sel[tt], a.k, s_mx[tt], s_es[tt], a.norm_topk, a.escale, w);
        for (uint32_t i = 0; i < a.k; i++) {
            a.ids[(size_t)(t0 + tt) * a.k + i] = s_sel[tt][i];
            a.wout[(size_t)(t0 + tt) * a.k + i] = w[i];
        }
    }
    if (tid == 0) a.counters[blockIdx.y] = 0;
}

template <int WT, int WE>
static cudaError_t launch_router_mm(const LaunchCfg &c, const RouterArgs &a) {
    using Gm = RmGeo<WT, WE>;
    const dim3 grid((a.E + Gm::EC - 1) / Gm::EC, (a.ntok + Gm::TC - 1) / Gm::TC);
    return launch_k(c, "router_topk", k_router_mm<WT, WE>, grid, dim3(Gm::NT), Gm::kSmem, a);
}

// The register-tiled kernel needs whole 32-column steps and 16-byte aligned rows (cp.async).
static bool router_mm_ok(const RouterArgs &a) {
    return a.ntok >= kRtMinTokens && a.cols % 32 == 0 && a.w_ld % 4 == 0 &&
           (reinterpret_cast<uintptr_t>(a.W) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
           (!a.norm_w || (reinterpret_cast<uintptr_t>(a.norm_w) & 15) == 0);
}

cudaError_t launch_router(const LaunchCfg &c, const float *w, uint32_t E, uint32_t cols, uint32_t w_ld,
                          const float *x, const float *norm_w, float eps, uint32_t ntok, uint32_t k, int norm_topk,
                          const float *escale, uint32_t *ids, float *wout, float *logits, uint32_t *counters,
                          uint8_t *xq, uint64_t xq_pitch, float *xn) {
    RouterArgs a{w,      E,   cols,      w_ld,   x,    norm_w, eps,      ntok, k,
                 norm_topk, escale, ids, wout, logits, counters, xq, xq_pitch, xn};
    if (router_mm_ok(a)) return ntok >= 2048 ? launch_router_mm<2, 4>(c, a) : launch_router_mm<1, 4>(c, a);
    if (ntok >= kRtMinTokens && cols <= kRtMaxCols) {
        const size_t smem = rt_layout(cols, E).total;
        return launch_k(c, "router_topk", k_router_tok, dim3((ntok + kRtTok - 1) / kRtTok), dim3(kRtWarps * 32), smem,
                        a);
    }
    const dim3 grid((E + kRouterWarps - 1) / kRouterWarps, router_token_groups(ntok));
    const size_t smem_x = (size_t)(kRouterTok + (norm_w ? 1 : 0)) * cols * 4;
    const size_t smem_topk = (size_t)kRouterTok * (kRouterMaxE * 4 + (kRouterMaxE + 2) * 8);
    const size_t smem = smem_x > smem_topk ? smem_x : smem_topk;
    return launch_k(c, "router_topk", k_router, grid, dim3(kRouterWarps * 32), smem, a);
}

}  // namespace lt
