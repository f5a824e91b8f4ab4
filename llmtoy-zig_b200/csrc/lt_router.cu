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

cudaError_t launch_router(const LaunchCfg &c, const float *w, uint32_t E, uint32_t cols, uint32_t w_ld,
                          const float *x, const float *norm_w, float eps, uint32_t ntok, uint32_t k, int norm_topk,
                          const float *escale, uint32_t *ids, float *wout, float *logits, uint32_t *counters,
                          uint8_t *xq, uint64_t xq_pitch, float *xn) {
    RouterArgs a{w,      E,   cols,      w_ld,   x,    norm_w, eps,      ntok, k,
                 norm_topk, escale, ids, wout, logits, counters, xq, xq_pitch, xn};
    const dim3 grid((E + kRouterWarps - 1) / kRouterWarps, router_token_groups(ntok));
    const size_t smem_x = (size_t)(kRouterTok + (norm_w ? 1 : 0)) * cols * 4;
    const size_t smem_topk = (size_t)kRouterTok * (kRouterMaxE * 4 + (kRouterMaxE + 2) * 8);
    const size_t smem = smem_x > smem_topk ? smem_x : smem_topk;
    return launch_k(c, "router_topk", k_router, grid, dim3(kRouterWarps * 32), smem, a);
}

}  // namespace lt
