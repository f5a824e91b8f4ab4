// lt_router.cu — MoE router: routerTopKSoftmax (src/model/gemma4/forward.zig:
// 648-668) with the pre-FFN RMSNorm (src/ops/math.zig:20-26) and the
// activation quantisation for the expert kernels fused in.
//
// Each warp computes one expert's logit with dotf32's exact evaluation order
// (src/ops/math.zig:96-116): lane l owns the chain over elements l, l+32, ...
// (acc_{l/8}[l%8] in the reference), then (a0+a1)+(a2+a3), the 8-wide tail,
// the ordered 8-lane reduction and the scalar tail.  Given the same input
// vector the logits, and so the selected ids, equal the CPU path bit for bit.
// The last CTA of each token group selects the top-k (strict '>', lowest
// index on ties, forward.zig:598-629) and the softmax weights.
#include "lt_qact.cuh"

namespace lt {

constexpr int kRouterWarps = 4;  // experts per CTA
constexpr int kRouterTok = 4;    // tokens per CTA (one warp each for norm and top-k)
constexpr int kRouterChunk = 64;  // weights per lane kept in registers (2048 columns)

uint32_t router_token_groups(uint32_t ntok) { return (ntok + kRouterTok - 1) / kRouterTok; }

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
};

__global__ void __launch_bounds__(kRouterWarps * 32) k_router(RouterArgs a) {
    extern __shared__ __align__(16) float xsm[];  // [kRouterTok][cols] x, then [cols] norm weights
    __shared__ int s_last;
    __shared__ float s_ss[kRouterWarps][kRouterTok];
    __shared__ float s_rms[kRouterTok];
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
            for (uint32_t i = threadIdx.x; i < cols / 4; i += blockDim.x)
                reinterpret_cast<float4 *>(nwsm)[i] = __ldg(reinterpret_cast<const float4 *>(a.norm_w) + i);
        } else {
            for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) nwsm[i] = __ldg(a.norm_w + i);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    {
        const float *xt = a.x + (size_t)t0 * cols;
        const uint32_t n = nt * cols;
        if ((cols & 3) == 0 && (reinterpret_cast<uintptr_t>(xt) & 15) == 0) {
            for (uint32_t i = threadIdx.x; i < n / 4; i += blockDim.x)
                reinterpret_cast<float4 *>(xsm)[i] = reinterpret_cast<const float4 *>(xt)[i];
        } else {
            for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) xsm[i] = xt[i];
        }
    }
    __syncthreads();
    if (a.norm_w) {  // rmsnorm(out, x, w, eps): x * (1/sqrt(ss/n + eps)) * w
        float ss[kRouterTok];
#pragma unroll
        for (int tt = 0; tt < kRouterTok; tt++) {
            ss[tt] = 0.0f;
            if (tt < (int)nt)
                for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) ss[tt] += xsm[tt * cols + i] * xsm[tt * cols + i];
            ss[tt] = warp_sum(ss[tt]);
        }
        if (lane == 0)
#pragma unroll
            for (int tt = 0; tt < kRouterTok; tt++) s_ss[warp][tt] = ss[tt];
        __syncthreads();
        if (threadIdx.x < nt) {
            float s = 0.0f;
            for (int w = 0; w < kRouterWarps; w++) s += s_ss[w][threadIdx.x];
            s_rms[threadIdx.x] = 1.0f / sqrtf(s / (float)cols + a.eps);
        }
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < nt * cols; i += blockDim.x) {
            const uint32_t tt = i / cols, c = i - tt * cols;
            xsm[i] = xsm[i] * s_rms[tt] * nwsm[c];
        }
        __syncthreads();
    }
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
    // top-k + softmax statistics, one warp per token
    for (uint32_t tt = warp; tt < nt; tt += kRouterWarps) {
        const float *lg = a.logits + (size_t)(t0 + tt) * a.E;
        float v[kRouterMaxE / 32];
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < kRouterMaxE / 32; j++) {
            const uint32_t ee = lane + 32 * j;
            v[j] = ee < a.E ? __ldcg(lg + ee) : -INFINITY;
            mx = fmaxf(mx, v[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float es = 0.0f;
#pragma unroll
        for (int j = 0; j < kRouterMaxE / 32; j++)
            if (lane + 32 * j < a.E) es += expf(v[j] - mx);
        es = warp_sum(es);
        uint32_t taken = 0;  // bit j: element lane+32j selected
        float psel[16];
        uint32_t isel[16];
        for (uint32_t i = 0; i < a.k; i++) {
            // best untaken: larger value, ties -> lower index
            float bv = -INFINITY;
            uint32_t bi = 0xffffffffu;
#pragma unroll
            for (int j = 0; j < kRouterMaxE / 32; j++) {
                const uint32_t ee = lane + 32 * j;
                if (ee < a.E && !((taken >> j) & 1u) && (v[j] > bv || bi == 0xffffffffu)) {
                    bv = v[j];
                    bi = ee;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (oi != 0xffffffffu && (bi == 0xffffffffu || ov > bv || (ov == bv && oi < bi))) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (bi != 0xffffffffu && (bi & 31u) == (uint32_t)lane) taken |= 1u << (bi >> 5);
            isel[i] = bi;
            psel[i] = expf(bv - mx) / es;
        }
        if (lane == 0) {
            float sum = 0.0f;
            if (a.norm_topk)
                for (uint32_t i = 0; i < a.k; i++) sum += psel[i];
            for (uint32_t i = 0; i < a.k; i++) {
                float w = a.norm_topk ? psel[i] / sum : psel[i];
                if (a.escale) w = a.escale[isel[i]] * w;
                a.ids[(size_t)(t0 + tt) * a.k + i] = isel[i];
                a.wout[(size_t)(t0 + tt) * a.k + i] = w;
            }
        }
    }
    if (threadIdx.x == 0) a.counters[blockIdx.y] = 0;
}

cudaError_t launch_router(const LaunchCfg &c, const float *w, uint32_t E, uint32_t cols, uint32_t w_ld,
                          const float *x, const float *norm_w, float eps, uint32_t ntok, uint32_t k, int norm_topk,
                          const float *escale, uint32_t *ids, float *wout, float *logits, uint32_t *counters,
                          uint8_t *xq, uint64_t xq_pitch) {
    RouterArgs a{w, E, cols, w_ld, x, norm_w, eps, ntok, k, norm_topk, escale, ids, wout, logits, counters, xq, xq_pitch};
    const dim3 grid((E + kRouterWarps - 1) / kRouterWarps, router_token_groups(ntok));
    const size_t smem = (size_t)(kRouterTok + (norm_w ? 1 : 0)) * cols * 4;
    return launch_k(c, "router_topk", k_router, grid, dim3(kRouterWarps * 32), smem, a);
}

}  // namespace lt
