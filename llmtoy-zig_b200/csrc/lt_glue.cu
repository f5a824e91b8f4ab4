// lt_glue.cu — the small vector steps between the big ops of a Gemma 4
// decoder layer (src/model/gemma4/forward.zig:117-120, 329-333, 401-413,
// 480-494, 526-531), one block per row of n values:
//
//   scale       x *= s                          (embedding scale, layer_output_scale)
//   add_rmsnorm x += rmsnorm(y) * w             (post_attention_norm + residual)
//   norm_pair   a = rmsnorm(x) * w, b = x * rms_inv * g * s   (rmsnormWeightedAndRawScaled)
//   ffn_tail    x = (x + rmsnorm(f' + rmsnorm(m) * w2) * w) * los, f' = rmsnorm(f) * w1 or f
//   softcap     x = tanh(x / cap) * cap
//
// The norms follow math.zig:20-26 (rms_inv = 1 / sqrt(sum(x^2) / n + eps)),
// products and sums rounded separately like the reference.
#include "lt_launch.cuh"

namespace lt {

constexpr int kGlueThreads = 512;

LT_DEVINL float glue_sum(float v, float *red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kGlueThreads / 32; i++) s += red[i];
    return s;
}

LT_DEVINL float glue_rms_inv(const float *v, uint32_t n, float eps, float *red) {
    float ss = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += kGlueThreads) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
    ss = glue_sum(ss, red);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
}

__global__ void __launch_bounds__(kGlueThreads) k_scale(float *x, uint32_t n, float s) {
    pdl_launch_dependents();
    pdl_wait();
    float *xt = x + (size_t)blockIdx.x * n;
    for (uint32_t i = threadIdx.x; i < n; i += kGlueThreads) xt[i] = __fmul_rn(xt[i], s);
}

__global__ void __launch_bounds__(kGlueThreads) k_add_rmsnorm(const float *y, const float *w, float eps, uint32_t n,
                                                              float *x) {
    __shared__ float red[kGlueThreads / 32];
    pdl_launch_dependents();
    pdl_wait();
    const float *yt = y + (size_t)blockIdx.x * n;
    float *xt = x + (size_t)blockIdx.x * n;
    const float r = glue_rms_inv(yt, n, eps, red);
    for (uint32_t i = threadIdx.x; i < n; i += kGlueThreads)
        xt[i] = __fadd_rn(xt[i], __fmul_rn(__fmul_rn(yt[i], r), w[i]));
}

__global__ void __launch_bounds__(kGlueThreads) k_norm_pair(const float *x, const float *w, const float *g, float gs,
                                                            float eps, uint32_t n, float *a, float *b) {
    __shared__ float red[kGlueThreads / 32];
    pdl_launch_dependents();
    pdl_wait();
    const float *xt = x + (size_t)blockIdx.x * n;
    const float r = glue_rms_inv(xt, n, eps, red);
    const float rb = __fmul_rn(r, gs);
    for (uint32_t i = threadIdx.x; i < n; i += kGlueThreads) {
        a[(size_t)blockIdx.x * n + i] = __fmul_rn(__fmul_rn(xt[i], r), w[i]);
        b[(size_t)blockIdx.x * n + i] = __fmul_rn(__fmul_rn(xt[i], rb), g[i]);
    }
}

LT_DEVINL float glue_rinv(float ss, uint32_t n, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
}

// Rows of up to kGlueThreads * kTailPer values: each thread keeps its values
// (i = tid + k * kGlueThreads) in registers, so the three norms take two block
// reductions and no global round trip; sums in glue_rms_inv's order.
constexpr int kTailPer = 16;

__global__ void __launch_bounds__(kGlueThreads) k_ffn_tail(const float *f, const float *w1, float *m, const float *w2,
                                                           const float *w, float los, float eps, uint32_t n, float *x) {
    __shared__ float red[kGlueThreads / 32], red2[kGlueThreads / 32];
    pdl_launch_dependents();
    pdl_wait();
    const size_t o = (size_t)blockIdx.x * n;
    float fv[kTailPer], mv[kTailPer];
    float sf = 0.0f, sm = 0.0f;
#pragma unroll
    for (int k = 0; k < kTailPer; k++) {
        const uint32_t i = threadIdx.x + k * kGlueThreads;
        fv[k] = i < n ? f[o + i] : 0.0f;
        mv[k] = i < n ? m[o + i] : 0.0f;
        if (i < n) {
            sf = __fadd_rn(sf, __fmul_rn(fv[k], fv[k]));
            sm = __fadd_rn(sm, __fmul_rn(mv[k], mv[k]));
        }
    }
    {  // both sums in one reduction (glue_sum's order for each)
        sf = warp_sum(sf);
        sm = warp_sum(sm);
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        if (lane == 0) {
            red[warp] = sf;
            red2[warp] = sm;
        }
        __syncthreads();
        sf = 0.0f;
        sm = 0.0f;
#pragma unroll
        for (int q = 0; q < kGlueThreads / 32; q++) {
            sf += red[q];
            sm += red2[q];
        }
    }
    const float rf1 = w1 ? glue_rinv(sf, n, eps) : 1.0f, rm = glue_rinv(sm, n, eps);
    float sh = 0.0f;
#pragma unroll
    for (int k = 0; k < kTailPer; k++) {
        const uint32_t i = threadIdx.x + k * kGlueThreads;
        if (i < n) {
            const float fi = w1 ? __fmul_rn(__fmul_rn(fv[k], rf1), w1[i]) : fv[k];
            mv[k] = __fadd_rn(fi, __fmul_rn(__fmul_rn(mv[k], rm), w2[i]));
            m[o + i] = mv[k];
            sh = __fadd_rn(sh, __fmul_rn(mv[k], mv[k]));
        }
    }
    const float rf = glue_rinv(glue_sum(sh, red), n, eps);
#pragma unroll
    for (int k = 0; k < kTailPer; k++) {
        const uint32_t i = threadIdx.x + k * kGlueThreads;
        if (i < n) {
            float v = __fadd_rn(x[o + i], __fmul_rn(__fmul_rn(mv[k], rf), w[i]));
            if (los != 1.0f) v = __fmul_rn(v, los);
            x[o + i] = v;
        }
    }
}

// Longer rows: the same arithmetic through global memory.
__global__ void __launch_bounds__(kGlueThreads) k_ffn_tail_long(const float *f, const float *w1, float *m,
                                                                const float *w2, const float *w, float los, float eps,
                                                                uint32_t n, float *x) {
    __shared__ float red[kGlueThreads / 32];
    pdl_launch_dependents();
    pdl_wait();
    const size_t o = (size_t)blockIdx.x * n;
    const float rf1 = w1 ? glue_rms_inv(f + o, n, eps, red) : 1.0f;
    const float rm = glue_rms_inv(m + o, n, eps, red);
    for (uint32_t i = threadIdx.x; i < n; i += kGlueThreads) {
        const float fi = w1 ? __fmul_rn(__fmul_rn(f[o + i], rf1), w1[i]) : f[o + i];
        m[o + i] = __fadd_rn(fi, __fmul_rn(__fmul_rn(m[o + i], rm), w2[i]));
    }
    __syncthreads();
    const float rf = glue_rms_inv(m + o, n, eps, red);
    for (uint32_t i = threadIdx.x; i < n; i += kGlueThreads) {
        float v = __fadd_rn(x[o + i], __fmul_rn(__fmul_rn(m[o + i], rf), w[i]));
        if (los != 1.0f) v = __fmul_rn(v, los);
        x[o + i] = v;
    }
}

__global__ void k_softcap(float *x, size_t n, float cap) {
    pdl_launch_dependents();
    pdl_wait();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        x[i] = __fmul_rn(tanhf(__fdiv_rn(x[i], cap)), cap);
}

cudaError_t launch_scale(const LaunchCfg &c, float *x, uint32_t n, uint32_t ntok, float s) {
    return launch_k(c, "scale", k_scale, dim3(ntok), dim3(kGlueThreads), 0, x, n, s);
}
cudaError_t launch_add_rmsnorm(const LaunchCfg &c, const float *y, const float *w, float eps, uint32_t n,
                               uint32_t ntok, float *x) {
    return launch_k(c, "add_rmsnorm", k_add_rmsnorm, dim3(ntok), dim3(kGlueThreads), 0, y, w, eps, n, x);
}
cudaError_t launch_norm_pair(const LaunchCfg &c, const float *x, const float *w, const float *g, float gs, float eps,
                             uint32_t n, uint32_t ntok, float *a, float *b) {
    return launch_k(c, "norm_pair", k_norm_pair, dim3(ntok), dim3(kGlueThreads), 0, x, w, g, gs, eps, n, a, b);
}
cudaError_t launch_ffn_tail(const LaunchCfg &c, const float *f, const float *w1, float *m, const float *w2,
                            const float *w, float los, float eps, uint32_t n, uint32_t ntok, float *x) {
    if (n > (uint32_t)(kGlueThreads * kTailPer))
        return launch_k(c, "ffn_tail", k_ffn_tail_long, dim3(ntok), dim3(kGlueThreads), 0, f, w1, m, w2, w, los, eps, n,
                        x);
    return launch_k(c, "ffn_tail", k_ffn_tail, dim3(ntok), dim3(kGlueThreads), 0, f, w1, m, w2, w, los, eps, n, x);
}
cudaError_t launch_softcap(const LaunchCfg &c, float *x, size_t n, float cap) {
    const size_t want = (n + 255) / 256;
    return launch_k(c, "softcap", k_softcap, dim3((unsigned)(want < 4096 ? (want ? want : 1) : 4096)), dim3(256), 0,
                    x, n, cap);
}

}  // namespace lt
