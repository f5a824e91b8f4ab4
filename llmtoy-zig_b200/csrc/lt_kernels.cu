// lt_kernels.cu — GGUF type table, kernel profiler, bit-exact dequant, and the
// small elementwise / reduction ops (rmsnorm, softmax, greedy argmax).
// The matvec, router and MoE kernels live in lt_qmv.cu, lt_router.cu and
// lt_moe.cu.
#include <cfloat>
#include <utility>

#include "lt_launch.cuh"

namespace lt {

// ── GGUF type table (src/gguf/types.zig:138-173, src/ops/math.zig:194) ─────

bool type_supported(uint32_t t) { return t == T_F32 || t == T_F16 || is_quant_type(t); }

uint32_t block_elems_of(uint32_t t) {
    if (t == T_F32 || t == T_F16) return 1;
    if (is_k_type(t)) return 256;
    return is_quant_type(t) ? 32 : 0;
}

uint64_t row_bytes_of(uint32_t t, uint64_t cols) {
    switch (t) {
    case T_F32: return cols * 4;
    case T_F16: return cols * 2;
    case T_Q5_0: return (cols / 32) * 22;
    case T_Q5_1: return (cols / 32) * 24;
    case T_Q8_0: return (cols / 32) * 34;
    case T_IQ4_NL: return (cols / 32) * 18;
    case T_Q3_K: return (cols / 256) * 110;
    case T_Q4_K: return (cols / 256) * 144;
    case T_Q5_K: return (cols / 256) * 176;
    case T_Q6_K: return (cols / 256) * 210;
    default: return 0;
    }
}

// ── launch helper ──────────────────────────────────────────────────────────

cudaEvent_t Profiler::get_event() {
    if (n_pool > 0) return pool[--n_pool];
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void Profiler::begin(const char *label, cudaStream_t s, Rec &r) {
    r.label = label;
    r.a = get_event();
    r.b = get_event();
    cudaEventRecord(r.a, s);
}

void Profiler::end(Rec &r, cudaStream_t s) {
    cudaEventRecord(r.b, s);
    if (n_pending < (int)(sizeof(pending) / sizeof(pending[0]))) {
        pending[n_pending++] = r;
    } else {  // table full: drop the sample, recycle its events
        if (n_pool + 2 <= (int)(sizeof(pool) / sizeof(pool[0]))) {
            pool[n_pool++] = r.a;
            pool[n_pool++] = r.b;
        } else {
            cudaEventDestroy(r.a);
            cudaEventDestroy(r.b);
        }
    }
}

cudaError_t Profiler::flush() {
    cudaError_t err = cudaSuccess;
    for (int i = 0; i < n_pending; i++) {
        Rec &r = pending[i];
        float ms = 0.0f;
        cudaError_t e = cudaEventSynchronize(r.b);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, r.a, r.b);
        if (e != cudaSuccess) {
            err = e;
        } else {
            int j = 0;
            while (j < n_agg && agg[j].label != r.label) j++;
            if (j == n_agg && n_agg < (int)(sizeof(agg) / sizeof(agg[0]))) {
                agg[n_agg++] = Agg{r.label, 0, 0.0, 1e30, 0.0};
            }
            if (j < n_agg) {
                agg[j].count++;
                agg[j].total_ms += ms;
                agg[j].min_ms = ms < agg[j].min_ms ? ms : agg[j].min_ms;
                agg[j].max_ms = ms > agg[j].max_ms ? ms : agg[j].max_ms;
            }
        }
        if (n_pool + 2 <= (int)(sizeof(pool) / sizeof(pool[0]))) {
            pool[n_pool++] = r.a;
            pool[n_pool++] = r.b;
        } else {
            cudaEventDestroy(r.a);
            cudaEventDestroy(r.b);
        }
    }
    n_pending = 0;
    return err;
}

void Profiler::reset() { n_agg = 0; }

void Profiler::destroy() {
    flush();
    for (int i = 0; i < n_pool; i++) cudaEventDestroy(pool[i]);
    n_pool = 0;
}

// ── exact element decoders (src/quant/dequant.zig) ─────────────────────────
// Each product and difference is rounded separately, as Zig's strict float
// mode does (no fused multiply-add), so results are bit-identical.

LT_DEVINL float f16_at(const uint8_t *p) { return f16_bits_to_f32((uint32_t)p[0] | ((uint32_t)p[1] << 8)); }

// dequant.zig:291-300
LT_DEVINL void scale_min_k4(int j, const uint8_t *s, uint32_t &sc, uint32_t &mn) {
    if (j < 4) {
        sc = s[j] & 63u;
        mn = s[j + 4] & 63u;
    } else {
        sc = (s[j + 4] & 0x0fu) | ((uint32_t)(s[j - 4] >> 6) << 4);
        mn = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
    }
}

// The 6-bit Q3_K scale k (0..15) from its 12 packed bytes (dequant.zig:398-411):
// low nibble from byte (k % 8) (high nibble for k >= 8), two high bits from
// byte 8 + k % 4 at bit 2 * (k / 4).
LT_DEVINL uint32_t q3k_scale(const uint8_t *s, uint32_t k) {
    const uint32_t b = k & 3, w = k >> 2;
    const uint32_t lo = (w & 2) ? (uint32_t)(s[4 * (w & 1) + b] >> 4) : (s[4 * (w & 1) + b] & 15u);
    return lo | (((uint32_t)s[8 + b] >> (2 * w)) & 3u) << 4;
}

LT_DEVINL float dq_elem(const uint8_t *row, uint32_t type, uint32_t i) {
    switch (type) {
    case T_F32: return reinterpret_cast<const float *>(row)[i];
    case T_F16: return f16_at(row + 2 * i);
    case T_Q8_0: {  // dequant.zig:42-52
        const uint8_t *b = row + (i / 32) * 34;
        return __fmul_rn(f16_at(b), (float)(int8_t)b[2 + (i & 31)]);
    }
    case T_Q4_K: {  // dequant.zig:157-187
        const uint8_t *sb = row + (i / 256) * 144;
        const uint32_t e = i & 255, c = e >> 6, p = e & 63;
        const int j = (int)(2 * c + (p >= 32 ? 1 : 0));
        const uint8_t byte = sb[16 + 32 * c + (p & 31)];
        const uint32_t q = p < 32 ? (byte & 15u) : (uint32_t)(byte >> 4);
        uint32_t sc, mn;
        scale_min_k4(j, sb + 4, sc, mn);
        const float d1 = __fmul_rn(f16_at(sb), (float)sc);
        const float m1 = __fmul_rn(f16_at(sb + 2), (float)mn);
        return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    case T_Q6_K: {  // dequant.zig:237-287
        const uint8_t *sb = row + (i / 256) * 210;
        const uint32_t e = i & 255, n = e >> 7, r = e & 127, kind = r >> 5, l = r & 31;
        const uint8_t ql = sb[64 * n + l + 32 * (kind & 1)];
        const uint8_t qh = sb[128 + 32 * n + l];
        const uint32_t lo4 = (ql >> (4 * (kind >> 1))) & 15u;
        const uint32_t hi2 = (qh >> (2 * kind)) & 3u;
        const int q = (int)(lo4 | (hi2 << 4)) - 32;
        const int8_t sc = (int8_t)sb[192 + 8 * n + (l >> 4) + 2 * kind];
        const float s = __fmul_rn(f16_at(sb + 208), (float)sc);
        return __fmul_rn(s, (float)q);
    }
    case T_Q5_0: {  // dequant.zig:201-217: d * (nibble | bit e of qh << 4) - 16
        const uint8_t *b = row + (i / 32) * 22;
        const uint32_t e = i & 31, qh = (uint32_t)b[2] | (uint32_t)b[3] << 8 | (uint32_t)b[4] << 16 | (uint32_t)b[5] << 24;
        const uint32_t nib = e < 16 ? (b[6 + e] & 15u) : (uint32_t)(b[6 + e - 16] >> 4);
        return __fmul_rn(f16_at(b), (float)((int)(nib | ((qh >> e) & 1u) << 4) - 16));
    }
    case T_Q5_1: {  // dequant.zig:469-487: d * q + m
        const uint8_t *b = row + (i / 32) * 24;
        const uint32_t e = i & 31;
        const uint32_t nib = e < 16 ? (b[8 + e] & 15u) : (uint32_t)(b[8 + e - 16] >> 4);
        const uint32_t q = nib | (((uint32_t)b[4 + e / 8] >> (e % 8)) & 1u) << 4;
        return __fadd_rn(__fmul_rn(f16_at(b), (float)q), f16_at(b + 2));
    }
    case T_IQ4_NL: {  // dequant.zig:618-640: d * table[nibble]
        const uint8_t *b = row + (i / 32) * 18;
        const uint32_t e = i & 31;
        const uint32_t nib = e < 16 ? (b[2 + e] & 15u) : (uint32_t)(b[2 + e - 16] >> 4);
        return __fmul_rn(f16_at(b), (float)iq4nl_value(nib));
    }
    case T_Q5_K: {  // dequant.zig:324-367: Q4_K with a fifth bit from qh
        const uint8_t *sb = row + (i / 256) * 176;
        const uint32_t e = i & 255, c = e >> 6, p = e & 63, up = p >= 32 ? 1u : 0u;
        const uint8_t byte = sb[48 + 32 * c + (p & 31)];
        const uint32_t lo = up ? (uint32_t)(byte >> 4) : (byte & 15u);
        const uint32_t q = lo + (((uint32_t)sb[16 + (p & 31)] >> (2 * c + up)) & 1u) * 16u;
        uint32_t sc, mn;
        scale_min_k4((int)(2 * c + up), sb + 4, sc, mn);
        const float d1 = __fmul_rn(f16_at(sb), (float)sc);
        const float m1 = __fmul_rn(f16_at(sb + 2), (float)mn);
        return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    case T_Q3_K: {  // dequant.zig:388-464
        const uint8_t *sb = row + (i / 256) * 110;
        const uint32_t e = i & 255, h = e >> 7, j = (e >> 5) & 3, g = (e >> 4) & 1, l = e & 15;
        const uint32_t lo2 = ((uint32_t)sb[32 + 32 * h + 16 * g + l] >> (2 * j)) & 3u;
        const bool hb = (sb[16 * g + l] >> (4 * h + j)) & 1u;
        const int v = (int)lo2 - (hb ? 0 : 4);
        const float dl = __fmul_rn(f16_at(sb + 108), (float)q3k_scale(sb + 96, 8 * h + 2 * j + g) - 32.0f);
        return __fmul_rn(dl, (float)v);
    }
    default: return 0.0f;
    }
}

__global__ void k_dequant(const uint8_t *base, uint32_t type, uint64_t pitch, uint64_t cols,
                          uint64_t row0, uint64_t n, float *out) {
    pdl_wait();
    for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < n;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = idx / cols, col = idx - r * cols;
        out[idx] = dq_elem(base + (row0 + r) * pitch, type, (uint32_t)col);
    }
}

__global__ void k_fill_f32(float *p, size_t n, float v) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        p[i] = v;
}

cudaError_t launch_fill_f32(cudaStream_t s, float *p, size_t n, float v) {
    const size_t want = (n + 255) / 256;
    k_fill_f32<<<(unsigned)(want < 4096 ? (want ? want : 1) : 4096), 256, 0, s>>>(p, n, v);
    return cudaGetLastError();
}

// embedLookup (src/model/forward.zig:319-341) of the token at the current
// position of a decode graph's token stream.
__global__ void k_embed(const uint8_t *base, uint32_t type, uint64_t pitch, uint32_t cols, uint64_t rows,
                        const uint32_t *tokens, const uint32_t *pos, float *out, int *dev_err) {
    pdl_wait();
    uint32_t row = tokens[*pos];
    if (row >= rows) {
        if (threadIdx.x == 0 && blockIdx.x == 0 && dev_err) atomicExch(dev_err, DEV_ERR_BAD_INDEX);
        row = 0;
    }
    const uint8_t *r = base + (uint64_t)row * pitch;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x)
        out[i] = dq_elem(r, type, i);
}

cudaError_t launch_embed(const LaunchCfg &c, const DevMat &m, const uint32_t *tokens, const uint32_t *pos,
                         float *out) {
    const uint32_t cols = (uint32_t)m.cols;
    return launch_k(c, "embed", k_embed, dim3((cols + 255) / 256), dim3(256), 0, m.data, m.type, m.pitch, cols,
                    m.rows, tokens, pos, out, c.dev_err);
}

cudaError_t launch_dequant(const LaunchCfg &c, const DevMat &m, uint64_t row0, uint64_t nrows, float *out) {
    const uint64_t n = nrows * m.cols;
    if (n == 0) return cudaSuccess;
    const uint64_t want = (n + 255) / 256;
    const unsigned grid = (unsigned)(want < 65535ull * 8 ? want : 65535ull * 8);
    return launch_k(c, "dequant", k_dequant, dim3(grid), dim3(256), 0, m.data, m.type, m.pitch, m.cols, row0, n, out);
}

// ── Q8_1 activation blocks (src/quant/dequant.zig:508-613) ─────────────────
// Block b of 36 bytes: f16 d = amax / 127, f16 s = d * sum(q), 32 int8 q =
// clamp(round(x / d)) with halves away from zero (Zig's @round, CUDA's
// roundf).  The x4 layout groups four blocks as {ds[4], qs[4][32]} (144 B).

LT_DEVINL size_t q81_ds_off(uint64_t b, int x4) { return x4 ? (b >> 2) * 144 + (b & 3) * 4 : b * 36; }
LT_DEVINL size_t q81_qs_off(uint64_t b, int x4) { return x4 ? (b >> 2) * 144 + 16 + (b & 3) * 32 : b * 36 + 4; }

// One warp per block; blocks past nb (the x4 padding of a partial last group) are zeroed.
__global__ void k_quantize_q8_1(const float *x, uint64_t nb, uint64_t nb_pad, int x4, uint8_t *out) {
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const uint64_t nw = (uint64_t)gridDim.x * (blockDim.x >> 5);
    for (uint64_t b = blockIdx.x * (uint64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); b < nb_pad; b += nw) {
        uint8_t *ds = out + q81_ds_off(b, x4), *qs = out + q81_qs_off(b, x4);
        if (b >= nb) {
            qs[lane] = 0;
            if (lane < 4) ds[lane] = 0;
            continue;
        }
        const float v = x[32 * b + lane];
        float amax = fabsf(v);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = __fdiv_rn(amax, 127.0f);
        const float inv = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const float q = fminf(fmaxf(roundf(__fmul_rn(v, inv)), -127.0f), 127.0f);
        const int qi = (int)q;
        int sum = qi;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        qs[lane] = (uint8_t)(int8_t)qi;
        if (lane == 0) {
            const uint32_t w = f32_to_f16_bits(d) | f32_to_f16_bits(__fmul_rn(d, (float)sum)) << 16;
            ds[0] = (uint8_t)w;
            ds[1] = (uint8_t)(w >> 8);
            ds[2] = (uint8_t)(w >> 16);
            ds[3] = (uint8_t)(w >> 24);
        }
    }
}

__global__ void k_dequant_q8_1(const uint8_t *q, uint64_t n, int x4, float *out) {
    pdl_wait();
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t b = i >> 5;
        const float d = f16_at(q + q81_ds_off(b, x4));
        out[i] = __fmul_rn(d, (float)(int8_t)q[q81_qs_off(b, x4) + (i & 31)]);
    }
}

cudaError_t launch_quantize_q8_1(const LaunchCfg &c, const float *x, uint64_t n, int x4, uint8_t *out) {
    const uint64_t nb = n / 32, nb_pad = x4 ? (nb + 3) / 4 * 4 : nb;
    if (nb_pad == 0) return cudaSuccess;
    const uint64_t want = (nb_pad + 7) / 8;
    const unsigned grid = (unsigned)(want < 65535ull * 8 ? want : 65535ull * 8);
    return launch_k(c, "quantize_q8_1", k_quantize_q8_1, dim3(grid), dim3(256), 0, x, nb, nb_pad, x4, out);
}

cudaError_t launch_dequant_q8_1(const LaunchCfg &c, const uint8_t *q, uint64_t n, int x4, float *out) {
    if (n == 0) return cudaSuccess;
    const uint64_t want = (n + 255) / 256;
    const unsigned grid = (unsigned)(want < 65535ull * 8 ? want : 65535ull * 8);
    return launch_k(c, "dequant_q8_1", k_dequant_q8_1, dim3(grid), dim3(256), 0, q, n, x4, out);
}

// Activation quantisation and block decoders: lt_decode.cuh.

// ── rmsnorm / softmax / argmax ─────────────────────────────────────────────

LT_DEVINL float block_max(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float m = red[0];
    for (int i = 1; i < nw; i++) m = fmaxf(m, red[i]);
    return m;
}

// src/ops/math.zig:20-26
__global__ void k_rmsnorm(const float *x, const float *w, float eps, uint32_t n, float *y) {
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const float *xt = x + (size_t)blockIdx.x * n;
    float *yt = y + (size_t)blockIdx.x * n;
    const float rms_inv = rms_inv_block(xt, n, eps, red);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) yt[i] = xt[i] * rms_inv * w[i];
}

cudaError_t launch_rmsnorm(const LaunchCfg &c, const float *x, const float *w, float eps, uint32_t n, uint32_t ntok,
                           float *y) {
    return launch_k(c, "rmsnorm", k_rmsnorm, dim3(ntok), dim3(256), 0, x, w, eps, n, y);
}

// src/ops/math.zig:29-35
__global__ void k_softmax(float *x, uint32_t n) {
    __shared__ float red[32];
    pdl_wait();
    float *xt = x + (size_t)blockIdx.x * n;
    float mx = -INFINITY;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, xt[i]);
    mx = block_max(mx, red);
    float s = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = expf(xt[i] - mx);
        xt[i] = v;
        s += v;
    }
    s = block_sum(s, red);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) xt[i] = xt[i] / s;
}

cudaError_t launch_softmax(const LaunchCfg &c, float *x, uint32_t n, uint32_t ntok) {
    return launch_k(c, "softmax", k_softmax, dim3(ntok), dim3(256), 0, x, n);
}

// greedy (src/model/sample.zig:11-17): first index of the maximum.  NaNs are
// never selected unless element 0 is NaN (then nothing beats it: index 0).
LT_DEVINL void argmax_combine(float &bv, uint32_t &bi, float ov, uint32_t oi) {
    if (oi == 0xffffffffu) return;
    if (bi == 0xffffffffu || ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
    }
}

__global__ void k_argmax(const float *x, uint32_t n, uint32_t *idx, float *pv, uint32_t *pi, uint32_t *counters,
                         uint32_t *tokens, uint32_t *pos, const uint32_t *n_prompt) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    __shared__ int s_last;
    pdl_wait();
    const uint32_t t = blockIdx.y;
    const float *xt = x + (size_t)t * n;
    float bv = -INFINITY;
    uint32_t bi = 0xffffffffu;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = xt[i];
        if (v == v) argmax_combine(bv, bi, v, i);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        argmax_combine(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < nw; w++) argmax_combine(bv, bi, sv[w], si[w]);
        pv[(size_t)t * gridDim.x + blockIdx.x] = bv;
        pi[(size_t)t * gridDim.x + blockIdx.x] = bi;
        __threadfence();
        s_last = atomicAdd(&counters[t], 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last || threadIdx.x != 0) return;
    __threadfence();
    float fv = -INFINITY;
    uint32_t fi = 0xffffffffu;
    for (uint32_t b = 0; b < gridDim.x; b++)
        argmax_combine(fv, fi, __ldcg(pv + (size_t)t * gridDim.x + b), __ldcg(pi + (size_t)t * gridDim.x + b));
    const float x0 = xt[0];
    if (x0 != x0 || fi == 0xffffffffu) fi = 0;
    if (idx) idx[t] = fi;
    if (tokens) {  // the step's sampled token goes after the prompt; advance the position
        const uint32_t p = *pos;
        if (p + 1 >= *n_prompt) tokens[p + 1] = fi;
        *pos = p + 1;
    }
    counters[t] = 0;
}

cudaError_t launch_argmax(const LaunchCfg &c, const float *x, uint32_t n, uint32_t ntok, uint32_t *idx, float *pv,
                          uint32_t *pi, uint32_t *counters, uint32_t *tokens, uint32_t *pos,
                          const uint32_t *n_prompt) {
    const uint32_t nb = max(1u, min(64u, (n + 4095) / 4096));
    return launch_k(c, "argmax", k_argmax, dim3(nb, ntok), dim3(256), 0, x, n, idx, pv, pi, counters, tokens, pos,
                    n_prompt);
}

// ── self-test of the bounded device waits ───────────────────────────────────
// Grid-barrier counter of the self-test kernel: grows by gridDim.x (2) per
// launch, like the persistent kernels' counters.
__device__ unsigned long long g_selftest_ctr;

// kind 0: a grid barrier every CTA reaches (completes); kind 1: the same
// barrier expecting one arrival more than the grid gives; kind 2: an mbarrier
// expecting one arrival more than it gets.  Kinds 1 and 2 give up after
// limit_ns through the same wait helpers the persistent kernels use, record
// the error code and return.
__global__ void k_selftest_wait(int kind, uint64_t limit_ns, int *dev_err) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint64_t s_epoch;
    if (kind == 2) {
        if (threadIdx.x == 0) {
            mbar_init(&bar, 2);
            fence_barrier_init();
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bar)) : "memory");
            if (!mbar_wait_bounded(&bar, 0, limit_ns) && dev_err) atomicExch(dev_err, DEV_ERR_TMA_TIMEOUT);
        }
        return;
    }
    if (threadIdx.x == 0) s_epoch = grid_epoch(&g_selftest_ctr, gridDim.x);
    __syncthreads();
    grid_wait(&g_selftest_ctr, s_epoch + (kind == 1 ? 1 : 0), dev_err, limit_ns);
}

cudaError_t launch_selftest_wait(const LaunchCfg &c, int kind, uint64_t limit_ns) {
    LaunchCfg plain = c;
    plain.pdl = false;
    return launch_k(plain, "selftest_wait", k_selftest_wait, dim3(2), dim3(32), 0, kind, limit_ns, c.dev_err);
}

}  // namespace lt
