// lt_qmv.cu — dense quantised matvec: quantMatvec / quantMatvecPar
// (src/ops/math.zig:133-171, :277-320) for ntok activation rows.
//
// Each warp owns `rw` consecutive weight rows (rw * items_per_row <= 32, one
// item per lane) and streams them into its shared-memory slice with one TMA
// bulk copy issued before the kernel waits on its producer (the weights are
// static).  Activations come pre-quantised (lt_qact.cuh), or for a single
// token as f32, which every CTA quantises into shared memory itself (one
// launch and one global round trip fewer than a separate quantiser).
#include "lt_qact.cuh"
#include "lt_rowdot.cuh"

namespace lt {

constexpr int kQmvWarps = 8;

struct QmvArgs {
    const uint8_t *rows;  // first row of the (expert) matrix
    uint64_t pitch;
    uint32_t nrows, cols, nitems, nblocks;
    const uint8_t *xq;  // nullptr: quantise xf (one token) in the CTA
    uint64_t xq_pitch;
    const float *xf;
    const float *norm_w;  // with xq == nullptr: quantise rmsnorm(xf) * norm_w instead
    float eps;
    float *y;
    const float *add;  // nullptr or y's shape: y = W . x + add
    uint32_t ntok;
    uint32_t rw;  // rows per warp
    int *dev_err;
};

__host__ __device__ inline size_t qmv_smem_bytes(uint64_t pitch, uint32_t rw, int nt, int ipr) {
    return 64 + 64 + align16((size_t)kQmvWarps * rw * pitch + 256) + align16(xs_bytes(nt, ipr)) +
           (size_t)kQmvWarps * nt * rw * ipr * 4;
}

// One CTA's rows (CTA index cta of the matrix's grid).
template <uint32_t TYPE, int NT>
LT_DEVINL void qmv_cta(const QmvArgs &a, uint32_t cta, uint8_t *smem) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ipr = (int)a.nitems;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    const uint8_t **src = reinterpret_cast<const uint8_t **>(smem + 64);
    uint8_t *tile = smem + 128;
    uint8_t *p = tile + align16((size_t)kQmvWarps * a.rw * a.pitch + 256);
    const XS X = xs_carve(p, NT, ipr);
    p += align16(xs_bytes(NT, ipr));
    float *part = reinterpret_cast<float *>(p);

    const uint32_t wr0 = (cta * kQmvWarps + warp) * a.rw;
    const int nr = wr0 < a.nrows ? (int)min(a.rw, a.nrows - wr0) : 0;
    uint8_t *wt = tile + (size_t)warp * a.rw * a.pitch;
    if (lane == 0 && nr > 0) {  // weights are static: fetch before waiting on the producer
        mbar_init(&bars[warp], 1);
        fence_barrier_init();
        const uint32_t bytes = (uint32_t)(nr * a.pitch);
        mbar_arrive_expect_tx(&bars[warp], bytes);
        tma_load_1d(wt, a.rows + (uint64_t)wr0 * a.pitch, bytes, &bars[warp]);
    }
    pdl_launch_dependents();
    pdl_wait();
    bool ok = true;
    const int nitem = nr * ipr;
    float *wpart = part + (size_t)warp * NT * a.rw * ipr;
    for (uint32_t c0 = 0; c0 < a.ntok; c0 += NT) {
        const int nt = (int)min((uint32_t)NT, a.ntok - c0);
        if (a.xq) {
            if (threadIdx.x < (unsigned)nt) src[threadIdx.x] = a.xq + (size_t)(c0 + threadIdx.x) * a.xq_pitch;
            __syncthreads();
            qact_to_smem(X, src, nt, (int)a.cols);
        } else if (a.norm_w) {  // one token, normalised as k_rmsnorm does, quantised as k_quantize does
            float *red = reinterpret_cast<float *>(smem + 64);  // the row-pointer slots, unused here
            const float r = rms_inv_block(a.xf, a.cols, a.eps, red);
            for (uint32_t b = warp; b < a.cols / 32; b += kQmvWarps) {
                const uint32_t i = 32 * b + lane;
                qact_block_to_xs(X, 0, (int)b, __ldcg(a.xf + i) * r * __ldg(a.norm_w + i), lane);
            }
        } else {  // one token: the same 16-group quantisation as k_quantize, here
            for (uint32_t b = warp; b < a.cols / 32; b += kQmvWarps)
                qact_block_to_xs(X, 0, (int)b, __ldcg(a.xf + 32 * b + lane), lane);
        }
        __syncthreads();
        if (c0 == 0 && nr > 0) ok = tile_wait(&bars[warp], a.dev_err);
        if (ok && nr > 0) {
            for (int f = lane; f < nitem; f += 32) {
                const int item = f % ipr, row = f / ipr;
                float res[NT];
#pragma unroll
                for (int t = 0; t < NT; t++) res[t] = 0.0f;
                dot_item<TYPE, NT>(wt + (size_t)row * a.pitch, item, (int)a.nblocks, X, 0, nt, res);
#pragma unroll
                for (int t = 0; t < NT; t++)
                    if (t < nt) wpart[t * nitem + f] = res[t];
            }
            __syncwarp();
            for (int l = lane; l < nt * nr; l += 32) {
                const int t = l / nr, r = l - t * nr;
                const float *pp = wpart + t * nitem + r * ipr;
                float s = 0.0f;
                for (int i = 0; i < ipr; i++) s += pp[i];
                const size_t yi = (size_t)(c0 + t) * a.nrows + wr0 + r;
                a.y[yi] = a.add ? __fadd_rn(a.add[yi], s) : s;
            }
        }
        __syncthreads();
    }
}

template <uint32_t TYPE, int NT>
__global__ void __launch_bounds__(kQmvWarps * 32) k_qmv(QmvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    qmv_cta<TYPE, NT>(a, blockIdx.x, smem);
}

// Up to four one-token matvecs on the same input in one launch: CTAs
// [begin[s], begin[s+1]) run matrix s, whatever its type.
constexpr int kQmvMaxSeg = 4;
struct QmvMulti {
    QmvArgs seg[kQmvMaxSeg];
    uint32_t type[kQmvMaxSeg];
    uint32_t begin[kQmvMaxSeg + 1];
    uint32_t n;
};

__global__ void __launch_bounds__(kQmvWarps * 32) k_qmv_multi(QmvMulti m) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint32_t s = 0;
    while (s + 1 < m.n && blockIdx.x >= m.begin[s + 1]) s++;
    const uint32_t cta = blockIdx.x - m.begin[s];
    switch (m.type[s]) {
    case T_Q4_K: qmv_cta<T_Q4_K, 1>(m.seg[s], cta, smem); break;
    case T_Q6_K: qmv_cta<T_Q6_K, 1>(m.seg[s], cta, smem); break;
    case T_Q8_0: qmv_cta<T_Q8_0, 1>(m.seg[s], cta, smem); break;
    case T_Q5_K: qmv_cta<T_Q5_K, 1>(m.seg[s], cta, smem); break;
    case T_Q3_K: qmv_cta<T_Q3_K, 1>(m.seg[s], cta, smem); break;
    case T_Q5_0: qmv_cta<T_Q5_0, 1>(m.seg[s], cta, smem); break;
    case T_Q5_1: qmv_cta<T_Q5_1, 1>(m.seg[s], cta, smem); break;
    case T_IQ4_NL: qmv_cta<T_IQ4_NL, 1>(m.seg[s], cta, smem); break;
    default: break;
    }
}

// f32 / f16 rows: one warp per row, plain loads.
__global__ void k_mv_float(const uint8_t *rows, uint64_t pitch, uint32_t type, uint32_t nrows, uint32_t cols,
                           const float *x, float *y, uint32_t ntok, const float *add) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t warps = (blockDim.x >> 5) * gridDim.x;
    for (uint32_t r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < nrows; r += warps) {
        const uint8_t *row = rows + (uint64_t)r * pitch;
        for (uint32_t t = 0; t < ntok; t++) {
            const float *xt = x + (size_t)t * cols;
            float s = 0.0f;
            for (uint32_t i = threadIdx.x & 31; i < cols; i += 32) {
                const float w = type == T_F32 ? reinterpret_cast<const float *>(row)[i]
                                              : __half2float(__ushort_as_half(reinterpret_cast<const unsigned short *>(row)[i]));
                s += w * xt[i];
            }
            s = warp_sum(s);
            const size_t yi = (size_t)t * nrows + r;
            if ((threadIdx.x & 31) == 0) y[yi] = add ? __fadd_rn(add[yi], s) : s;
        }
    }
}

// Large one-token matvecs (an lm_head of hundreds of MB): a persistent kernel,
// one CTA per SM with 16 warps, 8 to 16 of which stream rows (as many as
// have two stages' room).  Each streaming warp takes groups of rw rows (group
// g goes to streaming warp g % (CTAs * warps)) through its own ring of shared-memory
// stages, one TMA bulk copy per group, so the next groups' copies are in
// flight while it computes the current one.  Per-item partials and the
// per-row order of their sum are k_qmv's: the same bits.
constexpr int kQsWarps = 16;
constexpr uint32_t kQsMaxStages = 8;
constexpr size_t kQsBars = 0, kQsSrc = 1024, kQsPart = 1152, kQsX = 3200;  // + X, then the rings

struct QsArgs {
    QmvArgs a;
    uint32_t stages;  // ring depth per warp
    uint32_t stage;   // bytes per stage (a multiple of 128)
    uint32_t warps;   // warps that stream rows (the rest help stage the activations)
};

__host__ __device__ inline uint32_t qs_chunks(uint64_t cols) { return (uint32_t)((cols + 63) / 64); }

__host__ __device__ inline size_t qs_ring_offset(int ipr) { return kQsX + ((xs_bytes(1, ipr) + 127) & ~(size_t)127); }

template <uint32_t TYPE>
__global__ void __launch_bounds__(kQsWarps * 32, 1) k_qmv_stream(QsArgs q) {
    extern __shared__ __align__(128) uint8_t smem[];
    const QmvArgs &a = q.a;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ipr = (int)a.nitems;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kQsBars) + warp * kQsMaxStages;
    float *wpart = reinterpret_cast<float *>(smem + kQsPart) + warp * 32;
    const XS X = xs_carve(smem + kQsX, 1, ipr);
    uint8_t *ring = smem + qs_ring_offset(ipr) + (size_t)warp * q.stages * q.stage;
    const uint32_t W = gridDim.x * q.warps, gw = blockIdx.x * q.warps + warp;
    const uint32_t ngroups = (a.nrows + a.rw - 1) / a.rw;
    // groups gw, gw + W, ...
    const uint32_t mine = (uint32_t)warp < q.warps && gw < ngroups ? (ngroups - gw + W - 1) / W : 0;
    auto issue = [&](uint32_t i) {
        const uint32_t r0 = (gw + i * W) * a.rw, nr = min(a.rw, a.nrows - r0), st = i % q.stages;
        mbar_arrive_expect_tx(&bars[st], (uint32_t)(nr * a.pitch));
        tma_load_1d(ring + (size_t)st * q.stage, a.rows + (uint64_t)r0 * a.pitch, (uint32_t)(nr * a.pitch), &bars[st]);
    };
    if (lane == 0) {  // weights are static: the first stages before waiting on the producer
        for (uint32_t st = 0; st < q.stages; st++) mbar_init(&bars[st], 1);
        fence_barrier_init();
        for (uint32_t i = 0; i < min(mine, q.stages); i++) issue(i);
    }
    __syncwarp();
    pdl_launch_dependents();
    pdl_wait();
    if (a.xq) {
        const uint8_t **src = reinterpret_cast<const uint8_t **>(smem + kQsSrc);
        if (threadIdx.x == 0) src[0] = a.xq;
        __syncthreads();
        qact_to_smem(X, src, 1, (int)a.cols);
    } else {  // the same 16-group quantisation as k_quantize
        for (uint32_t b = warp; b < a.cols / 32; b += kQsWarps)
            qact_block_to_xs(X, 0, (int)b, __ldcg(a.xf + 32 * b + lane), lane);
    }
    __syncthreads();
    uint32_t i = 0;
    bool ok = true;
    for (; i < mine; i++) {
        const uint32_t st = i % q.stages;
        if (!mbar_wait_bounded(&bars[st], (i / q.stages) & 1, kWaitLimitNs)) {
            ok = false;
            break;
        }
        const uint32_t r0 = (gw + i * W) * a.rw, nr = min(a.rw, a.nrows - r0);
        const uint8_t *t = ring + (size_t)st * q.stage;
        const int nitem = (int)nr * ipr;
        for (int f = lane; f < nitem; f += 32) {
            float res[1] = {0.0f};
            dot_item<TYPE, 1>(t + (size_t)(f / ipr) * a.pitch, f % ipr, (int)a.nblocks, X, 0, 1, res);
            wpart[f] = res[0];
        }
        __syncwarp();
        if (lane == 0 && i + q.stages < mine) {  // the stage is read: the group after next takes it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(i + q.stages);
        }
        if ((uint32_t)lane < nr) {
            const float *pp = wpart + lane * ipr;
            float sum = 0.0f;
            for (int k = 0; k < ipr; k++) sum += pp[k];
            const size_t yi = r0 + lane;
            a.y[yi] = a.add ? __fadd_rn(a.add[yi], sum) : sum;
        }
        __syncwarp();
    }
    if (!ok && lane == 0) {  // report, then let the copies in flight land before the CTA exits
        if (a.dev_err) atomicExch(a.dev_err, DEV_ERR_TMA_TIMEOUT);
        for (uint32_t j = i; j < min(mine, i + q.stages); j++)
            mbar_wait_bounded(&bars[j % q.stages], (j / q.stages) & 1, kWaitLimitNs);
    }
}

// Q8_0: the same streaming with lanes on 64-column chunks of the
// activation held in registers (lt_rowdot.cuh): a lane walks the group's rows
// reading only its chunk's weight bytes, chunk partials are summed per row in
// column order.  Groups of rw rows; part: [rw][cpr] floats per warp after X.
template <uint32_t TYPE>
__global__ void __launch_bounds__(kQsWarps * 32, 1) k_qmv_stream64(QsArgs q) {
    extern __shared__ __align__(128) uint8_t smem[];
    const QmvArgs &a = q.a;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t cpr = qs_chunks(a.cols);
    const size_t part_w = ((size_t)a.rw * cpr * 4 + 127) & ~(size_t)127;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kQsBars) + warp * kQsMaxStages;
    const XS X = xs_carve(smem + kQsX, 1, (int)a.nitems);
    float *part = reinterpret_cast<float *>(smem + qs_ring_offset((int)a.nitems) + (size_t)warp * part_w);
    uint8_t *ring = smem + qs_ring_offset((int)a.nitems) + kQsWarps * part_w + (size_t)warp * q.stages * q.stage;
    const uint32_t W = gridDim.x * q.warps, gw = blockIdx.x * q.warps + warp;
    const uint32_t ngroups = (a.nrows + a.rw - 1) / a.rw;
    const uint32_t mine = (uint32_t)warp < q.warps && gw < ngroups ? (ngroups - gw + W - 1) / W : 0;
    auto issue = [&](uint32_t i) {
        const uint32_t r0 = (gw + i * W) * a.rw, nr = min(a.rw, a.nrows - r0), st = i % q.stages;
        mbar_arrive_expect_tx(&bars[st], (uint32_t)(nr * a.pitch));
        tma_load_1d(ring + (size_t)st * q.stage, a.rows + (uint64_t)r0 * a.pitch, (uint32_t)(nr * a.pitch), &bars[st]);
    };
    if (lane == 0) {
        for (uint32_t st = 0; st < q.stages; st++) mbar_init(&bars[st], 1);
        fence_barrier_init();
        for (uint32_t i = 0; i < min(mine, q.stages); i++) issue(i);
    }
    __syncwarp();
    pdl_launch_dependents();
    pdl_wait();
    if (a.xq) {
        const uint8_t **src = reinterpret_cast<const uint8_t **>(smem + kQsSrc);
        if (threadIdx.x == 0) src[0] = a.xq;
        __syncthreads();
        qact_to_smem(X, src, 1, (int)a.cols);
    } else {
        for (uint32_t b = warp; b < a.cols / 32; b += kQsWarps)
            qact_block_to_xs(X, 0, (int)b, __ldcg(a.xf + 32 * b + lane), lane);
    }
    __syncthreads();
    const bool one_pass = cpr <= 32;
    XChunk xc;
    if (one_pass && (uint32_t)lane < (32 / cpr) * cpr)
        xchunk_load(X, 0, (int)spread_chunk(lane % cpr, cpr), xc);
    uint32_t i = 0;
    bool ok = true;
    for (; i < mine; i++) {
        const uint32_t st = i % q.stages;
        if (!mbar_wait_bounded(&bars[st], (i / q.stages) & 1, kWaitLimitNs)) {
            ok = false;
            break;
        }
        const uint32_t r0 = (gw + i * W) * a.rw, nr = min(a.rw, a.nrows - r0);
        const uint8_t *t = ring + (size_t)st * q.stage;
        for (uint32_t cg = 0; cg < cpr; cg += 32) {  // lanes: n chunks of rps rows at a time
            const uint32_t n = min(32u, cpr - cg), rps = 32 / n, sub = lane / n;
            if (sub < rps) {
                const uint32_t cb = cg + spread_chunk(lane % n, n);
                if (!one_pass) xchunk_load(X, 0, (int)cb, xc);
                for (uint32_t r = sub; r < nr; r += rps)
                    part[r * cpr + cb] = dot64<TYPE>(t + (size_t)r * a.pitch, (int)cb, (int)a.nblocks, xc);
            }
        }
        __syncwarp();
        if (lane == 0 && i + q.stages < mine) {  // the stage is read: the group after next takes it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(i + q.stages);
        }
        if ((uint32_t)lane < nr) {
            const float *pp = part + lane * cpr;
            float sum = 0.0f;
            for (uint32_t k = 0; k < cpr; k++) sum += pp[k];
            const size_t yi = r0 + lane;
            a.y[yi] = a.add ? __fadd_rn(a.add[yi], sum) : sum;
        }
        __syncwarp();
    }
    if (!ok && lane == 0) {
        if (a.dev_err) atomicExch(a.dev_err, DEV_ERR_TMA_TIMEOUT);
        for (uint32_t j = i; j < min(mine, i + q.stages); j++)
            mbar_wait_bounded(&bars[j % q.stages], (j / q.stages) & 1, kWaitLimitNs);
    }
}

// Wide rows (64-column chunks >= 32, e.g. a 2048-column lm_head; Q8_0):
// lane l owns chunks l, l + 32, ... with the activation chunk in registers
// (loaded once when the row is exactly 32 chunks), so only weight bytes are
// read from shared memory per row; a group's <= 8 row partials are summed
// across the warp by a transpose reduction (three halving exchanges, then two
// butterfly steps: lane l ends with row ((l>>4)&1)*4 + ((l>>3)&1)*2 + ((l>>2)&1)).
constexpr uint32_t kQsWideRows = 8;

LT_DEVINL float qs_transpose_sum(float (&v)[kQsWideRows], int lane) {
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float send = b4 ? v[j] : v[j + 4], keep = b4 ? v[j + 4] : v[j];
        v[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const float send = b3 ? v[j] : v[j + 2], keep = b3 ? v[j + 2] : v[j];
        v[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    {
        const float send = b2 ? v[0] : v[1], keep = b2 ? v[1] : v[0];
        v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
    v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
    return v[0];
}

template <uint32_t TYPE>
__global__ void __launch_bounds__(kQsWarps * 32, 1) k_qmv_stream_w(QsArgs q) {
    extern __shared__ __align__(128) uint8_t smem[];
    const QmvArgs &a = q.a;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t cpr = qs_chunks(a.cols), npass = (cpr + 31) / 32;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kQsBars) + warp * kQsMaxStages;
    const XS X = xs_carve(smem + kQsX, 1, (int)a.nitems);
    uint8_t *ring = smem + qs_ring_offset((int)a.nitems) + (size_t)warp * q.stages * q.stage;
    const uint32_t W = gridDim.x * q.warps, gw = blockIdx.x * q.warps + warp;
    const uint32_t ngroups = (a.nrows + a.rw - 1) / a.rw;
    const uint32_t mine = (uint32_t)warp < q.warps && gw < ngroups ? (ngroups - gw + W - 1) / W : 0;
    auto issue = [&](uint32_t i) {
        const uint32_t r0 = (gw + i * W) * a.rw, nr = min(a.rw, a.nrows - r0), st = i % q.stages;
        mbar_arrive_expect_tx(&bars[st], (uint32_t)(nr * a.pitch));
        tma_load_1d(ring + (size_t)st * q.stage, a.rows + (uint64_t)r0 * a.pitch, (uint32_t)(nr * a.pitch), &bars[st]);
    };
    if (lane == 0) {  // weights are static: the first stages before waiting on the producer
        for (uint32_t st = 0; st < q.stages; st++) mbar_init(&bars[st], 1);
        fence_barrier_init();
        for (uint32_t i = 0; i < min(mine, q.stages); i++) issue(i);
    }
    __syncwarp();
    pdl_launch_dependents();
    pdl_wait();
    if (a.xq) {
        const uint8_t **src = reinterpret_cast<const uint8_t **>(smem + kQsSrc);
        if (threadIdx.x == 0) src[0] = a.xq;
        __syncthreads();
        qact_to_smem(X, src, 1, (int)a.cols);
    } else {
        for (uint32_t b = warp; b < a.cols / 32; b += kQsWarps)
            qact_block_to_xs(X, 0, (int)b, __ldcg(a.xf + 32 * b + lane), lane);
    }
    __syncthreads();
    XChunk xc;
    if (npass == 1) xchunk_load(X, 0, (int)spread_chunk((uint32_t)lane, 32), xc);
    const int row_l = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
    uint32_t i = 0;
    bool ok = true;
    for (; i < mine; i++) {
        const uint32_t st = i % q.stages;
        if (!mbar_wait_bounded(&bars[st], (i / q.stages) & 1, kWaitLimitNs)) {
            ok = false;
            break;
        }
        const uint32_t r0 = (gw + i * W) * a.rw, nr = min(a.rw, a.nrows - r0);
        const uint8_t *t = ring + (size_t)st * q.stage;
        float v[kQsWideRows];
#pragma unroll
        for (int r = 0; r < (int)kQsWideRows; r++) v[r] = 0.0f;
        for (uint32_t p = 0; p < npass; p++) {
            const uint32_t n = min(32u, cpr - 32 * p);
            if ((uint32_t)lane < n) {
                const uint32_t cb = 32 * p + spread_chunk((uint32_t)lane, n);
                if (npass > 1) xchunk_load(X, 0, (int)cb, xc);
#pragma unroll
                for (int r = 0; r < (int)kQsWideRows; r++)
                    if ((uint32_t)r < nr) v[r] += dot64<TYPE>(t + (size_t)r * a.pitch, (int)cb, (int)a.nblocks, xc);
            }
        }
        __syncwarp();
        if (lane == 0 && i + q.stages < mine) {  // the stage is read: the group after next takes it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(i + q.stages);
        }
        const float sum = qs_transpose_sum(v, lane);
        if ((lane & 3) == 0 && (uint32_t)row_l < nr) {
            const size_t yi = r0 + row_l;
            a.y[yi] = a.add ? __fadd_rn(a.add[yi], sum) : sum;
        }
    }
    if (!ok && lane == 0) {
        if (a.dev_err) atomicExch(a.dev_err, DEV_ERR_TMA_TIMEOUT);
        for (uint32_t j = i; j < min(mine, i + q.stages); j++)
            mbar_wait_bounded(&bars[j % q.stages], (j / q.stages) & 1, kWaitLimitNs);
    }
}

// Measured on the lm_heads: Q8_0 rows (d 896) run faster with register-held
// chunks (33 vs 37 us for 145 MB); Q6_K rows (d 2048, 2816) slower (86 vs 80,
// 265 vs 222 us), so the K types keep one item per lane.
static bool qs64_type(uint32_t t) { return t == T_Q8_0; }
// Q8_0 rows of 32+ chunks: the wide-row kernel (measured on a 151936 x 2048
// matrix: 54 us against 60 for k_qmv_stream64).  For Q6_K it measured no
// faster at 2048 columns (70 vs 72 us) and slower at 2816 (242 vs 212 us: the
// second pass over 12 of 44 chunks idles 20 lanes), so the K types keep one
// superblock per lane.
static bool qsw_type(const DevMat &m) { return m.type == T_Q8_0 && qs_chunks(m.cols) >= 32; }

// The ring layout for a one-token matvec over m, or false when the persistent
// kernel does not pay (few rows) or two stages per warp do not fit.
static bool qs_plan(const DevMat &m, uint32_t rw, uint32_t ipr, int num_sms, uint32_t &stages, uint32_t &stage,
                    uint32_t &warps, size_t &smem) {
    if (!is_quant_type(m.type) || num_sms <= 0 || ipr > 32) return false;  // a group's items: one per lane
    if (m.rows * m.pitch < ((uint64_t)32 << 20) || qmv_ctas(m) <= 4u * (uint32_t)num_sms) return false;
    stage = (uint32_t)((rw * m.pitch + 127) & ~(uint64_t)127);
    size_t fixed = qs_ring_offset((int)ipr) + 256;  // + slack: a Q8_0 chunk reads past its row
    if (qs64_type(m.type) && !qsw_type(m))
        fixed += kQsWarps * (((size_t)rw * qs_chunks((uint32_t)m.cols) * 4 + 127) & ~(size_t)127);
    for (warps = kQsWarps; warps >= 8; warps -= 4) {  // at least two stages per warp
        if (fixed + (size_t)2 * warps * stage > kDecodeSmemLimit) continue;
        stages = (uint32_t)min((size_t)kQsMaxStages, (kDecodeSmemLimit - fixed) / ((size_t)warps * stage));
        smem = fixed + (size_t)stages * warps * stage;
        return true;
    }
    return false;
}

// Rows per group: one item per lane (k_qmv_stream), or about 6 KB of rows
// (k_qmv_stream64, at most 8).
static uint32_t qs_rows(const DevMat &m, uint32_t ipr) {
    if (qsw_type(m)) {  // about 7 KB of rows per group, at most kQsWideRows
        const uint64_t r = 7168 / m.pitch;
        return r < 1 ? 1u : r > kQsWideRows ? kQsWideRows : (uint32_t)r;
    }
    if (!qs64_type(m.type)) return max(1u, 32u / ipr);
    const uint64_t r = 6144 / m.pitch;
    return r < 1 ? 1u : r > 8 ? 8u : (uint32_t)r;
}

bool qmv_streams(const DevMat &m, uint32_t ntok, int num_sms) {
    if (ntok != 1 || !is_quant_type(m.type)) return false;
    const uint32_t ipr = items_per_row(m.type, m.cols), rw = qs_rows(m, ipr);
    uint32_t stages, stage, warps;
    size_t smem;
    return qs_plan(m, rw, ipr, num_sms, stages, stage, warps, smem);
}

template <uint32_t TYPE>
static cudaError_t launch_qs_t(const LaunchCfg &c, const QsArgs &q, size_t smem, bool wide) {
    if constexpr (TYPE == T_Q8_0)
        if (wide)
            return launch_k(c, type_label<TYPE>("qmv_stream"), k_qmv_stream_w<TYPE>, dim3((unsigned)c.num_sms),
                            dim3(kQsWarps * 32), smem, q);
    if constexpr (TYPE == T_Q8_0)
        return launch_k(c, type_label<TYPE>("qmv_stream"), k_qmv_stream64<TYPE>, dim3((unsigned)c.num_sms),
                        dim3(kQsWarps * 32), smem, q);
    else
        return launch_k(c, type_label<TYPE>("qmv_stream"), k_qmv_stream<TYPE>, dim3((unsigned)c.num_sms),
                        dim3(kQsWarps * 32), smem, q);
}

static cudaError_t launch_qmv_stream(const LaunchCfg &c, const DevMat &m, QmvArgs a) {
    QsArgs q;
    const bool wide = qsw_type(m);
    a.rw = qs_rows(m, a.nitems);
    q.a = a;
    size_t smem;
    if (!qs_plan(m, a.rw, a.nitems, c.num_sms, q.stages, q.stage, q.warps, smem)) return cudaErrorInvalidValue;
    switch (m.type) {
    case T_Q4_K: return launch_qs_t<T_Q4_K>(c, q, smem, wide);
    case T_Q6_K: return launch_qs_t<T_Q6_K>(c, q, smem, wide);
    case T_Q8_0: return launch_qs_t<T_Q8_0>(c, q, smem, wide);
    case T_Q5_0: return launch_qs_t<T_Q5_0>(c, q, smem, wide);
    case T_Q5_1: return launch_qs_t<T_Q5_1>(c, q, smem, wide);
    case T_IQ4_NL: return launch_qs_t<T_IQ4_NL>(c, q, smem, wide);
    case T_Q5_K: return launch_qs_t<T_Q5_K>(c, q, smem, wide);
    case T_Q3_K: return launch_qs_t<T_Q3_K>(c, q, smem, wide);
    default: return cudaErrorInvalidValue;
    }
}

uint32_t qmv_ctas(const DevMat &m) {
    const uint32_t rw = max(1u, 32u / items_per_row(m.type, m.cols));
    return (uint32_t)((m.rows + kQmvWarps * rw - 1) / (kQmvWarps * rw));
}

template <uint32_t TYPE, int NT>
static cudaError_t launch_qmv_t(const LaunchCfg &c, const QmvArgs &a) {
    const size_t smem = qmv_smem_bytes(a.pitch, a.rw, NT, (int)a.nitems);
    const uint32_t rows_per_cta = kQmvWarps * a.rw;
    const dim3 grid((a.nrows + rows_per_cta - 1) / rows_per_cta);
    return launch_k(c, type_label<TYPE>("qmv"), k_qmv<TYPE, NT>, grid, dim3(kQmvWarps * 32), smem, a);
}

cudaError_t launch_qmatvec(const LaunchCfg &c, const DevMat &m, uint32_t expert, const uint8_t *xq,
                           uint64_t xq_pitch, const float *x, float *y, uint32_t ntok, const float *add) {
    const uint8_t *rows = m.data + (uint64_t)expert * m.rows * m.pitch;
    if (m.type == T_F32 || m.type == T_F16) {
        const uint64_t want = (m.rows + 7) / 8;
        const uint32_t blocks = (uint32_t)(want < 65535 ? want : 65535);
        return launch_k(c, "qmv_float", k_mv_float, dim3(blocks), dim3(256), 0, rows, m.pitch, m.type,
                        (uint32_t)m.rows, (uint32_t)m.cols, x, y, ntok, add);
    }
    QmvArgs a;
    a.rows = rows;
    a.pitch = m.pitch;
    a.nrows = (uint32_t)m.rows;
    a.cols = (uint32_t)m.cols;
    a.nitems = items_per_row(m.type, m.cols);
    a.nblocks = (uint32_t)(m.cols / 32);
    a.xq = xq;
    a.xq_pitch = xq_pitch;
    a.xf = x;
    a.norm_w = nullptr;
    a.eps = 0.0f;
    if (!xq && ntok != 1) return cudaErrorInvalidValue;
    a.y = y;
    a.add = add;
    a.ntok = ntok;
    a.rw = max(1u, 32u / a.nitems);
    a.dev_err = c.dev_err;
    if (qmv_streams(m, ntok, c.num_sms)) return launch_qmv_stream(c, m, a);
    const bool one = ntok == 1;
    switch (m.type) {
    case T_Q4_K: return one ? launch_qmv_t<T_Q4_K, 1>(c, a) : launch_qmv_t<T_Q4_K, 4>(c, a);
    case T_Q6_K: return one ? launch_qmv_t<T_Q6_K, 1>(c, a) : launch_qmv_t<T_Q6_K, 2>(c, a);
    case T_Q8_0: return one ? launch_qmv_t<T_Q8_0, 1>(c, a) : launch_qmv_t<T_Q8_0, 4>(c, a);
    case T_Q5_0: return one ? launch_qmv_t<T_Q5_0, 1>(c, a) : launch_qmv_t<T_Q5_0, 4>(c, a);
    case T_Q5_1: return one ? launch_qmv_t<T_Q5_1, 1>(c, a) : launch_qmv_t<T_Q5_1, 4>(c, a);
    case T_IQ4_NL: return one ? launch_qmv_t<T_IQ4_NL, 1>(c, a) : launch_qmv_t<T_IQ4_NL, 4>(c, a);
    case T_Q5_K: return one ? launch_qmv_t<T_Q5_K, 1>(c, a) : launch_qmv_t<T_Q5_K, 4>(c, a);
    case T_Q3_K: return one ? launch_qmv_t<T_Q3_K, 1>(c, a) : launch_qmv_t<T_Q3_K, 2>(c, a);
    default: return cudaErrorInvalidValue;
    }
}

static QmvArgs qmv_args_one(const LaunchCfg &c, const DevMat &m, const float *x, float *y, const float *norm_w,
                            float eps) {
    QmvArgs a{};
    a.rows = m.data;
    a.pitch = m.pitch;
    a.nrows = (uint32_t)m.rows;
    a.cols = (uint32_t)m.cols;
    a.nitems = items_per_row(m.type, m.cols);
    a.nblocks = (uint32_t)(m.cols / 32);
    a.xq = nullptr;
    a.xq_pitch = 0;
    a.xf = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.y = y;
    a.add = nullptr;
    a.ntok = 1;
    a.rw = max(1u, 32u / a.nitems);
    a.dev_err = c.dev_err;
    return a;
}

cudaError_t launch_qmatvec_multi(const LaunchCfg &c, uint32_t n, const DevMat *const *m, const float *x,
                                 const float *norm_w, float eps, float *const *y) {
    if (n == 0 || n > (uint32_t)kQmvMaxSeg) return cudaErrorInvalidValue;
    QmvMulti q{};
    q.n = n;
    size_t smem = 0;
    uint32_t ctas = 0;
    for (uint32_t s = 0; s < n; s++) {
        if (!is_quant_type(m[s]->type)) return cudaErrorInvalidValue;
        q.seg[s] = qmv_args_one(c, *m[s], x, y[s], norm_w, eps);
        q.type[s] = m[s]->type;
        q.begin[s] = ctas;
        ctas += qmv_ctas(*m[s]);
        const size_t b = qmv_smem_bytes(q.seg[s].pitch, q.seg[s].rw, 1, (int)q.seg[s].nitems);
        smem = b > smem ? b : smem;
    }
    q.begin[n] = ctas;
    return launch_k(c, "qmv_multi", k_qmv_multi, dim3(ctas), dim3(kQmvWarps * 32), smem, q);
}

}  // namespace lt
