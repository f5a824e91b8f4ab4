// lt_kernels.cu — sm_100a kernels for the quantized MoE forward path.
//
// Weight rows stream global -> shared memory with 1-D TMA bulk copies
// (cp.async.bulk + mbarrier) while the CTA quantises its activation rows to
// int16 per 32-element block in shared memory.  Each thread then decodes one
// "item" (a Q4_K/Q6_K superblock, or a group of eight Q8_0 blocks) against the
// activations with dp2a integer dot products, applies the block scales in
// f32, and per-row partial sums are reduced in a fixed order.
#include <cfloat>
#include <utility>

#include "lt_common.cuh"
#include "lt_decode.cuh"
#include "lt_internal.h"

namespace lt {

// ── GGUF type table (src/gguf/types.zig:138-173, src/ops/math.zig:194) ─────

bool type_supported(uint32_t t) {
    return t == T_F32 || t == T_F16 || t == T_Q8_0 || t == T_Q4_K || t == T_Q6_K;
}

uint32_t block_elems_of(uint32_t t) {
    switch (t) {
    case T_F32:
    case T_F16: return 1;
    case T_Q8_0: return 32;
    case T_Q4_K:
    case T_Q6_K: return 256;
    default: return 0;
    }
}

uint64_t row_bytes_of(uint32_t t, uint64_t cols) {
    switch (t) {
    case T_F32: return cols * 4;
    case T_F16: return cols * 2;
    case T_Q8_0: return (cols / 32) * 34;
    case T_Q4_K: return (cols / 256) * 144;
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

template <typename Kern, typename... Args>
static cudaError_t launch_k(const LaunchCfg &c, const char *label, Kern kern, dim3 grid, dim3 block, size_t smem,
                            Args... args) {
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    cfg.numAttrs = 0;
    const bool timed = c.prof && c.prof->on;
    if (c.pdl && !timed) {  // events between kernels would serialise them anyway
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    Profiler::Rec rec;
    if (timed) c.prof->begin(label, c.stream, rec);
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
    if (timed) c.prof->end(rec, c.stream);
    return e;
}

// Static per-type profiler labels for "qmv", "moe_gate_up" and "moe_down".
template <uint32_t TYPE>
static const char *type_label(const char *kind) {
    static const char *const names[3][3] = {{"qmv_q4k", "qmv_q6k", "qmv_q8_0"},
                                            {"moe_gate_up_q4k", "moe_gate_up_q6k", "moe_gate_up_q8_0"},
                                            {"moe_down_q4k", "moe_down_q6k", "moe_down_q8_0"}};
    const int t = TYPE == T_Q4_K ? 0 : TYPE == T_Q6_K ? 1 : 2;
    const int k = kind[0] == 'q' ? 0 : kind[4] == 'g' ? 1 : 2;
    return names[k][t];
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

cudaError_t launch_dequant(const LaunchCfg &c, const DevMat &m, uint64_t row0, uint64_t nrows, float *out) {
    const uint64_t n = nrows * m.cols;
    if (n == 0) return cudaSuccess;
    const uint64_t want = (n + 255) / 256;
    const unsigned grid = (unsigned)(want < 65535ull * 8 ? want : 65535ull * 8);
    return launch_k(c, "dequant", k_dequant, dim3(grid), dim3(256), 0, m.data, m.type, m.pitch, m.cols, row0, n, out);
}

// Activation quantisation and block decoders: lt_decode.cuh.

// ── shared-memory tile bookkeeping ─────────────────────────────────────────

struct TileSmem {
    uint64_t *bar;
    const float **src;
    uint8_t *tile;
    XS X;
    float *part;
};

constexpr int kMaxSrc = 16;
constexpr int kTileSlack = 256;  // item decoders may read up to 224 B past a row

__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~(size_t)15; }

__host__ __device__ inline size_t tile_smem_bytes(size_t tile_bytes, int ntok_x, int nitems, int npart) {
    return 16 + align16(kMaxSrc * sizeof(void *)) + align16(tile_bytes + kTileSlack) +
           align16(xs_bytes(ntok_x, nitems)) + (size_t)npart * 4;
}

LT_DEVINL TileSmem tile_carve(uint8_t *smem, size_t tile_bytes, int ntok_x, int nitems) {
    TileSmem s;
    uint8_t *p = smem;
    s.bar = reinterpret_cast<uint64_t *>(p);
    p += 16;
    s.src = reinterpret_cast<const float **>(p);
    p += align16(kMaxSrc * sizeof(void *));
    s.tile = p;
    p += align16(tile_bytes + kTileSlack);
    s.X = xs_carve(p, ntok_x, nitems);
    p += align16(xs_bytes(ntok_x, nitems));
    s.part = reinterpret_cast<float *>(p);
    return s;
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// All threads wait for the tile.  On timeout: record, wait once more, give up.
LT_DEVINL bool tile_wait(uint64_t *bar, int *dev_err) {
    if (mbar_wait_bounded(bar, 0, kWaitLimitNs)) return true;
    if (dev_err) atomicExch(dev_err, DEV_ERR_TMA_TIMEOUT);
    mbar_wait_bounded(bar, 0, kWaitLimitNs);
    return false;
}

LT_DEVINL float act_apply(int act, float g) {
    if (act == 1) {  // src/ops/math.zig:85-88
        const float c = 0.7978845608028654f;
        return 0.5f * g * (1.0f + tanhf(c * (g + 0.044715f * g * g * g)));
    }
    return g / (1.0f + expf(-g));  // src/ops/math.zig:38-40
}

// ── dense quantised matvec: quantMatvec(Par), src/ops/math.zig:133-320 ─────

struct QmvArgs {
    const uint8_t *rows;  // first row of the (expert) matrix
    uint64_t pitch;
    uint32_t nrows, cols, nitems, nblocks;
    const float *x;
    float *y;
    uint32_t ntok;
    uint32_t rt;  // rows per CTA
    int *dev_err;
};

template <uint32_t TYPE, int NT>
__global__ void __launch_bounds__(256) k_qmv(QmvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t r0 = blockIdx.x * a.rt;
    const uint32_t nr = min(a.rt, a.nrows - r0);
    const int ipr = (int)a.nitems;
    const int total = (int)nr * ipr;
    TileSmem S = tile_carve(smem, (size_t)a.rt * a.pitch, NT, ipr);
    if (threadIdx.x == 0) {
        mbar_init(S.bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // weights are static: fetch before waiting on the producer
        const uint32_t bytes = (uint32_t)(nr * a.pitch);
        mbar_arrive_expect_tx(S.bar, bytes);
        tma_load_1d(S.tile, a.rows + (uint64_t)r0 * a.pitch, bytes, S.bar);
    }
    pdl_launch_dependents();
    pdl_wait();
    bool ok = true;
    for (uint32_t c0 = 0; c0 < a.ntok; c0 += NT) {
        const int nt = (int)min((uint32_t)NT, a.ntok - c0);
        if (threadIdx.x < (unsigned)nt) S.src[threadIdx.x] = a.x + (size_t)(c0 + threadIdx.x) * a.cols;
        __syncthreads();
        prep_x(S.X, S.src, nt, (int)a.cols);
        if (c0 == 0) ok = tile_wait(S.bar, a.dev_err);
        __syncthreads();
        if (!ok) return;
        for (int f = threadIdx.x; f < total; f += blockDim.x) {
            const int item = f % ipr, row = f / ipr;
            float res[NT];
#pragma unroll
            for (int t = 0; t < NT; t++) res[t] = 0.0f;
            dot_item<TYPE, NT>(S.tile + (size_t)row * a.pitch, item, (int)a.nblocks, S.X, 0, nt, res);
#pragma unroll
            for (int t = 0; t < NT; t++)
                if (t < nt) S.part[t * total + f] = res[t];
        }
        __syncthreads();
        for (int idx = threadIdx.x; idx < nt * (int)nr; idx += blockDim.x) {
            const int t = idx / (int)nr, r = idx - t * (int)nr;
            const float *p = S.part + t * total + r * ipr;
            float s = 0.0f;
            for (int i = 0; i < ipr; i++) s += p[i];
            a.y[(size_t)(c0 + t) * a.nrows + r0 + r] = s;
        }
        __syncthreads();
    }
}

// f32 / f16 rows: one warp per row, plain loads.
__global__ void k_mv_float(const uint8_t *rows, uint64_t pitch, uint32_t type, uint32_t nrows, uint32_t cols,
                           const float *x, float *y, uint32_t ntok) {
    pdl_wait();
    const uint32_t warps = (blockDim.x >> 5) * gridDim.x;
    for (uint32_t r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < nrows; r += warps) {
        const uint8_t *row = rows + (uint64_t)r * pitch;
        for (uint32_t t = 0; t < ntok; t++) {
            const float *xt = x + (size_t)t * cols;
            float s = 0.0f;
            for (uint32_t i = threadIdx.x & 31; i < cols; i += 32) {
                const float w = type == T_F32 ? reinterpret_cast<const float *>(row)[i]
                                              : f16_at(row + 2 * i);
                s += w * xt[i];
            }
            s = warp_sum(s);
            if ((threadIdx.x & 31) == 0) y[(size_t)t * nrows + r] = s;
        }
    }
}

static uint32_t items_per_row(uint32_t type, uint64_t cols) {
    if (type == T_Q8_0) return (uint32_t)((cols / 32 + 7) / 8);
    return (uint32_t)(cols / 256);
}

template <uint32_t TYPE>
static cudaError_t launch_qmv_t(const LaunchCfg &c, const DevMat &m, const uint8_t *rows, const float *x,
                                float *y, uint32_t ntok) {
    constexpr int NT = 4;
    QmvArgs a;
    a.rows = rows;
    a.pitch = m.pitch;
    a.nrows = (uint32_t)m.rows;
    a.cols = (uint32_t)m.cols;
    a.nitems = items_per_row(TYPE, m.cols);
    a.nblocks = (uint32_t)(m.cols / 32);
    a.x = x;
    a.y = y;
    a.ntok = ntok;
    a.rt = max(1u, 256u / a.nitems);
    a.dev_err = c.dev_err;
    const size_t smem = tile_smem_bytes((size_t)a.rt * a.pitch, NT, (int)a.nitems, NT * (int)(a.rt * a.nitems));
    const dim3 grid((a.nrows + a.rt - 1) / a.rt);
    return launch_k(c, type_label<TYPE>("qmv"), k_qmv<TYPE, NT>, grid, dim3(256), smem, a);
}

cudaError_t launch_qmatvec(const LaunchCfg &c, const DevMat &m, uint32_t expert, const float *x, float *y,
                           uint32_t ntok) {
    const uint8_t *rows = m.data + (uint64_t)expert * m.rows * m.pitch;
    switch (m.type) {
    case T_Q4_K: return launch_qmv_t<T_Q4_K>(c, m, rows, x, y, ntok);
    case T_Q6_K: return launch_qmv_t<T_Q6_K>(c, m, rows, x, y, ntok);
    case T_Q8_0: return launch_qmv_t<T_Q8_0>(c, m, rows, x, y, ntok);
    default: {
        const uint64_t want = (m.rows + 7) / 8;
        const uint32_t blocks = (uint32_t)(want < 65535 ? want : 65535);
        return launch_k(c, "qmv_float", k_mv_float, dim3(blocks), dim3(256), 0, rows, m.pitch, m.type, (uint32_t)m.rows,
                        (uint32_t)m.cols, x, y, ntok);
    }
    }
}

// ── MoE: routing plan (dispatch bookkeeping) ───────────────────────────────

__global__ void k_moe_plan(const uint32_t *ids, uint32_t npairs, uint32_t E, MoePlan p) {
    extern __shared__ uint32_t sm_plan[];
    uint32_t *cnt = sm_plan, *cur = sm_plan + E;
    pdl_launch_dependents();
    pdl_wait();
    for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < npairs; i += blockDim.x) {
        const uint32_t e = ids[i];
        if (e < E) atomicAdd(&cnt[e], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t off = 0, n = 0;
        for (uint32_t e = 0; e < E; e++) {
            cur[e] = off;
            if (cnt[e]) {
                p.act_e[n] = e;
                p.act_off[n] = off;
                p.act_cnt[n] = cnt[e];
                n++;
            }
            off += cnt[e];
        }
        *p.n_active = n;
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < npairs; i += blockDim.x) {
        const uint32_t e = ids[i];
        if (e < E) {
            const uint32_t pos = atomicAdd(&cur[e], 1u);
            p.pair_pos[i] = pos;
            p.pos_pair[pos] = i;
        }
    }
}

cudaError_t launch_moe_plan(const LaunchCfg &c, const uint32_t *ids, uint32_t ntok, uint32_t k, uint32_t E,
                            const MoePlan &p) {
    return launch_k(c, "moe_plan", k_moe_plan, dim3(1), dim3(1024), (size_t)2 * E * 4, ids, ntok * k, E, p);
}

// ── MoE: grouped gate/up with fused activation ─────────────────────────────

struct GateUpArgs {
    const uint8_t *gate, *up;  // up == nullptr: fused gate_up tensor
    uint64_t pitch;
    uint32_t F, d, nitems, nblocks;
    int act;
    const float *x;
    uint32_t ntok, k;
    const uint32_t *ids;
    int direct;
    MoePlan p;
    float *h;
    uint32_t rt;
    int *dev_err;
};

template <uint32_t TYPE, int NT>
__global__ void __launch_bounds__(256) k_moe_gate_up(GateUpArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_wait();
    // Release the down kernel only now: it reads the router's ids before its
    // own wait, which is safe once this grid has seen the router complete.
    pdl_launch_dependents();
    uint32_t e, off, cnt;
    if (a.direct) {
        if (blockIdx.y >= a.k) return;
        e = a.ids[blockIdx.y];
        off = blockIdx.y;
        cnt = 1;
    } else {
        if (blockIdx.y >= *a.p.n_active) return;
        e = a.p.act_e[blockIdx.y];
        off = a.p.act_off[blockIdx.y];
        cnt = a.p.act_cnt[blockIdx.y];
    }
    const uint32_t r0 = blockIdx.x * a.rt;
    const uint32_t nr = min(a.rt, a.F - r0);
    const int ipr = (int)a.nitems;
    const int total = 2 * (int)nr * ipr;
    TileSmem S = tile_carve(smem, (size_t)2 * a.rt * a.pitch, NT, ipr);
    if (threadIdx.x == 0) {
        mbar_init(S.bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t bytes = (uint32_t)(nr * a.pitch);
        uint64_t grow, urow;
        const uint8_t *ub;
        if (a.up) {
            grow = (uint64_t)e * a.F + r0;
            urow = grow;
            ub = a.up;
        } else {  // fused: gate rows [0,F), up rows [F,2F) (gemma4/forward.zig:469-471)
            grow = (uint64_t)e * 2 * a.F + r0;
            urow = grow + a.F;
            ub = a.gate;
        }
        mbar_arrive_expect_tx(S.bar, 2 * bytes);
        tma_load_1d(S.tile, a.gate + grow * a.pitch, bytes, S.bar);
        tma_load_1d(S.tile + (size_t)nr * a.pitch, ub + urow * a.pitch, bytes, S.bar);
    }
    bool ok = true;
    for (uint32_t c0 = 0; c0 < cnt; c0 += NT) {
        const int nt = (int)min((uint32_t)NT, cnt - c0);
        if (threadIdx.x < (unsigned)nt) {
            const uint32_t pos = off + c0 + threadIdx.x;
            const uint32_t pair = a.direct ? pos : a.p.pos_pair[pos];
            S.src[threadIdx.x] = a.x + (size_t)(pair / a.k) * a.d;
        }
        __syncthreads();
        prep_x(S.X, S.src, nt, (int)a.d);
        if (c0 == 0) ok = tile_wait(S.bar, a.dev_err);
        __syncthreads();
        if (!ok) return;
        for (int f = threadIdx.x; f < total; f += blockDim.x) {
            const int item = f % ipr, rowm = f / ipr;  // rowm in [0, 2*nr): gate rows then up rows
            float res[NT];
#pragma unroll
            for (int t = 0; t < NT; t++) res[t] = 0.0f;
            dot_item<TYPE, NT>(S.tile + (size_t)rowm * a.pitch, item, (int)a.nblocks, S.X, 0, nt, res);
#pragma unroll
            for (int t = 0; t < NT; t++)
                if (t < nt) S.part[t * total + f] = res[t];
        }
        __syncthreads();
        for (int idx = threadIdx.x; idx < nt * (int)nr; idx += blockDim.x) {
            const int t = idx / (int)nr, r = idx - t * (int)nr;
            const float *pg = S.part + t * total + r * ipr;
            const float *pu = pg + (int)nr * ipr;
            float g = 0.0f, u = 0.0f;
            for (int i = 0; i < ipr; i++) {
                g += pg[i];
                u += pu[i];
            }
            a.h[(size_t)(off + c0 + t) * a.F + r0 + r] = act_apply(a.act, g) * u;
        }
        __syncthreads();
    }
}

template <uint32_t TYPE>
static cudaError_t launch_gate_up_t(const LaunchCfg &c, const DevMat &gate, const DevMat &up, int act,
                                    const float *x, uint32_t ntok, uint32_t k, const uint32_t *ids, bool direct,
                                    const MoePlan &p, float *h) {
    constexpr int NT = 4;
    GateUpArgs a;
    const bool fused = up.data == nullptr;
    a.gate = gate.data;
    a.up = up.data;
    a.pitch = gate.pitch;
    a.F = (uint32_t)(fused ? gate.rows / 2 : gate.rows);
    a.d = (uint32_t)gate.cols;
    a.nitems = items_per_row(TYPE, gate.cols);
    a.nblocks = (uint32_t)(gate.cols / 32);
    a.act = act;
    a.x = x;
    a.ntok = ntok;
    a.k = k;
    a.ids = ids;
    a.direct = direct ? 1 : 0;
    a.p = p;
    a.h = h;
    a.rt = max(1u, 256u / (2 * a.nitems));
    a.dev_err = c.dev_err;
    const size_t smem =
        tile_smem_bytes((size_t)2 * a.rt * a.pitch, NT, (int)a.nitems, NT * (int)(2 * a.rt * a.nitems));
    const uint32_t E = gate.n_experts ? gate.n_experts : 1;
    const uint32_t ny = direct ? k : min(E, ntok * k);
    const dim3 grid((a.F + a.rt - 1) / a.rt, ny);
    return launch_k(c, type_label<TYPE>("moe_gate_up"), k_moe_gate_up<TYPE, NT>, grid, dim3(256), smem, a);
}

cudaError_t launch_moe_gate_up(const LaunchCfg &c, const DevMat &gate, const DevMat &up, int act, const float *x,
                               uint32_t ntok, uint32_t k, const uint32_t *ids, bool direct, const MoePlan &p,
                               float *h) {
    switch (gate.type) {
    case T_Q4_K: return launch_gate_up_t<T_Q4_K>(c, gate, up, act, x, ntok, k, ids, direct, p, h);
    case T_Q6_K: return launch_gate_up_t<T_Q6_K>(c, gate, up, act, x, ntok, k, ids, direct, p, h);
    case T_Q8_0: return launch_gate_up_t<T_Q8_0>(c, gate, up, act, x, ntok, k, ids, direct, p, h);
    default: return cudaErrorInvalidValue;
    }
}

// ── MoE: down projection with the weighted combine fused ───────────────────

struct DownArgs {
    const uint8_t *down;
    uint64_t pitch;
    uint32_t D, F, nitems, nblocks;  // down: [E][D rows][F cols]
    const float *h;
    uint32_t ntok, k;
    const uint32_t *ids;
    const float *w;
    int direct;
    MoePlan p;
    float *out;
    uint32_t rt;
    int *dev_err;
};

template <uint32_t TYPE>
__global__ void __launch_bounds__(256) k_moe_down(DownArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    // Launched early (programmatic dependent launch) while the gate/up kernel
    // runs.  That kernel only released its dependents after its own wait, so
    // the router (and the dispatch plan) have completed: the expert ids are
    // final and this CTA's down-projection weights can stream in now.  The
    // activations h are read only after pdl_wait().
    pdl_launch_dependents();
    const uint32_t t = blockIdx.y;
    const uint32_t r0 = blockIdx.x * a.rt;
    const uint32_t nr = min(a.rt, a.D - r0);
    const int ipr = (int)a.nitems;
    const int k = (int)a.k;
    const int total = k * (int)nr * ipr;
    TileSmem S = tile_carve(smem, (size_t)k * a.rt * a.pitch, k, ipr);
    if (threadIdx.x == 0) {
        mbar_init(S.bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t bytes = (uint32_t)(nr * a.pitch);
        mbar_arrive_expect_tx(S.bar, (uint32_t)k * bytes);
        for (int s = 0; s < k; s++) {
            const uint32_t e = __ldcg(a.ids + t * a.k + s);
            tma_load_1d(S.tile + (size_t)s * nr * a.pitch, a.down + ((uint64_t)e * a.D + r0) * a.pitch, bytes,
                        S.bar);
        }
    }
    if (threadIdx.x < (unsigned)k) {
        const uint32_t pair = t * a.k + threadIdx.x;
        const uint32_t pos = a.direct ? pair : __ldcg(a.p.pair_pos + pair);
        S.src[threadIdx.x] = a.h + (size_t)pos * a.F;
    }
    pdl_wait();
    __syncthreads();
    prep_x(S.X, S.src, k, (int)a.F);
    const bool ok = tile_wait(S.bar, a.dev_err);
    __syncthreads();
    if (!ok) return;
    for (int f = threadIdx.x; f < total; f += blockDim.x) {
        const int item = f % ipr, rs = f / ipr;  // rs = slot*nr + row
        const int slot = rs / (int)nr;
        float res[1] = {0.0f};
        dot_item<TYPE, 1>(S.tile + (size_t)rs * a.pitch, item, (int)a.nblocks, S.X, slot, 1, res);
        S.part[f] = res[0];
    }
    __syncthreads();
    for (int r = threadIdx.x; r < (int)nr; r += blockDim.x) {
        float o = 0.0f;  // moe_buf is zeroed, then += scale * down, slot by slot
        for (int s = 0; s < k; s++) {
            const float *p = S.part + (s * (int)nr + r) * ipr;
            float y = 0.0f;
            for (int i = 0; i < ipr; i++) y += p[i];
            o += a.w[t * a.k + s] * y;
        }
        a.out[(size_t)t * a.D + r0 + r] = o;
    }
}

template <uint32_t TYPE>
static cudaError_t launch_down_t(const LaunchCfg &c, const DevMat &down, const float *h, uint32_t ntok, uint32_t k,
                                 const uint32_t *ids, const float *w, bool direct, const MoePlan &p, float *out) {
    DownArgs a;
    a.down = down.data;
    a.pitch = down.pitch;
    a.D = (uint32_t)down.rows;
    a.F = (uint32_t)down.cols;
    a.nitems = items_per_row(TYPE, down.cols);
    a.nblocks = (uint32_t)(down.cols / 32);
    a.h = h;
    a.ntok = ntok;
    a.k = k;
    a.ids = ids;
    a.w = w;
    a.direct = direct ? 1 : 0;
    a.p = p;
    a.out = out;
    a.rt = max(1u, 256u / (k * a.nitems));
    a.dev_err = c.dev_err;
    const size_t smem = tile_smem_bytes((size_t)k * a.rt * a.pitch, (int)k, (int)a.nitems, (int)(k * a.rt * a.nitems));
    const dim3 grid((a.D + a.rt - 1) / a.rt, ntok);
    return launch_k(c, type_label<TYPE>("moe_down"), k_moe_down<TYPE>, grid, dim3(256), smem, a);
}

cudaError_t launch_moe_down(const LaunchCfg &c, const DevMat &down, const float *h, uint32_t ntok, uint32_t k,
                            const uint32_t *ids, const float *w, bool direct, const MoePlan &p, float *out) {
    switch (down.type) {
    case T_Q4_K: return launch_down_t<T_Q4_K>(c, down, h, ntok, k, ids, w, direct, p, out);
    case T_Q6_K: return launch_down_t<T_Q6_K>(c, down, h, ntok, k, ids, w, direct, p, out);
    case T_Q8_0: return launch_down_t<T_Q8_0>(c, down, h, ntok, k, ids, w, direct, p, out);
    default: return cudaErrorInvalidValue;
    }
}

// ── router: routerTopKSoftmax (src/model/gemma4/forward.zig:648-668) ───────
// Each warp computes one expert's logit with dotf32's exact evaluation order
// (src/ops/math.zig:96-116): lane l owns the chain over elements l, l+32, ...
// (acc_{l/8}[l%8] in the reference), combined as (a0+a1)+(a2+a3), then the
// 8-wide tail, the ordered 8-lane reduction and the scalar tail.  The last
// CTA of each token group selects the top-k.

constexpr int kRouterWarps = 4;  // experts per CTA
constexpr int kRouterTok = 4;    // tokens per CTA

uint32_t router_token_groups(uint32_t ntok) { return (ntok + kRouterTok - 1) / kRouterTok; }

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

__global__ void __launch_bounds__(kRouterWarps * 32)
    k_router(const float *W, uint32_t E, uint32_t cols, uint32_t w_ld, const float *x, uint32_t ntok, uint32_t k,
             int norm_topk, const float *escale, uint32_t *ids, float *wout, float *logits, uint32_t *counters) {
    extern __shared__ __align__(16) float xsm[];  // [kRouterTok][cols]
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t e = blockIdx.x * kRouterWarps + warp;
    const uint32_t t0 = blockIdx.y * kRouterTok;
    const uint32_t nt = min((uint32_t)kRouterTok, ntok - t0);
    const uint32_t n32 = cols & ~31u;
    // router weights are static: fetch them while the producer of x finishes
    float w0[kRouterChunk];
#pragma unroll
    for (int j = 0; j < kRouterChunk; j++)
        w0[j] = (e < E && 32u * j < n32) ? __ldg(W + (size_t)e * w_ld + 32 * j + lane) : 0.0f;
    pdl_launch_dependents();
    pdl_wait();
    {
        const float *xt = x + (size_t)t0 * cols;
        const uint32_t n = nt * cols;
        if ((cols & 3) == 0 && (reinterpret_cast<uintptr_t>(xt) & 15) == 0) {
            for (uint32_t i = threadIdx.x; i < n / 4; i += blockDim.x)
                reinterpret_cast<float4 *>(xsm)[i] = reinterpret_cast<const float4 *>(xt)[i];
        } else {
            for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) xsm[i] = xt[i];
        }
    }
    __syncthreads();
    if (e < E) {
        for (uint32_t tt = 0; tt < nt; tt++) {
            const float v = router_logit(W + (size_t)e * w_ld, xsm + tt * cols, cols, lane, w0);
            if (lane == 0) logits[(size_t)(t0 + tt) * E + e] = v;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t ticket = atomicAdd(&counters[blockIdx.y], 1u);
        s_last = ticket == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // top-k + softmax statistics, one warp per token
    for (uint32_t tt = warp; tt < nt; tt += kRouterWarps) {
        const float *lg = logits + (size_t)(t0 + tt) * E;
        float v[kRouterMaxE / 32];
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < kRouterMaxE / 32; j++) {
            const uint32_t ee = lane + 32 * j;
            v[j] = ee < E ? __ldcg(lg + ee) : -INFINITY;
            mx = fmaxf(mx, v[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float es = 0.0f;
#pragma unroll
        for (int j = 0; j < kRouterMaxE / 32; j++)
            if (lane + 32 * j < E) es += expf(v[j] - mx);
        es = warp_sum(es);
        uint32_t taken = 0;  // bit j: element lane+32j selected
        float psel[16];
        uint32_t isel[16];
        for (uint32_t i = 0; i < k; i++) {
            // best untaken: larger value, ties -> lower index (strict '>' in insertion order)
            float bv = -INFINITY;
            uint32_t bi = 0xffffffffu;
#pragma unroll
            for (int j = 0; j < kRouterMaxE / 32; j++) {
                const uint32_t ee = lane + 32 * j;
                if (ee < E && !((taken >> j) & 1u) && (v[j] > bv || bi == 0xffffffffu)) {
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
            if (norm_topk)
                for (uint32_t i = 0; i < k; i++) sum += psel[i];
            for (uint32_t i = 0; i < k; i++) {
                float w = norm_topk ? psel[i] / sum : psel[i];
                if (escale) w = escale[isel[i]] * w;
                ids[(size_t)(t0 + tt) * k + i] = isel[i];
                wout[(size_t)(t0 + tt) * k + i] = w;
            }
        }
    }
    if (threadIdx.x == 0) counters[blockIdx.y] = 0;
}

cudaError_t launch_router(const LaunchCfg &c, const float *w, uint32_t E, uint32_t cols, uint32_t w_ld,
                          const float *x, uint32_t ntok, uint32_t k, int norm_topk, const float *escale, uint32_t *ids,
                          float *wout, float *logits, uint32_t *counters) {
    const dim3 grid((E + kRouterWarps - 1) / kRouterWarps, router_token_groups(ntok));
    const size_t smem = (size_t)kRouterTok * cols * 4;
    return launch_k(c, "router_topk", k_router, grid, dim3(kRouterWarps * 32), smem, w, E, cols, w_ld, x, ntok, k,
                    norm_topk, escale, ids, wout, logits, counters);
}

// ── rmsnorm / softmax / argmax ─────────────────────────────────────────────

LT_DEVINL float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
    for (int i = 0; i < nw; i++) s += red[i];
    return s;
}

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
    constexpr int kBatch = 16;
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const float *xt = x + (size_t)blockIdx.x * n;
    float *yt = y + (size_t)blockIdx.x * n;
    float ss = 0.0f;
    for (uint32_t base = threadIdx.x; base < n; base += kBatch * blockDim.x) {
        float v[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; j++) {
            const uint32_t i = base + j * blockDim.x;
            v[j] = i < n ? xt[i] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kBatch; j++) ss += v[j] * v[j];
    }
    ss = block_sum(ss, red);
    const float rms_inv = 1.0f / sqrtf(ss / (float)n + eps);
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

__global__ void k_argmax(const float *x, uint32_t n, uint32_t *idx, float *pv, uint32_t *pi, uint32_t *counters) {
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
    idx[t] = fi;
    counters[t] = 0;
}

cudaError_t launch_argmax(const LaunchCfg &c, const float *x, uint32_t n, uint32_t ntok, uint32_t *idx, float *pv,
                          uint32_t *pi, uint32_t *counters) {
    const uint32_t nb = max(1u, min(64u, (n + 4095) / 4096));
    return launch_k(c, "argmax", k_argmax, dim3(nb, ntok), dim3(256), 0, x, n, idx, pv, pi, counters);
}

}  // namespace lt
