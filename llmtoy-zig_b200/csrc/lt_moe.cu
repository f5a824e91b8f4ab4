// lt_moe.cu — token->expert dispatch, grouped expert gate/up, and the down
// projection with the weighted combine fused (src/model/gemma4/forward.zig:
// 463-479, src/ops/moe.zig:61-76).
//
// Every warp owns a few weight rows: its lane 0 issues one TMA bulk copy per
// matrix into the warp's slice of shared memory, signalling a per-warp
// mbarrier, so each warp computes as soon as its own rows land.  Activations
// arrive pre-quantised (lt_qact.cuh) and are copied, not re-quantised.
#include "lt_qact.cuh"

namespace lt {

size_t qact_row_pitch(uint64_t cols) { return qact_pitch(cols); }

// ── activation quantiser (for ops whose input comes from the caller) ────────

__global__ void k_quantize(const float *x, uint32_t cols, uint32_t nrows, uint8_t *q, uint64_t qpitch) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t nblk = cols / 32;
    const uint32_t gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (gw >= nrows * nblk) return;
    const uint32_t r = gw / nblk, b = gw - r * nblk;
    const int lane = threadIdx.x & 31;
    const float v = x[(size_t)r * cols + 32 * b + lane];
    qact_store_block(q + (size_t)r * qpitch, (int)cols, (int)b, v, lane);
}

cudaError_t launch_quantize(const LaunchCfg &c, const float *x, uint32_t cols, uint32_t nrows, uint8_t *q,
                            uint64_t qpitch) {
    const uint32_t warps = nrows * (cols / 32);
    return launch_k(c, "quantize", k_quantize, dim3((warps + 7) / 8), dim3(256), 0, x, cols, nrows, q, qpitch);
}

// ── routing plan (dispatch bookkeeping for more than one token) ───────────────

// Pairs whose id is not below E (an invalid caller id) get no position: the
// down kernel skips them and the context's error word records it.
constexpr uint32_t kNoPos = 0xffffffffu;

__global__ void k_moe_plan(const uint32_t *ids, uint32_t npairs, uint32_t E, MoePlan p, int *dev_err) {
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
        } else {
            p.pair_pos[i] = kNoPos;
            if (dev_err) atomicExch(dev_err, DEV_ERR_BAD_INDEX);
        }
    }
}

cudaError_t launch_moe_plan(const LaunchCfg &c, const uint32_t *ids, uint32_t ntok, uint32_t k, uint32_t E,
                            const MoePlan &p) {
    return launch_k(c, "moe_plan", k_moe_plan, dim3(1), dim3(1024), (size_t)2 * E * 4, ids, ntok * k, E, p, c.dev_err);
}

// ── grouped gate/up with the activation fused ────────────────────────────────
// A CTA covers 8 rows of one expert (each of its 4 warps: 2 gate rows and the
// same 2 up rows, one superblock per lane at 2048 columns).  The 8 finished h
// values go to an f32 buffer; the last of the 4 CTAs that share a 32-element
// block (device-scope counter, reset by that CTA) quantises the block.

constexpr int kGuWarps = 4;
constexpr int kGuRowsPerWarp = 2;
constexpr int kGuRows = kGuWarps * kGuRowsPerWarp;  // 8
constexpr int kGuCtasPerBlock = 32 / kGuRows;       // 4

struct GateUpArgs {
    const uint8_t *gate, *up;  // up == nullptr: fused gate_up tensor
    uint64_t pitch;
    uint32_t F, d, nitems, nblocks;
    uint32_t E;  // experts (1 for a dense FFN)
    int act;
    const uint8_t *xq;  // qact rows of the tokens
    uint64_t xq_pitch;
    uint32_t ntok, k;
    const uint32_t *ids;
    int direct;
    MoePlan p;
    float *hf;        // f32 h rows [pos][F]
    uint32_t *hcnt;   // [pos][F/32] zero-initialised block counters
    uint8_t *hq;      // qact rows of h, one per (token, slot) position
    uint64_t hq_pitch;
    int *dev_err;
};

__host__ __device__ inline size_t gu_smem_bytes(uint64_t pitch, int nt, int ipr) {
    return 64 + 64 + align16((size_t)kGuWarps * 2 * kGuRowsPerWarp * pitch + 256) + align16(xs_bytes(nt, ipr)) +
           align16((size_t)kGuWarps * nt * 2 * kGuRowsPerWarp * ipr * 4) + align16((size_t)nt * kGuRows * 4) + 64;
}

template <uint32_t TYPE, int NT>
__global__ void __launch_bounds__(kGuWarps * 32) k_moe_gate_up(GateUpArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ipr = (int)a.nitems;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    const uint8_t **src = reinterpret_cast<const uint8_t **>(smem + 64);
    uint8_t *tile = smem + 128;
    const size_t wtile = (size_t)2 * kGuRowsPerWarp * a.pitch;
    uint8_t *p = tile + align16((size_t)kGuWarps * wtile + 256);
    const XS X = xs_carve(p, NT, ipr);
    p += align16(xs_bytes(NT, ipr));
    float *part = reinterpret_cast<float *>(p);
    p += align16((size_t)kGuWarps * NT * 2 * kGuRowsPerWarp * ipr * 4);
    float *hbuf = reinterpret_cast<float *>(p);
    p += align16((size_t)NT * kGuRows * 4);
    int *s_fin = reinterpret_cast<int *>(p);

    pdl_wait();
    // Release the down kernel only now: it reads the router's ids before its
    // own wait, which is safe once this grid has seen the router complete.
    pdl_launch_dependents();
    uint32_t e, off, cnt;
    if (a.direct) {
        if (blockIdx.y >= a.k) return;
        e = a.ids[blockIdx.y];
        if (e >= a.E) {  // an invalid caller id: expert 0's rows stand in, the error word says so
            if (threadIdx.x == 0 && a.dev_err) atomicExch(a.dev_err, DEV_ERR_BAD_INDEX);
            e = 0;
        }
        off = blockIdx.y;
        cnt = 1;
    } else {
        if (blockIdx.y >= *a.p.n_active) return;
        e = a.p.act_e[blockIdx.y];
        off = a.p.act_off[blockIdx.y];
        cnt = a.p.act_cnt[blockIdx.y];
    }
    const uint32_t r0 = blockIdx.x * kGuRows;  // F % 32 == 0, so the tile is whole
    const uint32_t wr0 = r0 + warp * kGuRowsPerWarp;
    uint8_t *wt = tile + warp * wtile;
    if (lane == 0) {
        mbar_init(&bars[warp], 1);
        fence_barrier_init();
        const uint32_t bytes = (uint32_t)(kGuRowsPerWarp * a.pitch);
        uint64_t grow, urow;
        const uint8_t *ub;
        if (a.up) {
            grow = (uint64_t)e * a.F + wr0;
            urow = grow;
            ub = a.up;
        } else {  // fused: gate rows [0,F), up rows [F,2F) (gemma4/forward.zig:469-471)
            grow = (uint64_t)e * 2 * a.F + wr0;
            urow = grow + a.F;
            ub = a.gate;
        }
        mbar_arrive_expect_tx(&bars[warp], 2 * bytes);
        tma_load_1d(wt, a.gate + grow * a.pitch, bytes, &bars[warp]);
        tma_load_1d(wt + bytes, ub + urow * a.pitch, bytes, &bars[warp]);
    }
    bool ok = true;
    const int nitem = 2 * kGuRowsPerWarp * ipr;  // per warp: 2 gate rows then 2 up rows
    float *wpart = part + (size_t)warp * NT * nitem;
    const uint32_t nblkF = a.F / 32, blk = r0 / 32;
    for (uint32_t c0 = 0; c0 < cnt; c0 += NT) {
        const int nt = (int)min((uint32_t)NT, cnt - c0);
        if (threadIdx.x < (unsigned)nt) {
            const uint32_t pos = off + c0 + threadIdx.x;
            const uint32_t pair = a.direct ? pos : a.p.pos_pair[pos];
            src[threadIdx.x] = a.xq + (size_t)(pair / a.k) * a.xq_pitch;
        }
        __syncthreads();
        qact_to_smem(X, src, nt, (int)a.d);
        __syncthreads();
        if (c0 == 0) ok = tile_wait(&bars[warp], a.dev_err);
        if (ok) {
            for (int f = lane; f < nitem; f += 32) {
                const int item = f % ipr, rowm = f / ipr;
                float res[NT];
#pragma unroll
                for (int t = 0; t < NT; t++) res[t] = 0.0f;
                dot_item<TYPE, NT>(wt + (size_t)rowm * a.pitch, item, (int)a.nblocks, X, 0, nt, res);
#pragma unroll
                for (int t = 0; t < NT; t++)
                    if (t < nt) wpart[t * nitem + f] = res[t];
            }
            __syncwarp();
            if (lane < kGuRowsPerWarp * nt) {
                const int t = lane / kGuRowsPerWarp, r = lane % kGuRowsPerWarp;
                const float *pg = wpart + t * nitem + r * ipr;
                const float *pu = pg + kGuRowsPerWarp * ipr;
                float g = 0.0f, u = 0.0f;
                for (int i = 0; i < ipr; i++) {
                    g += pg[i];
                    u += pu[i];
                }
                hbuf[t * kGuRows + warp * kGuRowsPerWarp + r] = act_apply(a.act, g) * u;
            }
        }
        __syncthreads();
        if (threadIdx.x < (unsigned)(nt * kGuRows)) {
            const int t = threadIdx.x / kGuRows, i = threadIdx.x % kGuRows;
            a.hf[(size_t)(off + c0 + t) * a.F + r0 + i] = hbuf[t * kGuRows + i];
            __threadfence();
        }
        __syncthreads();
        if (threadIdx.x < (unsigned)nt) {
            const uint32_t old = atomicAdd(&a.hcnt[(size_t)(off + c0 + threadIdx.x) * nblkF + blk], 1u);
            s_fin[threadIdx.x] = old == kGuCtasPerBlock - 1;
        }
        __syncthreads();
        if (warp < nt && s_fin[warp]) {  // last CTA of this 32-element block: quantise it
            __threadfence();
            const uint32_t pos = off + c0 + warp;
            const float v = __ldcg(a.hf + (size_t)pos * a.F + 32 * blk + lane);
            qact_store_block(a.hq + (size_t)pos * a.hq_pitch, (int)a.F, (int)blk, v, lane);
            if (lane == 0) a.hcnt[(size_t)pos * nblkF + blk] = 0;
        }
        __syncthreads();
    }
}

template <uint32_t TYPE, int NT>
static cudaError_t launch_gate_up_t(const LaunchCfg &c, const GateUpArgs &a, uint32_t ny) {
    const size_t smem = gu_smem_bytes(a.pitch, NT, (int)a.nitems);
    const dim3 grid(a.F / kGuRows, ny);
    return launch_k(c, type_label<TYPE>("moe_gate_up"), k_moe_gate_up<TYPE, NT>, grid, dim3(kGuWarps * 32), smem, a);
}

cudaError_t launch_moe_gate_up(const LaunchCfg &c, const DevMat &gate, const DevMat &up, int act, const uint8_t *xq,
                               uint64_t xq_pitch, uint32_t ntok, uint32_t k, const uint32_t *ids, bool direct,
                               const MoePlan &p, float *hf, uint32_t *hcnt, uint8_t *hq, uint64_t hq_pitch) {
    GateUpArgs a;
    const bool fused = up.data == nullptr;
    a.gate = gate.data;
    a.up = up.data;
    a.pitch = gate.pitch;
    a.F = (uint32_t)(fused ? gate.rows / 2 : gate.rows);
    a.d = (uint32_t)gate.cols;
    a.E = gate.n_experts ? gate.n_experts : 1;
    a.nitems = items_per_row(gate.type, gate.cols);
    a.nblocks = (uint32_t)(gate.cols / 32);
    a.act = act;
    a.xq = xq;
    a.xq_pitch = xq_pitch;
    a.ntok = ntok;
    a.k = k;
    a.ids = ids;
    a.direct = direct ? 1 : 0;
    a.p = p;
    a.hf = hf;
    a.hcnt = hcnt;
    a.hq = hq;
    a.hq_pitch = hq_pitch;
    a.dev_err = c.dev_err;
    const uint32_t E = gate.n_experts ? gate.n_experts : 1;
    const uint32_t ny = direct ? k : min(E, ntok * k);
    if (direct) {
        switch (gate.type) {
        case T_Q4_K: return launch_gate_up_t<T_Q4_K, 1>(c, a, ny);
        case T_Q6_K: return launch_gate_up_t<T_Q6_K, 1>(c, a, ny);
        case T_Q8_0: return launch_gate_up_t<T_Q8_0, 1>(c, a, ny);
        case T_Q5_0: return launch_gate_up_t<T_Q5_0, 1>(c, a, ny);
        case T_Q5_1: return launch_gate_up_t<T_Q5_1, 1>(c, a, ny);
        case T_IQ4_NL: return launch_gate_up_t<T_IQ4_NL, 1>(c, a, ny);
        case T_Q5_K: return launch_gate_up_t<T_Q5_K, 1>(c, a, ny);
        case T_Q3_K: return launch_gate_up_t<T_Q3_K, 1>(c, a, ny);
        default: return cudaErrorInvalidValue;
        }
    }
    switch (gate.type) {
    case T_Q4_K: return launch_gate_up_t<T_Q4_K, 4>(c, a, ny);
    case T_Q6_K: return launch_gate_up_t<T_Q6_K, 2>(c, a, ny);
    case T_Q8_0: return launch_gate_up_t<T_Q8_0, 4>(c, a, ny);
    case T_Q5_0: return launch_gate_up_t<T_Q5_0, 4>(c, a, ny);
    case T_Q5_1: return launch_gate_up_t<T_Q5_1, 4>(c, a, ny);
    case T_IQ4_NL: return launch_gate_up_t<T_IQ4_NL, 4>(c, a, ny);
    case T_Q5_K: return launch_gate_up_t<T_Q5_K, 4>(c, a, ny);
    case T_Q3_K: return launch_gate_up_t<T_Q3_K, 2>(c, a, ny);
    default: return cudaErrorInvalidValue;
    }
}

// ── down projection + weighted combine (+ residual) ──────────────────────────

constexpr int kDnWarps = 8;
constexpr int kMaxK = 16;

struct DownArgs {
    const uint8_t *down;
    uint64_t pitch;
    uint32_t D, F, nitems, nblocks;  // down: [E][D rows][F cols]
    uint32_t E;
    const uint8_t *hq;
    uint64_t hq_pitch;
    uint32_t ntok, k;
    const uint32_t *ids;
    const float *w;
    int direct;
    MoePlan p;
    const float *resid;  // nullable: out = resid + sum_s w_s * y_s
    float *out;
    uint32_t rt;  // rows per CTA (rt * nitems <= 32: one item per lane)
    int *dev_err;
};

__host__ __device__ inline size_t dn_smem_bytes(uint64_t pitch, uint32_t rt, int k, int ipr) {
    return 128 + 128 + align16((size_t)k * rt * pitch + 256) + align16(xs_bytes(k, ipr)) + (size_t)k * rt * ipr * 4;
}

template <uint32_t TYPE>
__global__ void __launch_bounds__(kDnWarps * 32) k_moe_down(DownArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    // Launched early (programmatic dependent launch) while the gate/up kernel
    // runs.  That kernel released its dependents only after its own wait, so
    // the router (and the dispatch plan) have completed: the expert ids are
    // final and this CTA's down-projection rows can stream in now.  h and the
    // residual are read only after pdl_wait().
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ipr = (int)a.nitems;
    const int k = (int)a.k;
    const uint32_t t = blockIdx.y;
    const uint32_t r0 = blockIdx.x * a.rt;
    const uint32_t nr = min(a.rt, a.D - r0);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    const uint8_t **src = reinterpret_cast<const uint8_t **>(smem + 128);
    uint8_t *tile = smem + 256;
    uint8_t *p = tile + align16((size_t)k * a.rt * a.pitch + 256);
    const XS X = xs_carve(p, k, ipr);
    p += align16(xs_bytes(k, ipr));
    float *part = reinterpret_cast<float *>(p);

    for (int s = warp; s < k; s += kDnWarps) {
        if (lane == 0) {
            mbar_init(&bars[s], 1);
            fence_barrier_init();
            const uint32_t bytes = (uint32_t)(nr * a.pitch);
            uint32_t e = __ldcg(a.ids + t * a.k + s);
            if (e >= a.E) e = 0;  // an invalid caller id (recorded by the plan or gate/up): weight ignored below
            mbar_arrive_expect_tx(&bars[s], bytes);
            tma_load_1d(tile + (size_t)s * a.rt * a.pitch, a.down + ((uint64_t)e * a.D + r0) * a.pitch, bytes,
                        &bars[s]);
        }
    }
    if (threadIdx.x < (unsigned)k) {
        const uint32_t pair = t * a.k + threadIdx.x;
        uint32_t pos = a.direct ? pair : __ldcg(a.p.pair_pos + pair);
        if (pos == kNoPos) pos = 0;  // skipped in the combine below
        src[threadIdx.x] = a.hq + (size_t)pos * a.hq_pitch;
    }
    pdl_wait();
    __syncthreads();
    qact_to_smem(X, src, k, (int)a.F);
    __syncthreads();
    const int nitem = (int)nr * ipr;
    for (int s = warp; s < k; s += kDnWarps) {
        if (!tile_wait(&bars[s], a.dev_err)) continue;
        for (int f = lane; f < nitem; f += 32) {
            const int item = f % ipr, row = f / ipr;
            float res[1] = {0.0f};
            dot_item<TYPE, 1>(tile + ((size_t)s * a.rt + row) * a.pitch, item, (int)a.nblocks, X, s, 1, res);
            part[(s * (int)a.rt + row) * ipr + item] = res[0];
        }
    }
    __syncthreads();
    for (int r = threadIdx.x; r < (int)nr; r += blockDim.x) {
        float o = 0.0f;  // moe_buf is zeroed, then += scale * down, slot by slot
        for (int s = 0; s < k; s++) {
            if (__ldcg(a.ids + t * a.k + s) >= a.E) continue;  // an invalid id contributes nothing
            const float *pp = part + (s * (int)a.rt + r) * ipr;
            float y = 0.0f;
            for (int i = 0; i < ipr; i++) y += pp[i];
            o += a.w[t * a.k + s] * y;
        }
        const size_t oi = (size_t)t * a.D + r0 + r;
        a.out[oi] = a.resid ? a.resid[oi] + o : o;
    }
}

cudaError_t launch_moe_down(const LaunchCfg &c, const DevMat &down, const uint8_t *hq, uint64_t hq_pitch,
                            uint32_t ntok, uint32_t k, const uint32_t *ids, const float *w, bool direct,
                            const MoePlan &p, const float *resid, float *out) {
    DownArgs a;
    a.down = down.data;
    a.pitch = down.pitch;
    a.D = (uint32_t)down.rows;
    a.F = (uint32_t)down.cols;
    a.E = down.n_experts ? down.n_experts : 1;
    a.nitems = items_per_row(down.type, down.cols);
    a.nblocks = (uint32_t)(down.cols / 32);
    a.hq = hq;
    a.hq_pitch = hq_pitch;
    a.ntok = ntok;
    a.k = k;
    a.ids = ids;
    a.w = w;
    a.direct = direct ? 1 : 0;
    a.p = p;
    a.resid = resid;
    a.out = out;
    a.rt = max(1u, 32u / a.nitems);
    a.dev_err = c.dev_err;
    const size_t smem = dn_smem_bytes(a.pitch, a.rt, (int)k, (int)a.nitems);
    const dim3 grid((a.D + a.rt - 1) / a.rt, ntok);
#define LT_DOWN_CASE(T) \
    case T: return launch_k(c, type_label<T>("moe_down"), k_moe_down<T>, grid, dim3(kDnWarps * 32), smem, a);
    switch (down.type) {
        LT_DOWN_CASE(T_Q4_K)
        LT_DOWN_CASE(T_Q6_K)
        LT_DOWN_CASE(T_Q8_0)
        LT_DOWN_CASE(T_Q5_0)
        LT_DOWN_CASE(T_Q5_1)
        LT_DOWN_CASE(T_IQ4_NL)
        LT_DOWN_CASE(T_Q5_K)
        LT_DOWN_CASE(T_Q3_K)
    default: return cudaErrorInvalidValue;
    }
#undef LT_DOWN_CASE
}

}  // namespace lt
