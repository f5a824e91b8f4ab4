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
//            cache; each split publishes (max, sum, weighted values), and the
//            last split of a head to finish (a per-head counter) merges the
//            head's splits and quantises the head into the attention row.
//                                                      -> grid barrier
//   phase O  every CTA copies the quantised attention row and computes its
//            wo rows plus the residual: out = x + wo . att (forward.zig:304-305).
//
// The weights are static, so both tiles (this CTA's Q/K/V rows and wo rows)
// stream in while the previous kernel finishes; an optional L2 prefetch
// range (the next kernel's weights) is issued once the Q/K/V rows are done.
#include "lt_attn_common.cuh"

namespace lt {

// Layout of the context's attention sync block.
constexpr size_t kAbEpoch = 0, kAbHeadCnt = 256;
// the three hand-offs' split counters (kGridSplitBytes each) after the head counters
constexpr size_t kAbB1 = 256 + 4 * 1024, kAbB2 = kAbB1 + kGridSplitBytes, kAbB3 = kAbB2 + kGridSplitBytes;
static_assert(kAbB3 + kGridSplitBytes <= kAttnSyncBytes, "attention sync block");
constexpr uint32_t kAbMaxSplits = 8;  // splits of a head's positions (one CTA each)
constexpr uint32_t kAbSplitPositions = 256;  // positions per split before another CTA joins

struct AttnBlockArgs {
    AttnGeom g;
    uint32_t d;
    const float *x, *norm_w;
    float eps;
    // the Q/K/V rows: qrows = nq + nkv (+ nkv) rows in segments, rows
    // [seg_end[s-1], seg_end[s]) from seg_w[s] (one segment for a stacked tensor)
    const uint8_t *seg_w[3];
    uint64_t seg_pitch[3];
    uint32_t seg_type[3], seg_end[3], nseg;
    uint32_t qrows, qnb;  // rows, 32-blocks per row (d / 32)
    uint32_t v_is_k;      // no V rows: V is the raw K head (gemma4/forward.zig:250)
    const float *bias;    // nullable [qrows]
    const float *q_norm, *k_norm;
    const uint32_t *pos;
    void *kc, *vc;  // f32 or f16 elements (g.kv_f16)
    const uint8_t *wo;
    uint64_t opitch;
    uint32_t onb, otype;  // 32-blocks per wo row (nq / 32), type
    const float *post_norm;  // nullable: out = x + rmsnorm(wo . att) * post_norm (gemma4/forward.zig:329-333)
    // nullable tail_f: the previous layer's FFN tail applied to x first (gemma4/forward.zig:520-532)
    const float *tail_f, *tail_w1, *tail_m, *tail_w2, *tail_w;
    float tail_los, tail_eps;
    float *ss_part;          // [grid] partial sums of squares for post_norm
    uint32_t late_wo;        // the wo tile lands in the Q/K/V tile's space once phase Q is done
    float *out;
    float *qkv, *part;  // global scratch
    uint8_t *att;       // the attention vector as a quantised activation row (qact layout)
    uint8_t *sync;
    const uint8_t *pf[2];
    uint64_t pf_bytes[2];
    int *dev_err;
    uint32_t splits, qtile, maxo;  // qtile: bytes of the largest CTA's Q/K/V rows
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
    // + slack: a Q8_0 chunk reads up to 34 bytes past a row
    const size_t qb = (size_t)a.qtile + 128, ob = (size_t)a.maxo * a.opitch + 128;
    // the head vectors live only in phase A, when the Q/K/V rows are consumed:
    // they take the Q/K/V tile's space (after the wo rows, when those follow there)
    const size_t hb = (size_t)(3 * a.g.hd + kAbWarps * (a.g.hd + 2) + kAbWarps + 2) * 4;
    const size_t ob128 = (ob + 127) & ~(size_t)127;
    size_t head_in = SIZE_MAX;
    if (a.late_wo) {
        L.wq = take(qb > ob ? qb : ob);
        L.wo = L.wq;
        if (qb >= ob128 + hb) head_in = L.wq + ob128;
    } else {
        L.wq = take(qb);
        L.wo = take(ob);
        if (qb >= hb) head_in = L.wq;
    }
    L.xs = take(xs_bytes(1, (int)((a.d + 255) / 256)));
    L.as = take(xs_bytes(1, (int)((nq + 255) / 256)));
    L.xf = take((size_t)(a.d > nq ? a.d : nq) * 4);
    L.nw = take((size_t)a.d * 4);
    L.xres = take((size_t)a.maxo * 4);
    // per-item head vectors q, k, v and the warps' softmax partials
    L.head = head_in != SIZE_MAX ? head_in : take(hb);
    L.total = off;
    return L;
}


// The FFN tail's values per thread: elements i = tid + k * kAbThreads (d <= 8192).
constexpr int kAbTailPer = 16;
struct AbTailW {
    float w1[kAbTailPer], w2[kAbTailPer], w[kAbTailPer];
};

// The tail's norm weights, into registers before the kernel waits on its producer (they are static).
LT_DEVINL void ab_tail_weights(const AttnBlockArgs &a, AbTailW &t) {
#pragma unroll
    for (int k = 0; k < kAbTailPer; k++) {
        const uint32_t i = threadIdx.x + k * kAbThreads;
        const bool in = i < a.d;
        t.w1[k] = in && a.tail_w1 ? __ldg(a.tail_w1 + i) : 0.0f;
        t.w2[k] = in ? __ldg(a.tail_w2 + i) : 0.0f;
        t.w[k] = in ? __ldg(a.tail_w + i) : 0.0f;
    }
}

// xf = (xf + rmsnorm(f' + rmsnorm(m) * w2) * w) * los, f' = rmsnorm(f) * w1 or f:
// k_ffn_tail's arithmetic and sum orders (512 threads, strided, then warps in
// order), so the fused and separate paths give the same bits.  One global
// round trip (f and m); the weights are already in registers.
LT_DEVINL void ab_tail(const AttnBlockArgs &a, const AbTailW &t, float *xf, float *red) {
    const uint32_t n = a.d, tid = threadIdx.x;
    float fv[kAbTailPer], hv[kAbTailPer];
    float sf = 0.0f, sm = 0.0f;
#pragma unroll
    for (int k = 0; k < kAbTailPer; k++) {
        const uint32_t i = tid + k * kAbThreads;
        fv[k] = i < n ? __ldcg(a.tail_f + i) : 0.0f;
        hv[k] = i < n ? __ldcg(a.tail_m + i) : 0.0f;
        if (i < n) {
            sf = __fadd_rn(sf, __fmul_rn(fv[k], fv[k]));
            sm = __fadd_rn(sm, __fmul_rn(hv[k], hv[k]));
        }
    }
    sf = ab_block_sum(sf, red);
    sm = ab_block_sum(sm, red);
    const float rf1 = a.tail_w1 ? ab_rinv(sf, n, a.tail_eps) : 1.0f, rm = ab_rinv(sm, n, a.tail_eps);
    float sh = 0.0f;
#pragma unroll
    for (int k = 0; k < kAbTailPer; k++) {
        const uint32_t i = tid + k * kAbThreads;
        if (i < n) {
            const float fi = a.tail_w1 ? __fmul_rn(__fmul_rn(fv[k], rf1), t.w1[k]) : fv[k];
            hv[k] = __fadd_rn(fi, __fmul_rn(__fmul_rn(hv[k], rm), t.w2[k]));
            sh = __fadd_rn(sh, __fmul_rn(hv[k], hv[k]));
        }
    }
    const float rf = ab_rinv(ab_block_sum(sh, red), n, a.tail_eps);
#pragma unroll
    for (int k = 0; k < kAbTailPer; k++) {
        const uint32_t i = tid + k * kAbThreads;
        if (i < n) {
            float v = __fadd_rn(xf[i], __fmul_rn(__fmul_rn(hv[k], rf), t.w[k]));
            if (a.tail_los != 1.0f) v = __fmul_rn(v, a.tail_los);
            xf[i] = v;
        }
    }
    __syncthreads();
}

// Phase timestamps for tuning builds (-DLT_DECODE_TRACE): thread 0 of each
// CTA records globaltimer at the phase boundaries of the latest launch.  Off
// in the library the package builds.
#ifdef LT_DECODE_TRACE
constexpr int kAtCtas = 160, kAtMarks = 24;
__device__ unsigned long long g_ab_trace[kAtCtas * kAtMarks];
#define AT_MARK(m)                                                                     \
    do {                                                                               \
        if (tid == 0 && c < kAtCtas) g_ab_trace[c * kAtMarks + (m)] = globaltimer_ns(); \
    } while (0)
extern "C" int lt_ab_trace_copy(void *dst, size_t bytes) { return (int)cudaMemcpyFromSymbol(dst, g_ab_trace, bytes); }
#else
#define AT_MARK(m) \
    do {           \
    } while (0)
#endif

// GEN: segments, V = K, the post-attention norm or the late wo tile may occur
// (otherwise: one stacked Q/K/V tensor, plain residual, both tiles at once).
template <uint32_t QT, uint32_t OT, int HD, bool GEN>
__global__ void __launch_bounds__(kAbThreads, 1) k_attn_block(AttnBlockArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int PER = HD / 32;
    constexpr int NB = HD <= 128 ? 4 : 2;  // positions a warp loads before using them
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t G = gridDim.x, c = blockIdx.x;
    const AbLayout L = ab_layout(a);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    float *red = reinterpret_cast<float *>(smem + L.misc);            // [16]
    uint64_t *s_epoch = reinterpret_cast<uint64_t *>(smem + L.misc + 64);
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
    unsigned long long *ctr3 = reinterpret_cast<unsigned long long *>(a.sync + kAbB3);
    uint32_t *head_cnt = reinterpret_cast<uint32_t *>(a.sync + kAbHeadCnt);
    int *s_last = reinterpret_cast<int *>(smem + L.misc + 128);

    const uint32_t q0 = (uint32_t)((uint64_t)c * a.qrows / G), q1 = (uint32_t)((uint64_t)(c + 1) * a.qrows / G);
    const uint32_t o0 = (uint32_t)((uint64_t)c * a.d / G), o1 = (uint32_t)((uint64_t)(c + 1) * a.d / G);
    const uint32_t nqr = q1 - q0, nor = o1 - o0;
    AT_MARK(0);

    // static inputs first: both weight tiles, the norm weights, the L2 prefetch
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_init(&bars[2], 1);  // the norm weights
        fence_barrier_init();
        if (nqr && !GEN) {
            mbar_arrive_expect_tx(&bars[0], (uint32_t)(nqr * a.seg_pitch[0]));
            tma_load_1d(wq, a.seg_w[0] + (uint64_t)q0 * a.seg_pitch[0], (uint32_t)(nqr * a.seg_pitch[0]), &bars[0]);
        } else if (nqr) {  // this CTA's rows of each segment, one after another
            uint32_t total = 0;
            for (uint32_t sg = 0; sg < a.nseg; sg++) {
                const uint32_t sb = sg ? a.seg_end[sg - 1] : 0, lo = max(q0, sb), hi = min(q1, a.seg_end[sg]);
                if (lo < hi) total += (uint32_t)((hi - lo) * a.seg_pitch[sg]);
            }
            mbar_arrive_expect_tx(&bars[0], total);
            uint32_t off = 0;
            for (uint32_t sg = 0; sg < a.nseg; sg++) {
                const uint32_t sb = sg ? a.seg_end[sg - 1] : 0, lo = max(q0, sb), hi = min(q1, a.seg_end[sg]);
                if (lo < hi) {
                    const uint32_t bytes = (uint32_t)((hi - lo) * a.seg_pitch[sg]);
                    tma_load_1d(wq + off, a.seg_w[sg] + (uint64_t)(lo - sb) * a.seg_pitch[sg], bytes, &bars[0]);
                    off += bytes;
                }
            }
        }
        if (nor && (!GEN || !a.late_wo)) {
            mbar_arrive_expect_tx(&bars[1], (uint32_t)(nor * a.opitch));
            tma_load_1d(wo, a.wo + (uint64_t)o0 * a.opitch, (uint32_t)(nor * a.opitch), &bars[1]);
        }
    }
    AbTailW tw;
    if (GEN && a.tail_f) ab_tail_weights(a, tw);
    // the third hand-off (post-norm only) counts every launch: without it, CTA 0
    // adds the whole grid's arrivals at once, off the critical path
    if (!a.post_norm && c == 0 && tid == 0) grid_arrive_split_all(ctr3, G);
    // the norm weights by TMA as well: a load loop here would hold every thread
    // until its loads return before it reaches the wait for the producer
    const bool nw_tma = (reinterpret_cast<uintptr_t>(a.norm_w) & 15) == 0;
    if (nw_tma && tid == 0) {
        mbar_arrive_expect_tx(&bars[2], a.d * 4);
        tma_load_1d(nw, a.norm_w, a.d * 4, &bars[2]);
    } else if (!nw_tma) {
        for (uint32_t i = tid; i < a.d; i += kAbThreads) nw[i] = __ldg(a.norm_w + i);
    }
    pdl_launch_dependents();
    pdl_wait();
    AT_MARK(1);

    // ── phase Q ──────────────────────────────────────────────────────────────
    if (tid == 0) *s_epoch = grid_epoch(ctr_epoch, G);
    const uint32_t pos = *a.pos;
    ab_load(xf, a.x, a.d);
    __syncthreads();
    AT_MARK(2);
    if (GEN && a.tail_f) ab_tail(a, tw, xf, red);  // the block's input is the previous layer's output
    for (uint32_t r = tid; r < nor; r += kAbThreads) xres[r] = xf[o0 + r];
    {
        float ss = 0.0f;
        for (uint32_t i = tid; i < a.d; i += kAbThreads) ss += xf[i] * xf[i];
        ss = ab_block_sum(ss, red);
        const float rms_inv = 1.0f / sqrtf(ss / (float)a.d + a.eps);
        if (nw_tma) tile_wait(&bars[2], a.dev_err);
        ab_quantise_norm(Xx, xf, a.d, rms_inv, nw, warp, lane);  // the rows need only the quantised x
    }
    __syncthreads();
    AT_MARK(3);
    const uint64_t epoch = *s_epoch;
    float *yq = xf;  // the normalised x is quantised already
    if constexpr (!GEN) {
        if (nqr && tile_wait(&bars[0], a.dev_err)) ab_rows_fit<QT>(wq, a.seg_pitch[0], nqr, a.d, a.qnb, Xx, warp, lane, yq);
    } else if (nqr && tile_wait(&bars[0], a.dev_err)) {
        uint32_t off = 0;
        for (uint32_t sg = 0; sg < a.nseg; sg++) {
            const uint32_t sb = sg ? a.seg_end[sg - 1] : 0, lo = max(q0, sb), hi = min(q1, a.seg_end[sg]);
            if (lo < hi) {
                ab_rows_any<QT>(a.seg_type[sg], wq + off, a.seg_pitch[sg], hi - lo, a.d, a.qnb, Xx, warp, lane,
                                yq + (lo - q0));
                off += (uint32_t)((hi - lo) * a.seg_pitch[sg]);
            }
        }
    }
    __syncthreads();
    AT_MARK(4);
    // the L2 prefetch of the next kernel's weights, once this CTA's weight
    // tiles have landed (issued at the start, it queued behind them in the
    // copy engine and held threads 0 and 1 back from the wait for the producer)
    if (tid < 2 && a.pf[tid]) prefetch_l2_share(a.pf[tid], a.pf_bytes[tid], c, G);
    for (uint32_t r = tid; r < nqr; r += kAbThreads)
        a.qkv[q0 + r] = a.bias ? __fadd_rn(yq[r], a.bias[q0 + r]) : yq[r];
    grid_arrive_split(ctr1);
    grid_wait_split(ctr1, epoch, a.dev_err, kWaitLimitNs);
    AT_MARK(5);

    // ── phase A ──────────────────────────────────────────────────────────────
    if (GEN && a.late_wo) {  // the Q/K/V rows are consumed: the wo rows take their place
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0 && nor) {
            mbar_arrive_expect_tx(&bars[1], (uint32_t)(nor * a.opitch));
            tma_load_1d(wo, a.wo + (uint64_t)o0 * a.opitch, (uint32_t)(nor * a.opitch), &bars[1]);
        }
    }
    const uint32_t group = a.g.n_heads / a.g.n_kv;
    const uint32_t seq = pos + 1, win = a.g.window ? min(seq, a.g.window) : seq, first = seq - win;
    // splits of a head's window: one per kAbSplitPositions positions (a short
    // window is one CTA's, with no merge across CTAs), at most a.splits
    const uint32_t S = min(a.splits, max(1u, (win + kAbSplitPositions - 1) / kAbSplitPositions));
    for (uint32_t item = c; item < a.g.n_heads * S; item += G) {
        const uint32_t h = item / S, s = item - h * S, kh = h / group;
        if (tid < 3 * HD / 4) {  // q, k, v heads: one float4 each
            const uint32_t part = tid / (HD / 4), i = tid % (HD / 4);
            const size_t off = part == 0   ? (size_t)h * HD
                               : part == 1 ? nq + (size_t)kh * HD
                                           : (GEN && a.v_is_k ? nq : nq + nkv) + (size_t)kh * HD;
            reinterpret_cast<float4 *>(hq + part * HD)[i] = __ldcg(reinterpret_cast<const float4 *>(a.qkv + off) + i);
        }
        __syncthreads();
        AT_MARK(6);
        if (a.g.v_norm) {  // rmsnormRaw (math.zig:43-48) of the V head
            const float vv = tid < HD ? hv[tid] : 0.0f;
            const float ss = ab_block_sum(tid < HD ? __fmul_rn(vv, vv) : 0.0f, red);
            const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), a.g.eps)));
            __syncthreads();
            if (tid < HD) hv[tid] = __fmul_rn(vv, r);
            __syncthreads();
        }
        ab_norm_rope2(hq, a.q_norm, hk, a.k_norm, a.g, pos, red);
        AT_MARK(7);
        if (s == 0 && h % group == 0) {  // this position's K/V into the cache
            const size_t slot = (size_t)(pos % a.g.cap) * nkv + (size_t)kh * HD;
            for (uint32_t i = tid; i < HD; i += kAbThreads) {
                kv_st(a.kc, slot + i, hk[i], a.g.kv_f16);
                kv_st(a.vc, slot + i, hv[i], a.g.kv_f16);
            }
        }
        if (a.g.kv_f16) {  // attend to this position as the cache holds it
            __syncthreads();
            for (uint32_t i = tid; i < HD; i += kAbThreads) {
                hk[i] = kv_round(hk[i], 1u);
                hv[i] = kv_round(hv[i], 1u);
            }
            __syncthreads();
        }
        float o[PER], m = -INFINITY, l = 0.0f;
        if (a.g.kv_f16)
            ab_attend<HD, true>(a.kc, a.vc, a.g, s, S, win, first, (size_t)kh * HD, nkv, hq, hk, hv, warp, lane, m, l, o);
        else
            ab_attend<HD, false>(a.kc, a.vc, a.g, s, S, win, first, (size_t)kh * HD, nkv, hq, hk, hv, warp, lane, m, l, o);
        AT_MARK(8);
        float *wp = wpart + warp * (HD + 2);
        if (lane == 0) {
            wp[0] = m;
            wp[1] = l;
        }
#pragma unroll
        for (int i = 0; i < PER; i++) wp[2 + lane * PER + i] = o[i];  // lane owns dims [lane*PER, +PER)
        __syncthreads();
        // the warps' partials: warp 0 finds the maximum and each warp's scale once
        float *sf = wpart + kAbWarps * (HD + 2);  // [kAbWarps] scales, then the sum
        if (warp == 0) {
            const float mw = lane < kAbWarps ? wpart[lane * (HD + 2)] : -INFINITY;
            float M = mw;
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
            if (lane < kAbWarps) sf[lane] = mw != -INFINITY ? expf(mw - M) : 0.0f;
            __syncwarp();
            if (lane == 0) {
                float Lsum = 0.0f;
                for (int w = 0; w < kAbWarps; w++) Lsum += wpart[w * (HD + 2) + 1] * sf[w];
                sf[kAbWarps] = Lsum;
                sf[kAbWarps + 1] = M;
            }
        }
        __syncthreads();
        if (S == 1) {  // the whole window: normalise, quantise into the attention row
            const float Lsum = sf[kAbWarps];
            for (uint32_t t = tid; t < HD; t += kAbThreads) {
                float acc = 0.0f;
#pragma unroll
                for (int w = 0; w < kAbWarps; w++) acc += wpart[w * (HD + 2) + 2 + t] * sf[w];
                hq[t] = acc / Lsum;  // this item's query head is no longer needed
            }
            __syncthreads();
            for (uint32_t b = warp; b < (uint32_t)HD / 32; b += kAbWarps)
                qact_store_block(a.att, (int)nq, (int)(h * HD / 32 + b), hq[32 * b + lane], lane);
            __syncthreads();
            AT_MARK(9);
            continue;
        }
        // split partials: o [h][s][HD] (16-byte aligned rows), (max, sum) [h][s]
        float *po = a.part + ((size_t)h * S + s) * HD;
        float *pml = a.part + (size_t)a.g.n_heads * S * HD + 2 * ((size_t)h * S + s);
        for (uint32_t t = tid; t < HD; t += kAbThreads) {
            float acc = 0.0f;
#pragma unroll
            for (int w = 0; w < kAbWarps; w++) acc += wpart[w * (HD + 2) + 2 + t] * sf[w];
            po[t] = acc;
        }
        if (tid == 0) *reinterpret_cast<float2 *>(pml) = make_float2(sf[kAbWarps + 1], sf[kAbWarps]);
        // the last split of head h to get here merges the head's splits and
        // quantises it (16-groups never straddle heads: HD % 32 == 0)
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            s_last[0] = atomicAdd(head_cnt + h, 1u) == S - 1;
        }
        __syncthreads();
        if (s_last[0]) {
            __threadfence();
            const float *ho = a.part + (size_t)h * S * HD;
            const float *hml = a.part + (size_t)a.g.n_heads * S * HD + 2 * (size_t)h * S;
            for (uint32_t t = tid; t < HD; t += kAbThreads) {
                float GM = -INFINITY;
                for (uint32_t k = 0; k < S; k++) GM = fmaxf(GM, __ldcg(hml + 2 * k));
                float GL = 0.0f, acc = 0.0f;
                for (uint32_t k = 0; k < S; k++) {
                    const float mk = __ldcg(hml + 2 * k);
                    if (mk != -INFINITY) {
                        const float f = expf(mk - GM);
                        GL += __ldcg(hml + 2 * k + 1) * f;
                        acc += __ldcg(ho + (size_t)k * HD + t) * f;
                    }
                }
                hq[t] = acc / GL;
            }
            __syncthreads();
            for (uint32_t b = warp; b < (uint32_t)HD / 32; b += kAbWarps)
                qact_store_block(a.att, (int)nq, (int)(h * HD / 32 + b), hq[32 * b + lane], lane);
            if (tid == 0) head_cnt[h] = 0;
        }
        __syncthreads();
    }
    AT_MARK(10);
    grid_arrive_split(ctr2);
    grid_wait_split(ctr2, epoch, a.dev_err, kWaitLimitNs);
    AT_MARK(11);

    // ── phase O ──────────────────────────────────────────────────────────────
    ab_load_qact(Xa, a.att, nq);
    __syncthreads();
    AT_MARK(12);
    float *yo = xf;  // the attention vector is quantised already
    if (nor && tile_wait(&bars[1], a.dev_err)) ab_rows_any<OT>(a.otype, wo, a.opitch, nor, nq, a.onb, Xa, warp, lane, yo);
    __syncthreads();
    AT_MARK(13);
    if (GEN && a.post_norm) {  // x + rmsnorm(y) * w over all d outputs: partial sums, a third hand-off
        float ss = 0.0f;
        for (uint32_t r = tid; r < nor; r += kAbThreads) ss = __fadd_rn(ss, __fmul_rn(yo[r], yo[r]));
        ss = ab_block_sum(ss, red);
        if (tid == 0) a.ss_part[c] = ss;
        grid_arrive_split(ctr3);
        grid_wait_split(ctr3, epoch, a.dev_err, kWaitLimitNs);
        float t = 0.0f;
        for (uint32_t i = tid; i < G; i += kAbThreads) t = __fadd_rn(t, __ldcg(a.ss_part + i));
        t = ab_block_sum(t, red);
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)a.d), a.eps)));
        for (uint32_t i = tid; i < nor; i += kAbThreads)
            a.out[o0 + i] = __fadd_rn(xres[i], __fmul_rn(__fmul_rn(yo[i], r), __ldg(a.post_norm + o0 + i)));
    } else {
        for (uint32_t r = tid; r < nor; r += kAbThreads) a.out[o0 + r] = __fadd_rn(xres[r], yo[r]);
    }
    AT_MARK(14);
}

static bool ab_type_ok(uint32_t t) { return t == T_Q8_0 || t == T_Q4_K || t == T_Q6_K; }

// Arguments without the pointers that vary per call; false if the shape is outside the kernel.
static bool ab_args(const AttnBlockParams &p, int num_sms, AttnBlockArgs &a) {
    const AttnGeom &g = p.g;
    a = AttnBlockArgs{};
    if (g.hd != 64 && g.hd != 128 && g.hd != 256) return false;
    if (p.nseg < 1 || p.nseg > 3 || p.d % 32 != 0 || p.d > 8192) return false;
    const uint32_t nq = g.n_heads * g.hd, nkv = g.n_kv * g.hd;
    const uint32_t want = nq + nkv + (p.v_is_k ? 0u : nkv);
    uint32_t rows = 0;
    for (uint32_t s = 0; s < p.nseg; s++) {
        const DevMat &m = p.seg[s];
        if (!ab_type_ok(m.type) || m.cols != p.d || m.n_experts) return false;
        rows += (uint32_t)m.rows;
        a.seg_w[s] = m.data;
        a.seg_pitch[s] = m.pitch;
        a.seg_type[s] = m.type;
        a.seg_end[s] = rows;
    }
    if (rows != want) return false;
    if (!ab_type_ok(p.wo.type) || p.wo.rows != p.d || p.wo.cols != nq || nq > 16384) return false;
    a.g = g;
    a.d = p.d;
    a.nseg = p.nseg;
    a.v_is_k = p.v_is_k ? 1u : 0u;
    a.qrows = rows;
    a.qnb = p.d / 32;
    a.opitch = p.wo.pitch;
    a.onb = (uint32_t)(p.wo.cols / 32);
    a.otype = p.wo.type;
    const uint32_t G = (uint32_t)num_sms;
    a.splits = max(1u, min(kAbMaxSplits, G / g.n_heads));
    a.qtile = 0;
    for (uint32_t c = 0; c < G; c++) {  // the kernel's split of the rows over the CTAs
        const uint32_t q0 = (uint32_t)((uint64_t)c * a.qrows / G), q1 = (uint32_t)((uint64_t)(c + 1) * a.qrows / G);
        uint64_t bytes = 0;
        for (uint32_t sg = 0; sg < a.nseg; sg++) {
            const uint32_t sb = sg ? a.seg_end[sg - 1] : 0, lo = max(q0, sb), hi = min(q1, a.seg_end[sg]);
            if (lo < hi) bytes += (uint64_t)(hi - lo) * a.seg_pitch[sg];
        }
        if (bytes > a.qtile) a.qtile = (uint32_t)bytes;
    }
    a.maxo = (p.d + G - 1) / G;
    a.late_wo = 0;
    if (ab_layout(a).total > kDecodeSmemLimit) {  // the wo rows wait for the Q/K/V rows' space
        a.late_wo = 1;
        if (ab_layout(a).total > kDecodeSmemLimit) return false;
    }
    return true;
}

static size_t ab_scratch_floats(const AttnBlockArgs &a, int num_sms) {
    return (size_t)((a.qrows + 31) & ~31u) + (((size_t)a.g.n_heads * a.splits * (a.g.hd + 2) + 31) & ~(size_t)31) +
           ((qact_pitch((uint64_t)a.g.n_heads * a.g.hd) / 4 + 31) & ~(size_t)31) + (size_t)num_sms + 64;
}

bool attn_block_plan(const AttnBlockParams &p, int num_sms, size_t *scratch_floats) {
    AttnBlockArgs a;
    if (!ab_args(p, num_sms, a)) return false;
    if (scratch_floats) *scratch_floats = ab_scratch_floats(a, num_sms);
    return true;
}

template <uint32_t QT, uint32_t OT, bool GEN>
static cudaError_t launch_ab_g(const LaunchCfg &c, const AttnBlockArgs &a, size_t smem) {
    switch (a.g.hd) {
    case 64:
        return launch_k(c, "attn_block", k_attn_block<QT, OT, 64, GEN>, dim3(c.num_sms), dim3(kAbThreads), smem, a);
    case 128:
        return launch_k(c, "attn_block", k_attn_block<QT, OT, 128, GEN>, dim3(c.num_sms), dim3(kAbThreads), smem, a);
    case 256:
        return launch_k(c, "attn_block", k_attn_block<QT, OT, 256, GEN>, dim3(c.num_sms), dim3(kAbThreads), smem, a);
    default: return cudaErrorInvalidValue;
    }
}

template <uint32_t QT, uint32_t OT>
static cudaError_t launch_ab_t(const LaunchCfg &c, const AttnBlockArgs &a, size_t smem) {
    if constexpr (QT == 0) {
        return launch_ab_g<QT, OT, true>(c, a, smem);
    } else {
        if (a.nseg > 1 || a.v_is_k || a.post_norm || a.late_wo || a.tail_f)
            return launch_ab_g<QT, OT, true>(c, a, smem);
        return launch_ab_g<QT, OT, false>(c, a, smem);
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
    AttnBlockArgs a;
    if (!ab_args(p, c.num_sms, a)) return cudaErrorInvalidValue;
    a.x = p.x;
    a.norm_w = p.norm_w;
    a.eps = p.eps;
    a.bias = p.bias;
    a.q_norm = p.q_norm;
    a.k_norm = p.k_norm;
    a.post_norm = p.post_norm;
    a.tail_f = p.tail_f;
    a.tail_w1 = p.tail_w1;
    a.tail_m = p.tail_m;
    a.tail_w2 = p.tail_w2;
    a.tail_w = p.tail_w;
    a.tail_los = p.tail_los;
    a.tail_eps = p.tail_eps;
    a.pos = p.pos;
    a.kc = p.kc;
    a.vc = p.vc;
    a.wo = p.wo.data;
    a.out = p.out;
    float *sc = p.scratch;
    a.qkv = sc;
    a.part = sc + ((a.qrows + 31) & ~31u);
    float *att = a.part + (((size_t)p.g.n_heads * a.splits * (p.g.hd + 2) + 31) & ~(size_t)31);
    a.att = reinterpret_cast<uint8_t *>(att);
    a.ss_part = att + ((qact_pitch((uint64_t)p.g.n_heads * p.g.hd) / 4 + 31) & ~(size_t)31);
    a.sync = p.sync;
    for (int i = 0; i < 2; i++) {
        a.pf[i] = p.pf[i];
        a.pf_bytes[i] = p.pf_bytes[i];
    }
    a.dev_err = c.dev_err;
    const size_t smem = ab_layout(a).total;
    bool uniform = true;  // one Q/K/V type: the instantiation for it; otherwise run-time types
    for (uint32_t s = 1; s < a.nseg; s++) uniform = uniform && a.seg_type[s] == a.seg_type[0];
    if (!uniform) return launch_ab_t<0, 0>(c, a, smem);
    switch (a.seg_type[0]) {
    case T_Q8_0: return launch_ab_q<T_Q8_0>(c, a, smem, a.otype);
    case T_Q4_K: return launch_ab_q<T_Q4_K>(c, a, smem, a.otype);
    case T_Q6_K: return launch_ab_q<T_Q6_K>(c, a, smem, a.otype);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace lt
