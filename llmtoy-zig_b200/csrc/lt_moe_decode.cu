// lt_moe_decode.cu — one token through a whole MoE block in one persistent
// kernel: pre-FFN RMSNorm, router logits, top-k + softmax weights, grouped
// gate/up with the activation, down projection, weighted combine and the
// residual add (src/model/gemma4/forward.zig:463-479 and 648-668,
// src/ops/moe.zig:61-76).
//
// At batch 1 the block is a chain of small dependent steps (x -> logits ->
// ids -> expert rows -> h -> out) whose weights are read once, and every
// global round trip on the chain costs about a microsecond.  One CTA per SM
// runs the chain with two grid-wide hand-offs:
//
//   phase R  every CTA stages x and normalises it (the router kernel's
//            reduction order); CTA e % G computes the logit of expert e with
//            its router row prefetched into registers before the wait for the
//            previous kernel, and publishes it as one 64-bit word tagged with
//            the launch's epoch.  Every CTA polls the E words directly (no
//            separate barrier) and ranks them itself: identical inputs and
//            code, so identical ids everywhere.
//   phase G  each CTA issues one TMA bulk copy per 8 gate/up pairs of its
//            share (whole 16-pair units of the k*F (slot, row) pairs), all at
//            once, computes its h values as the copies land, requests its
//            share of the down rows (one copy per slot), quantises h
//            (16-groups) and writes it into the shared-memory image of its
//            slot in global memory.                       -> grid barrier
//   phase D  each CTA copies the k slot images with one TMA copy each and
//            finishes its down rows for every slot, combines them in slot
//            order and adds the residual kept from phase R.
//
// Dense mode (a dense FFN block, forward.zig:307-312): no router; one slot
// holds "expert" 0 -- the 2-D gate/up/down tensors -- with weight 1.
// Scaled-router mode (Gemma 4, gemma4/forward.zig:401-413): the experts take
// rmsnorm(x) * norm_w and the router x * rms_inv * router_gs * router_scale
// (rmsnormWeightedAndRawScaled, math.zig:51-82), both from one rms_inv with
// the norm_pair glue kernel's arithmetic.
//
// Per-item decoding, partial-sum orders and the combine are those of the
// router / gate_up / down kernels, so both paths give the same bits.
#include "lt_qact.cuh"
#include "lt_router.cuh"
#include "lt_rowdot.cuh"

namespace lt {

constexpr int kDecWarps = 16;
constexpr int kDecThreads = kDecWarps * 32;
constexpr int kDecChunk = 8;          // gate/up pairs per TMA chunk
constexpr int kDecUnit = 16;          // pairs per work unit (one quantisation group)
constexpr int kDecMaxChunks = 48;     // chunk mbarriers; then k down-slot barriers, then the h barrier
constexpr int kDecNormThreads = 128;  // RMSNorm reduction width of the router kernel

// Layout of the context's sync block (DecodeParams::sync).
constexpr size_t kSyncEpoch = 0;   // u64 counter: epoch arrivals
constexpr size_t kSyncB = 33024;   // split counters (kGridSplitBytes): the hand-off after h, after the logits
constexpr size_t kSyncLogits = 256;  // tagged logits, one 128-byte line each (u64 [kRouterMaxE][16])
// Every CTA polls every logit: with the words packed into a few lines, the
// 148 x E polls queue at a few L2 slices (measured: the exchange ended up to
// 3 us after the last logit was stored); one line per logit spreads them.
constexpr size_t kSyncLogitStride = 16;
static_assert(kSyncLogits + 8 * kSyncLogitStride * kRouterMaxE <= kSyncB && kSyncB + kGridSplitBytes <= kDecodeSyncBytes,
              "decode sync block");

struct DecodeArgs {
    // router
    const float *rw;  // [E][rw_ld]
    uint32_t E, d, rw_ld;
    const float *x;       // [d]
    const float *norm_w;  // nullable
    const float *router_scale;  // nullable: the router input is x * rms_inv * router_gs * router_scale
    float router_gs;
    float eps;
    uint32_t k;
    int norm_topk;
    const float *escale;  // nullable
    uint32_t *ids;
    float *wout;
    // experts
    const uint8_t *gate, *up;  // up == nullptr: fused gate_up tensor
    uint64_t gpitch;
    uint32_t F, gi, gnb;  // items and 32-blocks per gate row
    int act;
    const uint8_t *down;
    uint64_t dpitch;
    uint32_t di, dnb;
    uint8_t *himg;  // [k][img] quantised h in the shared-memory layout (xs_bytes(1, di) per slot)
    uint32_t img;
    int residual;
    int dense;   // no router: slot 0 = expert 0 with weight 1
    int late_down;  // down tiles copied after the h barrier into the gate/up tiles' space
    float *out;  // [d], may alias x
    uint8_t *sync;
    int *dev_err;
    uint32_t maxpairs, maxrows;  // per-CTA maxima the layout is sized for
    uint32_t gchunks;            // gate/up chunks the tile space holds: more are copied in rounds
    const uint8_t *pf[2];        // optional L2 prefetch ranges (the next kernel's weights)
    uint64_t pf_bytes[2];
};

struct DecodeLayout {
    size_t bars, misc, lg, keys, cnt, part, ys, hs, xres, xsx, rr, gt, dt, total;
};

__host__ __device__ inline uint32_t chunks64(uint32_t cols) { return (cols + 63) / 64; }

// late_down: the down tiles share the gate/up tiles' space and are copied
// after the h barrier (when both do not fit at once).
__host__ __device__ inline DecodeLayout decode_layout(uint32_t E, uint32_t d, uint32_t F, uint32_t k, uint64_t gpitch,
                                                      uint32_t gi, uint64_t dpitch, uint32_t di, uint32_t img,
                                                      uint32_t maxpairs, uint32_t maxrows, int late_down,
                                                      uint32_t gchunks) {
    DecodeLayout L;
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off += (b + 127) & ~(size_t)127;
        return o;
    };
    L.bars = take((size_t)(kDecMaxChunks + 19) * 8);
    L.misc = take(256);
    L.lg = take((size_t)E * 4);
    L.keys = take((size_t)(E + 2) * 8);
    L.cnt = take((size_t)4 * E * 4);
    const size_t pg = (size_t)(2 * maxpairs + 1) * chunks64(d), pd = (size_t)(k * maxrows + 1) * chunks64(F);
    L.part = take((pg > pd ? pg : pd) * 4);
    L.ys = take((size_t)k * maxrows * 4);
    L.hs = take((size_t)maxpairs * 4);
    L.xres = take((size_t)maxrows * 4);
    L.xsx = take(xs_bytes(1, gi));
    const size_t rr0 = (size_t)2 * d * 4, rr1 = (size_t)k * img;
    L.rr = take(rr0 > rr1 ? rr0 : rr1);
    const size_t gtb = (size_t)gchunks * 2 * kDecChunk * gpitch, dtb = (size_t)k * maxrows * dpitch;
    if (late_down) {
        L.gt = take(gtb > dtb ? gtb : dtb);
        L.dt = L.gt;
    } else {
        L.gt = take(gtb);
        L.dt = take(dtb);
    }
    take(128);  // the last Q8_0 chunk of a row reads up to 34 bytes past it
    L.total = off;
    return L;
}

// Phase timestamps for tuning builds (-DLT_DECODE_TRACE): thread 0 of each
// CTA records globaltimer at the phase boundaries of the latest launch.  Off
// in the library the package builds.
#ifdef LT_DECODE_TRACE
constexpr int kDtCtas = 160, kDtMarks = 24;
__device__ unsigned long long g_moe_trace[kDtCtas * kDtMarks];
#define DT_MARK(m)                                                                      \
    do {                                                                                \
        if (tid == 0 && c < kDtCtas) g_moe_trace[c * kDtMarks + (m)] = globaltimer_ns(); \
    } while (0)
extern "C" int lt_moe_trace_copy(void *dst, size_t bytes) {
    return (int)cudaMemcpyFromSymbol(dst, g_moe_trace, bytes);
}
#else
#define DT_MARK(m) \
    do {           \
    } while (0)
#endif

// ROUNDS: the gate/up share is taken in rounds of a.gchunks chunks (only
// instantiated for launches whose share exceeds the tile space).
template <uint32_t GT, uint32_t DT, bool ROUNDS>
__global__ void __launch_bounds__(kDecThreads) k_moe_decode(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t G = gridDim.x, c = blockIdx.x;
    const DecodeLayout L =
        decode_layout(a.E, a.d, a.F, a.k, a.gpitch, a.gi, a.dpitch, a.di, a.img, a.maxpairs, a.maxrows, a.late_down,
                      a.gchunks);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *hbar = bars + kDecMaxChunks + 16;
    uint64_t *rbar = bars + kDecMaxChunks + 17;  // this CTA's router rows
    uint64_t *nbar = bars + kDecMaxChunks + 18;  // the norm weights
    uint32_t *s_sel = reinterpret_cast<uint32_t *>(smem + L.misc);    // [16]
    float *s_w = reinterpret_cast<float *>(smem + L.misc + 64);       // [16]
    float *s_ss = reinterpret_cast<float *>(smem + L.misc + 128);     // [4]
    float *s_stat = reinterpret_cast<float *>(smem + L.misc + 160);   // rms, max, expsum
    uint64_t *s_epoch = reinterpret_cast<uint64_t *>(smem + L.misc + 192);
    float *s_lg = reinterpret_cast<float *>(smem + L.lg);
    uint64_t *s_key = reinterpret_cast<uint64_t *>(smem + L.keys);
    uint32_t *s_cnt = reinterpret_cast<uint32_t *>(smem + L.cnt);
    float *part = reinterpret_cast<float *>(smem + L.part);
    float *s_y = reinterpret_cast<float *>(smem + L.ys);
    float *s_h = reinterpret_cast<float *>(smem + L.hs);
    float *s_xres = reinterpret_cast<float *>(smem + L.xres);
    const XS Xx = xs_carve(smem + L.xsx, 1, (int)a.gi);
    float *xsm = reinterpret_cast<float *>(smem + L.rr);  // [d] x, normalised in place
    float *nwsm = xsm + a.d;                              // [d] norm weights
    uint8_t *gt = smem + L.gt, *dt = smem + L.dt;
    unsigned long long *ctr_epoch = reinterpret_cast<unsigned long long *>(a.sync + kSyncEpoch);
    unsigned long long *ctr_b = reinterpret_cast<unsigned long long *>(a.sync + kSyncB);
    unsigned long long *lslots = reinterpret_cast<unsigned long long *>(a.sync + kSyncLogits);

    // this CTA's shares: gate/up pairs [p0, p1) of the k*F (slot, row) pairs
    // in whole 16-pair units, down rows [r0, r1) of d (for every slot)
    const uint32_t nunits = a.k * a.F / kDecUnit;
    const uint32_t p0 = kDecUnit * (uint32_t)((uint64_t)c * nunits / G);
    const uint32_t p1 = kDecUnit * (uint32_t)((uint64_t)(c + 1) * nunits / G);
    const uint32_t r0 = (uint32_t)((uint64_t)c * a.d / G), r1 = (uint32_t)((uint64_t)(c + 1) * a.d / G);
    const uint32_t np = p1 - p0, nr = r1 - r0;
    const uint32_t ch0 = p0 / kDecChunk;
    const uint32_t nchunks = np / kDecChunk;  // p0, p1 are multiples of 16

    DT_MARK(0);
    if (tid < 16) s_sel[tid] = 0;  // ranks form a permutation; this only keeps ids in range regardless
    // static inputs first: this CTA's router rows (expert c + w*G for warp w,
    // into the gate/up tile space, free until phase G) and the norm weights
    const uint32_t e_mine = c + (uint32_t)warp * G;
    const bool has_e = !a.dense && e_mine < a.E;
    const uint32_t nlw = a.dense ? 0 : a.E > c ? (a.E - c + G - 1) / G : 0;  // warps with a logit
    const float *wrow = reinterpret_cast<const float *>(gt) + (size_t)warp * a.d;
    if (tid == 0) {
        for (uint32_t i = 0; i < nchunks; i++) mbar_init(&bars[i], 1);
        for (uint32_t i = 0; i < a.k; i++) mbar_init(&bars[kDecMaxChunks + i], 1);
        mbar_init(hbar, 1);
        mbar_init(rbar, 1);
        mbar_init(nbar, 1);
        fence_barrier_init();
        if (nlw) {
            mbar_arrive_expect_tx(rbar, nlw * a.d * 4);
            for (uint32_t w = 0; w < nlw; w++)
                tma_load_1d(gt + (size_t)w * a.d * 4, a.rw + (size_t)(c + w * G) * a.rw_ld, a.d * 4, rbar);
        }
    }
    // the norm weights by TMA as well: a load loop here would hold every thread
    // until its loads return before it reaches the wait for the producer
    const bool nw_tma = a.norm_w && (reinterpret_cast<uintptr_t>(a.norm_w) & 15) == 0;
    if (nw_tma && tid == 0) {
        mbar_arrive_expect_tx(nbar, a.d * 4);
        tma_load_1d(nwsm, a.norm_w, a.d * 4, nbar);
    } else if (a.norm_w && !nw_tma) {
        for (uint32_t i = tid; i < a.d; i += kDecThreads) nwsm[i] = __ldg(a.norm_w + i);
    }
    pdl_launch_dependents();
    pdl_wait();
    DT_MARK(1);

    // ── phase R ──────────────────────────────────────────────────────────────
    uint64_t epoch = 0;
    if (tid == 0) epoch = grid_epoch(ctr_epoch, G);  // returns while x streams in
    if ((a.d & 3) == 0) {
#pragma unroll 4
        for (uint32_t i = tid; i < a.d / 4; i += kDecThreads)
            reinterpret_cast<float4 *>(xsm)[i] = __ldcg(reinterpret_cast<const float4 *>(a.x) + i);
    } else {
#pragma unroll 4
        for (uint32_t i = tid; i < a.d; i += kDecThreads) xsm[i] = __ldcg(a.x + i);
    }
    __syncthreads();
    DT_MARK(2);
    if (nw_tma) tile_wait(nbar, a.dev_err);
    for (uint32_t r = tid; r < nr; r += kDecThreads) s_xres[r] = xsm[r0 + r];
    const float *xrouter = xsm;  // the router's input
    if (a.norm_w && a.router_scale) {  // norm_pair: one rms_inv, per-thread sums over 512 strided values
        float ss = 0.0f;
        for (uint32_t i = tid; i < a.d; i += kDecThreads) ss = __fadd_rn(ss, __fmul_rn(xsm[i], xsm[i]));
        ss = warp_sum(ss);
        if (lane == 0) part[warp] = ss;
        __syncthreads();
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < kDecWarps; w++) s += part[w];
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)a.d), a.eps)));
        const float rb = __fmul_rn(r, a.router_gs);
        for (uint32_t i = tid; i < a.d; i += kDecThreads) {  // each thread its own elements: no hazard
            const float xi = xsm[i];
            const float e = __fmul_rn(__fmul_rn(xi, r), nwsm[i]);
            nwsm[i] = __fmul_rn(__fmul_rn(xi, rb), __ldg(a.router_scale + i));
            xsm[i] = e;
        }
        xrouter = nwsm;
    } else if (a.norm_w) {  // rmsnorm(out, x, w, eps) with the router kernel's reduction order
        float ss = 0.0f;
        if (tid < kDecNormThreads)
            for (uint32_t i = tid; i < a.d; i += kDecNormThreads) ss += xsm[i] * xsm[i];
        ss = warp_sum(ss);
        if (lane == 0 && warp < kDecNormThreads / 32) s_ss[warp] = ss;
        __syncthreads();
        if (tid == 0) {
            float s = 0.0f;
            for (int w = 0; w < kDecNormThreads / 32; w++) s += s_ss[w];
            s_stat[0] = 1.0f / sqrtf(s / (float)a.d + a.eps);
        }
        __syncthreads();
        const float rms = s_stat[0];
        for (uint32_t i = tid; i < a.d; i += kDecThreads) xsm[i] = xsm[i] * rms * nwsm[i];
    }
    if (tid == 0) *s_epoch = epoch;  // the atomic has long returned by now
    __syncthreads();
    epoch = *s_epoch;
    DT_MARK(3);
    const uint32_t tag = (uint32_t)epoch;
    // warps [0, nlw) compute this CTA's logits; the others quantise the
    // normalised x for this CTA's gate/up meanwhile
    if (has_e) {
        const float v = tile_wait(rbar, a.dev_err) ? router_logit_sm(wrow, xrouter, a.d, lane) : 0.0f;
        // the row's space takes the gate/up tiles (async proxy) after this read
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (lane == 0) st_relaxed_u64(lslots + kSyncLogitStride * e_mine, ((uint64_t)tag << 32) | __float_as_uint(v));
        DT_MARK(4);
    } else {
        for (uint32_t b = warp - nlw; b < a.d / 32; b += kDecWarps - nlw)
            qact_block_to_xs(Xx, 0, (int)b, xsm[32 * b + lane], lane);
    }
    if (!a.dense && tid < a.E) {  // poll this expert's logit until it carries this launch's tag
        uint64_t v = ld_relaxed_u64(lslots + kSyncLogitStride * tid);
        if ((uint32_t)(v >> 32) != tag) {
            const uint64_t t0 = globaltimer_ns();
            for (;;) {
                v = ld_relaxed_u64(lslots + kSyncLogitStride * tid);
                if ((uint32_t)(v >> 32) == tag) break;
                if (globaltimer_ns() - t0 > kWaitLimitNs) {
                    if (a.dev_err) atomicExch(a.dev_err, DEV_ERR_GRID_TIMEOUT);
                    break;
                }
            }
        }
        const float lv = __uint_as_float((uint32_t)v);
        s_lg[tid] = lv;
        s_key[tid] = router_key(lv, tid);
    }
    if (tid == 0) s_key[a.E] = 0;
    __syncthreads();
    DT_MARK(5);
    if (!a.dense) {
        if (warp == kDecWarps - 1) {  // softmax statistics while the other warps rank
            float mx, es;
            router_softmax_stats(s_lg, a.E, lane, mx, es);
            if (lane == 0) {
                s_stat[1] = mx;
                s_stat[2] = es;
            }
        }
        router_rank_keys_split(s_key, a.E, a.k, s_sel, min(4u, (uint32_t)(kDecThreads - 32) / a.E), s_cnt, tid);
    }
    __syncthreads();
    DT_MARK(6);

    // ── phase G ──────────────────────────────────────────────────────────────
    // chunk j: [8 gate rows][8 up rows] of pairs p0 + 8j.., into tile slot j % gchunks
    auto issue_chunk = [&](uint32_t j) {
        const uint32_t q0 = p0 + j * kDecChunk;
        const uint32_t s = q0 / a.F, f0 = q0 - s * a.F;
        const uint32_t e = min(s_sel[s], a.E - 1);
        const uint32_t bytes = (uint32_t)(kDecChunk * a.gpitch);
        uint64_t grow, urow;
        const uint8_t *ub;
        if (a.up) {
            grow = (uint64_t)e * a.F + f0;
            urow = grow;
            ub = a.up;
        } else {  // fused: gate rows [0,F), up rows [F,2F) (gemma4/forward.zig:469-471)
            grow = (uint64_t)e * 2 * a.F + f0;
            urow = grow + a.F;
            ub = a.gate;
        }
        uint8_t *dst = gt + (size_t)2 * (ROUNDS ? j % a.gchunks : j) * kDecChunk * a.gpitch;
        mbar_arrive_expect_tx(&bars[j], 2 * bytes);
        tma_load_1d(dst, a.gate + grow * a.gpitch, bytes, &bars[j]);
        tma_load_1d(dst + bytes, ub + urow * a.gpitch, bytes, &bars[j]);
    };
    if (warp == 0) {  // one TMA chunk per lane: the first round's
        for (uint32_t j = lane; j < (ROUNDS ? min(nchunks, a.gchunks) : nchunks); j += 32) issue_chunk(j);
        DT_MARK(7);
    } else if (warp == 2 && lane == 0) {
        if (a.dense)
            s_w[0] = 1.0f;
        else
            router_weights(s_lg, s_sel, a.k, s_stat[1], s_stat[2], a.norm_topk, a.escale, s_w);
        if (c == 0 && !a.dense)
            for (uint32_t i = 0; i < a.k; i++) {
                a.ids[i] = s_sel[i];
                a.wout[i] = s_w[i];
            }
    }
    // gate/up: warp w takes tile rows w*rps.., one TMA chunk (16 tile rows)
    // after another; a lane owns one 64-column chunk of x in registers.  When
    // the tile space holds fewer chunks than this CTA's share, the share goes
    // in rounds of gchunks chunks, each copied over the previous round's.
    const uint32_t cpr_g = chunks64(a.d);
    const uint32_t gstride = 2 * a.maxpairs + 1;  // partials [chunk][tile row], odd stride: no bank conflicts
    // tile rows [rbase, nrows) of the share, held from tile row 0
    auto gate_up_rows = [&](uint32_t rbase, uint32_t nrows) {
        const uint32_t lpr = min(cpr_g, 32u), rps = 32 / lpr;  // lanes per row, rows per step
        const uint32_t sub = lane / lpr;
        if (sub < rps) {
            for (uint32_t cg = 0; cg < cpr_g; cg += lpr) {
                const uint32_t n = min(lpr, cpr_g - cg);
                if (lane % lpr >= n) continue;
                const uint32_t cb = cg + spread_chunk(lane % lpr, n);
                XChunk xc;
                xchunk_load(Xx, 0, (int)cb, xc);
                // two rows per iteration (independent chains for the scheduler);
                // an odd last row is computed twice and stored once
                const uint32_t step = kDecWarps * rps;
                for (uint32_t r = rbase + warp * rps + sub; r < nrows; r += 2 * step) {
                    const uint32_t rb = r + step < nrows ? r + step : r;
                    const bool ok = tile_wait(&bars[r / (2 * kDecChunk)], a.dev_err) &
                                    tile_wait(&bars[rb / (2 * kDecChunk)], a.dev_err);
                    float ya = 0.0f, yb = 0.0f;
                    if (ok) {
                        ya = dot64<GT>(gt + (size_t)(r - rbase) * a.gpitch, (int)cb, (int)a.gnb, xc);
                        yb = dot64<GT>(gt + (size_t)(rb - rbase) * a.gpitch, (int)cb, (int)a.gnb, xc);
                    }
                    part[cb * gstride + r] = ya;
                    part[cb * gstride + rb] = yb;
                }
            }
        }
    };
    if constexpr (ROUNDS) {
        const uint32_t rows_round = 2 * kDecChunk * a.gchunks;
        for (uint32_t rbase = 0; rbase < 2 * np; rbase += rows_round) {
            if (rbase) {  // the previous round's rows are consumed
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncthreads();
                if (tid == 0)
                    for (uint32_t j = rbase / (2 * kDecChunk); j < min(nchunks, (rbase + rows_round) / (2 * kDecChunk));
                         j++)
                        issue_chunk(j);
            }
            gate_up_rows(rbase, min(2 * np, rbase + rows_round));
        }
    } else {
        gate_up_rows(0, 2 * np);
    }
    DT_MARK(8);
    __syncthreads();
    DT_MARK(9);
    // down rows [r0, r1) of each slot's expert, requested once this CTA's
    // gate/up rows are consumed: until then every CTA's HBM requests are the
    // gate/up rows, which the grid's slowest CTA (and so the h barrier) waits for
    if (warp == 1 && !a.late_down && (uint32_t)lane < a.k && nr) {
        const uint32_t e = min(s_sel[lane], a.E - 1);
        const uint32_t bytes = (uint32_t)(nr * a.dpitch);
        mbar_arrive_expect_tx(&bars[kDecMaxChunks + lane], bytes);
        tma_load_1d(dt + (size_t)lane * a.maxrows * a.dpitch, a.down + ((uint64_t)e * a.d + r0) * a.dpitch, bytes,
                    &bars[kDecMaxChunks + lane]);
    }
    for (uint32_t lp = tid; lp < np; lp += kDecThreads) {  // chunk partials summed in column order
        const uint32_t rg = 2 * kDecChunk * (lp / kDecChunk) + lp % kDecChunk;
        const float *pg = part + rg, *pu = pg + kDecChunk;
        float g = 0.0f, u = 0.0f;
        for (uint32_t i = 0; i < cpr_g; i++) {
            g += pg[i * gstride];
            u += pu[i * gstride];
        }
        s_h[lp] = act_apply(a.act, g) * u;
    }
    __syncthreads();
    DT_MARK(10);
    // quantise this CTA's h values into their slots' images (32-blocks; a
    // block may be half this CTA's)
    for (uint32_t b = p0 / 32 + warp; b * 32 < p1; b += kDecWarps) {
        const uint32_t q = 32 * b + lane;
        const bool own = q >= p0 && q < p1;
        const uint32_t s = (32 * b) / a.F, bs = (32 * b - s * a.F) / 32;  // F % 32 == 0: blocks stay in a slot
        const XS Xs = xs_carve(a.himg + (size_t)s * a.img, 1, (int)a.di);
        qact_block_to_xs(Xs, 0, (int)bs, own ? s_h[q - p0] : 0.0f, lane, own);
    }
    fence_proxy_async_global();  // the images are read by TMA after the barrier
    // the slot images land (by TMA) where x and the norm weights were
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    DT_MARK(11);
    grid_arrive_split(ctr_b);
    grid_wait_split(ctr_b, epoch, a.dev_err, kWaitLimitNs);
    DT_MARK(12);
    // the L2 prefetch of the next kernel's weights: after the h hand-off, so
    // that it does not compete with this launch's down rows for DRAM
    if (tid >= 64 && tid < 66 && a.pf[tid - 64]) prefetch_l2_share(a.pf[tid - 64], a.pf_bytes[tid - 64], c, G);

    // ── phase D ──────────────────────────────────────────────────────────────
    uint8_t *himg_s = smem + L.rr;  // k slot images, a.img bytes each
    if (tid == 0) {
        fence_proxy_async_global();
        mbar_arrive_expect_tx(hbar, a.k * a.img);
        for (uint32_t s = 0; s < a.k; s++)
            tma_load_1d(himg_s + (size_t)s * a.img, a.himg + (size_t)s * a.img, a.img, hbar);
        if (a.late_down && nr)  // the gate/up tiles are consumed: the down rows take their place
            for (uint32_t s = 0; s < a.k; s++) {
                const uint32_t e = min(s_sel[s], a.E - 1);
                const uint32_t bytes = (uint32_t)(nr * a.dpitch);
                mbar_arrive_expect_tx(&bars[kDecMaxChunks + s], bytes);
                tma_load_1d(dt + (size_t)s * a.maxrows * a.dpitch, a.down + ((uint64_t)e * a.d + r0) * a.dpitch, bytes,
                            &bars[kDecMaxChunks + s]);
            }
    }
    const bool hok = tile_wait(hbar, a.dev_err);
    DT_MARK(13);
    // down: warps [s*wps, (s+1)*wps) take slot s; a lane owns one 64-column
    // chunk of that slot's h in registers
    const uint32_t cpr_d = chunks64(a.F);
    const uint32_t dstride = a.k * a.maxrows + 1;  // partials [chunk][slot row]
    {
        const uint32_t lpr = min(cpr_d, 32u), rps = 32 / lpr;
        const uint32_t sub = lane / lpr;
        const uint32_t wps = max(1u, (uint32_t)kDecWarps / a.k);
        const uint32_t s = warp / wps, ws = warp % wps;
        if (s < a.k && sub < rps && nr) {
            const bool ok = tile_wait(&bars[kDecMaxChunks + s], a.dev_err) && hok;
            const XS Xh = xs_carve(himg_s + (size_t)s * a.img, 1, (int)a.di);
            for (uint32_t cg = 0; cg < cpr_d; cg += lpr) {
                const uint32_t n = min(lpr, cpr_d - cg);
                if (lane % lpr >= n) continue;
                const uint32_t cb = cg + spread_chunk(lane % lpr, n);
                XChunk xc;
                xchunk_load(Xh, 0, (int)cb, xc);
                const uint32_t step = wps * rps;
                for (uint32_t r = ws * rps + sub; r < nr; r += 2 * step) {
                    const uint32_t rb = r + step < nr ? r + step : r;
                    const uint32_t ta = s * a.maxrows + r, tb = s * a.maxrows + rb;
                    float ya = 0.0f, yb = 0.0f;
                    if (ok) {
                        ya = dot64<DT>(dt + (size_t)ta * a.dpitch, (int)cb, (int)a.dnb, xc);
                        yb = dot64<DT>(dt + (size_t)tb * a.dpitch, (int)cb, (int)a.dnb, xc);
                    }
                    part[cb * dstride + ta] = ya;
                    part[cb * dstride + tb] = yb;
                }
            }
        }
    }
    __syncthreads();
    DT_MARK(14);
    for (uint32_t w = tid; w < a.k * nr; w += kDecThreads) {  // y[s][r]: chunk partials in column order
        const uint32_t s = w / nr, r = w - s * nr;
        const float *pp = part + s * a.maxrows + r;
        float y = 0.0f;
        for (uint32_t i = 0; i < cpr_d; i++) y += pp[i * dstride];
        s_y[s * a.maxrows + r] = y;
    }
    __syncthreads();
    DT_MARK(15);
    for (uint32_t r = tid; r < nr; r += kDecThreads) {
        float o = 0.0f;  // moe_buf is zeroed, then += scale * down, slot by slot
        for (uint32_t s = 0; s < a.k; s++) o += s_w[s] * s_y[s * a.maxrows + r];
        a.out[r0 + r] = a.residual ? s_xres[r] + o : o;
    }
    DT_MARK(16);
}

namespace {

struct DecodePlan {
    DecodeArgs a;
    size_t smem;
};

bool decode_plan(const DecodeParams &p, int num_sms, DecodePlan &out) {
    if (num_sms <= 0 || p.k == 0 || p.k > 16 || p.E == 0 || p.E > (uint32_t)kRouterMaxE) return false;
    if (!p.router && (p.k != 1 || p.E != 1)) return false;  // dense mode: one slot, expert 0
    auto ok_type = [](uint32_t t) { return t == T_Q8_0 || t == T_Q4_K || t == T_Q6_K; };
    if (!ok_type(p.gate.type) || !ok_type(p.down.type)) return false;  // the grouped kernels take the rest
    const uint32_t G = (uint32_t)num_sms;
    DecodeArgs &a = out.a;
    a.rw = p.router;
    a.E = p.E;
    a.d = p.d;
    a.rw_ld = p.router_ld;
    a.x = p.x;
    a.norm_w = p.norm_w;
    a.router_scale = p.router_scale;
    a.router_gs = p.router_gs;
    a.eps = p.eps;
    a.k = p.k;
    a.norm_topk = p.norm_topk;
    a.escale = p.escale;
    a.ids = p.ids;
    a.wout = p.w;
    a.gate = p.gate.data;
    a.up = p.up_data;
    a.gpitch = p.gate.pitch;
    a.F = p.F;
    a.gi = items_per_row(p.gate.type, p.gate.cols);
    a.gnb = (uint32_t)(p.gate.cols / 32);
    a.act = p.act;
    a.down = p.down.data;
    a.dpitch = p.down.pitch;
    a.di = items_per_row(p.down.type, p.down.cols);
    a.dnb = (uint32_t)(p.down.cols / 32);
    a.himg = p.himg;
    a.img = (uint32_t)moe_decode_img_bytes(p.F);
    a.residual = p.residual;
    a.dense = p.router == nullptr;
    a.out = p.out;
    a.sync = p.sync;
    a.dev_err = nullptr;
    for (int i = 0; i < 2; i++) {
        a.pf[i] = p.pf[i];
        a.pf_bytes[i] = p.pf_bytes[i];
    }
    if (p.d % 32 != 0 || p.F % 32 != 0) return false;
    if (a.rw && ((p.router_ld % 4) != 0 || (reinterpret_cast<uintptr_t>(a.rw) & 15) != 0 || p.E > 2 * G)) return false;
    const uint64_t nunits = (uint64_t)p.k * p.F / kDecUnit;
    a.maxpairs = (uint32_t)(kDecUnit * ((nunits + G - 1) / G));
    a.maxrows = (p.d + G - 1) / G;
    if (a.maxpairs / kDecChunk > (uint32_t)kDecMaxChunks) return false;
    // the whole share at once with the down rows beside it; else the down rows
    // after the h barrier in the gate/up space; else the gate/up share in rounds
    for (uint32_t gc = a.maxpairs / kDecChunk; gc >= 1; gc--) {
        for (int late = 0; late < 2; late++) {
            const DecodeLayout L = decode_layout(a.E, a.d, a.F, a.k, a.gpitch, a.gi, a.dpitch, a.di, a.img,
                                                 a.maxpairs, a.maxrows, late, gc);
            if (L.total <= kDecodeSmemLimit) {
                a.late_down = late;
                a.gchunks = gc;
                out.smem = L.total;
                return true;
            }
        }
    }
    return false;
}

template <uint32_t GT, uint32_t DT>
cudaError_t launch_decode_t(const LaunchCfg &c, const DecodePlan &pl) {
    if (pl.a.gchunks * kDecChunk < pl.a.maxpairs)
        return launch_k(c, "moe_decode", k_moe_decode<GT, DT, true>, dim3((unsigned)c.num_sms), dim3(kDecThreads),
                        pl.smem, pl.a);
    return launch_k(c, "moe_decode", k_moe_decode<GT, DT, false>, dim3((unsigned)c.num_sms), dim3(kDecThreads),
                    pl.smem, pl.a);
}

template <uint32_t GT>
cudaError_t launch_decode_g(const LaunchCfg &c, const DecodePlan &pl, uint32_t dtype) {
    switch (dtype) {
    case T_Q4_K: return launch_decode_t<GT, T_Q4_K>(c, pl);
    case T_Q6_K: return launch_decode_t<GT, T_Q6_K>(c, pl);
    case T_Q8_0: return launch_decode_t<GT, T_Q8_0>(c, pl);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace

size_t moe_decode_img_bytes(uint64_t F) { return xs_bytes(1, (int)((F + 255) / 256)); }

bool moe_decode_fits(const DecodeParams &p, int num_sms) {
    DecodePlan pl;
    return decode_plan(p, num_sms, pl);
}

cudaError_t launch_moe_decode(const LaunchCfg &c, const DecodeParams &p) {
    DecodePlan pl;
    if (!decode_plan(p, c.num_sms, pl)) return cudaErrorInvalidValue;
    pl.a.dev_err = c.dev_err;
    switch (p.gate.type) {
    case T_Q4_K: return launch_decode_g<T_Q4_K>(c, pl, p.down.type);
    case T_Q6_K: return launch_decode_g<T_Q6_K>(c, pl, p.down.type);
    case T_Q8_0: return launch_decode_g<T_Q8_0>(c, pl, p.down.type);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace lt
