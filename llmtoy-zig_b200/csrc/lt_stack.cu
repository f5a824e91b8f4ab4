// lt_stack.cu — every decoder layer of one token in one persistent kernel
// (one CTA per SM): the loop body of forwardOneModel (src/model/forward.zig:
// 260-316) for the Qwen-style layers of configs 0 and 2 -- RMSNorm, stacked
// Q/K/V rows (+bias), per-head Q/K RMSNorm and RoPE, the K/V append,
// attention, wo + residual, then the FFN half: a MoE block (router, top-k,
// renormalised weights, SwiGLU experts, slot-order combine, residual;
// src/model/gemma4/forward.zig:463-479, src/ops/moe.zig:61-76) or a dense
// SwiGLU block (forward.zig:307-312).
//
// At batch 1 each layer is a chain of small dependent steps whose weights
// are read once.  Launching a kernel per half-layer costs a hand-off of about
// two microseconds each time (the next kernel's CTAs start only when the
// previous ones leave their SM) and leaves no room to fetch the next layer's
// weights early.  Here the CTAs stay resident for the whole stack; the phases
// of a layer hand over through grid barriers (bounded waits), and every
// weight tile that does not depend on the data is copied into shared memory
// (TMA) or prefetched into L2 while an earlier phase runs:
//
//   Q  x -> RMSNorm -> quantised row; this CTA's Q/K/V rows (copied during
//      the previous layer's D phase)                          -> barrier
//   A  (head, split) items: Q/K norm, RoPE, K/V append, online-softmax
//      attention over the split's positions; the last split of a head merges
//      it into the quantised attention row.  The wo rows are copied meanwhile
//      (an L2 prefetch of the next layer's rows here measured ~1.5 us slower
//      per layer: it competes with the attention's loads)       -> barrier
//   O  wo rows, residual: x' (kept in shared memory for the MoE residual)
//                                                             -> barrier
//   R  x' -> RMSNorm; CTA e computes the logit of expert e (router row copied
//      during the previous layer) and publishes it tagged with (launch,
//      layer); every CTA ranks the E logits itself
//   G  TMA of the selected experts' gate/up rows (this CTA's 16-pair units)
//      and down rows; h = act(g) * u quantised into per-slot images
//                                                             -> barrier
//   D  slot images copied in; down rows, slot-order combine, residual; the
//      next layer's Q/K/V rows and router row start copying   -> barrier
//
// Per-item decoding, row dots and partial-sum orders are those of
// k_attn_block and k_moe_decode, so the stack and the per-layer kernels
// give the same results up to the attention split merge order.
#include "lt_attn_common.cuh"
#include "lt_router.cuh"

namespace lt {

constexpr int kStWarps = kAbWarps;
constexpr int kStThreads = kAbThreads;
constexpr uint32_t kStChunk = 8;          // gate/up pairs per TMA chunk
constexpr uint32_t kStUnit = 16;          // pairs per work unit (one quantisation group)
constexpr uint32_t kStMaxChunks = 32;     // gate/up chunk mbarriers per CTA
constexpr uint32_t kStMaxSlots = 16;      // top-k slots
constexpr uint32_t kStSplitPositions = 256;  // positions per attention split before another CTA joins
                                              // (a merge across CTAs costs two L2 round trips: measured
                                              // slower than one CTA per head up to a few hundred positions)
constexpr uint32_t kStMaxSplits = 8;
constexpr int kStNormThreads = 128;       // k_moe_decode's RMSNorm reduction width

// The plan's sync block (kStackSyncBytes): launch counter, hand-off counter,
// tagged logits, per-head merge counters.
constexpr size_t kStEpoch = 0, kStBar = 128, kStLogits = 256, kStHeadCnt = kStLogits + 8 * kRouterMaxE;
constexpr uint32_t kStMaxCtas = 1024;
static_assert(kStHeadCnt + 4 * 1024 <= kStackSyncBytes, "sync block");

struct StackArgs {
    AttnGeom g;
    uint32_t d, qrows, nq, nkv;
    uint64_t qpitch, opitch;
    uint32_t qnb, onb;
    uint32_t E, k, F;
    int norm_topk, act, dense;
    uint64_t gpitch, dpitch;
    uint32_t gnb, dnb, di, img;
    float eps;
    uint32_t n_layers, nbar;  // barriers per launch
    const StackLayerDev *layers;
    float *x;
    const uint32_t *pos;
    float *qkv, *part;
    uint8_t *att, *himg, *sync;
    int *dev_err;
    uint32_t splits, maxq, maxo, maxpairs;
};

struct StLayout {
    size_t bars, misc, lg, keys, cnt, w, dn, rt, xs, xf, hs, ys, xres, lay, bias, total;
    size_t an, fn, qn, kn;  // norm weights inside W, after the Q/K/V or wo tile
};

__host__ __device__ inline uint32_t st_chunks64(uint32_t cols) { return (cols + 63) / 64; }
__host__ __device__ inline uint32_t st_items(uint32_t cols) { return (cols + 255) / 256; }

__host__ __device__ inline StLayout st_layout(const StackArgs &a) {
    StLayout L;
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off += (b + 127) & ~(size_t)127;
        return o;
    };
    auto mx = [](size_t p, size_t q) { return p > q ? p : q; };
    L.bars = take((size_t)(8 + kStMaxSlots + kStMaxChunks) * 8);
    L.misc = take(512);
    L.lg = take((size_t)a.E * 4);
    L.keys = take((size_t)(a.E + 2) * 8);
    L.cnt = take((size_t)4 * a.E * 4);
    // + slack: the last Q8_0 chunk of a row reads up to 34 bytes past it
    const size_t qt = (size_t)a.maxq * a.qpitch, ot = (size_t)a.maxo * a.opitch;
    const size_t gt = (size_t)2 * a.maxpairs * a.gpitch;
    // the layer's norm weights ride with its static tiles: attn_norm and the
    // Q/K norms with the Q/K/V rows, ffn_norm with the wo rows
    const size_t t0 = (mx(qt, ot) + 128 + 127) & ~(size_t)127;
    L.an = t0;
    L.fn = L.an + (size_t)a.d * 4;
    L.qn = L.fn + (size_t)a.d * 4;
    L.kn = L.qn + (size_t)a.g.hd * 4;
    L.w = take(mx(L.kn + (size_t)a.g.hd * 4, gt + 128));
    L.an += L.w;
    L.fn += L.w;
    L.qn += L.w;
    L.kn += L.w;
    L.dn = take((size_t)a.k * a.maxo * a.dpitch + 128);
    L.rt = take(a.dense ? 0 : (size_t)a.d * 4);
    L.xs = take(mx(mx(xs_bytes(1, (int)st_items(a.d)), xs_bytes(1, (int)st_items(a.nq))), (size_t)a.k * a.img));
    // f32 rows (x, x', the wo outputs), the attention item's head vectors, and
    // the gate/up and down partials: never live at the same time
    const size_t head = (size_t)(3 * a.g.hd + kStWarps * (a.g.hd + 2) + kStWarps + 2) * 4;
    const size_t pg = (size_t)(2 * a.maxpairs + 1) * st_chunks64(a.d) * 4;
    const size_t pd = (size_t)(a.k * a.maxo + 1) * st_chunks64(a.F) * 4;
    L.xf = take(mx(mx((size_t)mx(a.d, a.nq) * 4, head), mx(pg, pd)));
    L.hs = take((size_t)a.maxpairs * 4);
    L.ys = take((size_t)a.k * a.maxo * 4);
    L.xres = take((size_t)a.maxo * 4);
    L.lay = take((size_t)a.n_layers * sizeof(StackLayerDev));
    L.bias = take((size_t)a.maxq * 4);
    L.total = off;
    return L;
}

// Wait for phase `par` of a TMA barrier; on timeout record the error, wait
// once more for the copies in flight (they target this CTA's shared memory)
// and give up.
LT_DEVINL bool st_wait(uint64_t *bar, uint32_t par, int *dev_err) {
    if (mbar_wait_bounded(bar, par, kWaitLimitNs)) return true;
    if (dev_err) atomicExch(dev_err, DEV_ERR_TMA_TIMEOUT);
    mbar_wait_bounded(bar, par, kWaitLimitNs);
    return false;
}

// rows [r0, r0 + n) of a row-major tensor (pitch bytes) into L2, in pieces of
// at most 64 KB (bytes a multiple of 16: GGUF rows at a 16-byte pitch).
LT_DEVINL void st_prefetch_rows(const uint8_t *base, uint64_t pitch, uint32_t r0, uint32_t n) {
    const uint8_t *p = base + (uint64_t)r0 * pitch;
    const uint64_t bytes = (uint64_t)n * pitch;
    for (uint64_t b = 0; b < bytes; b += 65536) prefetch_l2(p + b, (uint32_t)(bytes - b < 65536 ? bytes - b : 65536));
}

// Phase timestamps for tuning builds (-DLT_STACK_TRACE): thread 0 of each CTA
// records globaltimer at the phase boundaries of every layer.  Off in the
// library the package builds.
#ifdef LT_STACK_TRACE
constexpr int kTraceCtas = 160, kTraceLayers = 64, kTraceMarks = 32;
__device__ unsigned long long g_stack_trace[kTraceCtas * kTraceLayers * kTraceMarks];
#define ST_MARK(m)                                                                              \
    do {                                                                                       \
        if (tid == 0 && c < kTraceCtas && l < kTraceLayers)                                    \
            g_stack_trace[((size_t)c * kTraceLayers + l) * kTraceMarks + (m)] = globaltimer_ns(); \
    } while (0)
#else
#define ST_MARK(m) \
    do {           \
    } while (0)
#endif

// ── grid hand-off ───────────────────────────────────────────────────────────
// One counter that only grows: every CTA adds 1 per hand-off, so hand-off n
// (counted over all launches of the plan, from 1) completes at n * G.  The
// arrival is one release add by thread 0 after the block barrier (the
// release covers the CTA's writes ordered before it by that barrier), the
// wait one acquire poll by thread 0 before the next block barrier.  Measured
// on B200: ~1 us from the last arrival to the first departure, against ~3.5
// us for per-CTA flags polled by every CTA (G x G acquire loads at once) and
// ~2 us with a full fence before the add.
LT_DEVINL void st_grid_sync(unsigned long long *ctr, uint32_t G, uint64_t seqn, int *dev_err) {
    __syncthreads();
    if (threadIdx.x == 0) {
        red_release_add_u64(ctr, 1ull);
        const uint64_t target = seqn * G;
        if (ld_acquire_u64(ctr) < target) {
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_u64(ctr) < target) {
                if (globaltimer_ns() - t0 > kWaitLimitNs) {
                    if (dev_err) atomicExch(dev_err, DEV_ERR_GRID_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncthreads();
}

// The heavy inner loops live in functions of their own (not inlined), so
// their registers are allocated apart from the long-lived state of the
// layer loop.

// rows [0, nrows) of a shared tile against X (ab_rows).
// Rows per warp: as few as fill the 16 warps (a warp's rows run one after
// another; the chunk each lane takes, so every row's sum order, is the same).
template <uint32_t T>
__device__ __noinline__ void st_rows(const uint8_t *tile, uint64_t pitch, uint32_t nrows, uint32_t cols, uint32_t nb,
                                     XS X, float *y) {
    const int warp = (int)(threadIdx.x >> 5), lane = (int)(threadIdx.x & 31);
    if (nrows <= (uint32_t)kStWarps)
        ab_rows<T, 1>(tile, pitch, nrows, cols, nb, X, warp, lane, y);
    else if (nrows <= 2u * kStWarps)
        ab_rows<T, 2>(tile, pitch, nrows, cols, nb, X, warp, lane, y);
    else if (nrows <= 3u * kStWarps)
        ab_rows<T, 3>(tile, pitch, nrows, cols, nb, X, warp, lane, y);
    else
        ab_rows<T, 4>(tile, pitch, nrows, cols, nb, X, warp, lane, y);
}

// Phase A: the (head, split) items of this CTA (k_attn_block's phase A).
template <int HD>
__device__ __noinline__ void st_attention(const StackArgs &a, const float *q_norm, const float *k_norm, void *kc,
                                          void *vc, float *XF, float *red, int *s_last, uint32_t *head_cnt,
                                          uint32_t pos, uint32_t S, uint32_t win, uint32_t first) {
    constexpr int PER = HD / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t G = gridDim.x, c = blockIdx.x;
    const uint32_t nq = a.nq, nkv = a.nkv, group = a.g.n_heads / a.g.n_kv;
    float *hq = XF, *hk = hq + HD, *hv = hk + HD;
    float *wpart = hv + HD;  // [16][HD + 2]: m, l, o[HD]
    for (uint32_t item = c; item < a.g.n_heads * S; item += G) {
        const uint32_t h = item / S, s = item - h * S, kh = h / group;
        if (tid < 3 * HD / 4) {  // q, k, v heads: one float4 each
            const uint32_t pt = tid / (HD / 4), i = tid % (HD / 4);
            const size_t off = pt == 0 ? (size_t)h * HD : pt == 1 ? nq + (size_t)kh * HD : nq + nkv + (size_t)kh * HD;
            reinterpret_cast<float4 *>(hq + pt * HD)[i] = __ldcg(reinterpret_cast<const float4 *>(a.qkv + off) + i);
        }
        __syncthreads();
        ab_norm_rope2(hq, q_norm, hk, k_norm, a.g, pos, red);
        if (s == 0 && h % group == 0) {  // this position's K/V into the cache
            const size_t slot = (size_t)(pos % a.g.cap) * nkv + (size_t)kh * HD;
            for (uint32_t i = tid; i < HD; i += kStThreads) {
                kv_st(kc, slot + i, hk[i], a.g.kv_f16);
                kv_st(vc, slot + i, hv[i], a.g.kv_f16);
            }
        }
        if (a.g.kv_f16) {  // attend to this position as the cache holds it
            __syncthreads();
            for (uint32_t i = tid; i < HD; i += kStThreads) {
                hk[i] = kv_round(hk[i], 1u);
                hv[i] = kv_round(hv[i], 1u);
            }
            __syncthreads();
        }
        float o[PER], m = -INFINITY, lsum = 0.0f;
        if (a.g.kv_f16)
            ab_attend<HD, true>(kc, vc, a.g, s, S, win, first, (size_t)kh * HD, nkv, hq, hk, hv, warp, lane, m, lsum, o);
        else
            ab_attend<HD, false>(kc, vc, a.g, s, S, win, first, (size_t)kh * HD, nkv, hq, hk, hv, warp, lane, m, lsum, o);
        float *wp = wpart + warp * (HD + 2);
        if (lane == 0) {
            wp[0] = m;
            wp[1] = lsum;
        }
#pragma unroll
        for (int i = 0; i < PER; i++) wp[2 + lane * PER + i] = o[i];
        __syncthreads();
        float *sf = wpart + kStWarps * (HD + 2);  // [16] scales, then the sum and the maximum
        if (warp == 0) {
            const float mw = lane < kStWarps ? wpart[lane * (HD + 2)] : -INFINITY;
            float M = mw;
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
            if (lane < kStWarps) sf[lane] = mw != -INFINITY ? expf(mw - M) : 0.0f;
            __syncwarp();
            if (lane == 0) {
                float Ls = 0.0f;
                for (int w = 0; w < kStWarps; w++) Ls += wpart[w * (HD + 2) + 1] * sf[w];
                sf[kStWarps] = Ls;
                sf[kStWarps + 1] = M;
            }
        }
        __syncthreads();
        if (S == 1) {  // the whole window: normalise, quantise into the attention row
            const float Ls = sf[kStWarps];
            for (uint32_t t = tid; t < HD; t += kStThreads) {
                float acc = 0.0f;
#pragma unroll
                for (int w = 0; w < kStWarps; w++) acc += wpart[w * (HD + 2) + 2 + t] * sf[w];
                hq[t] = acc / Ls;
            }
            __syncthreads();
            for (uint32_t b = warp; b < (uint32_t)HD / 32; b += kStWarps)
                qact_store_block(a.att, (int)nq, (int)(h * HD / 32 + b), hq[32 * b + lane], lane);
            __syncthreads();
            continue;
        }
        float *po = a.part + ((size_t)h * S + s) * HD;
        float *pml = a.part + (size_t)a.g.n_heads * S * HD + 2 * ((size_t)h * S + s);
        for (uint32_t t = tid; t < HD; t += kStThreads) {
            float acc = 0.0f;
#pragma unroll
            for (int w = 0; w < kStWarps; w++) acc += wpart[w * (HD + 2) + 2 + t] * sf[w];
            po[t] = acc;
        }
        if (tid == 0) *reinterpret_cast<float2 *>(pml) = make_float2(sf[kStWarps + 1], sf[kStWarps]);
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            s_last[0] = atomicAdd(head_cnt + h, 1u) == S - 1;
        }
        __syncthreads();
        if (s_last[0]) {  // the last split of head h merges the head's splits
            __threadfence();
            const float *ho = a.part + (size_t)h * S * HD;
            const float *hml = a.part + (size_t)a.g.n_heads * S * HD + 2 * (size_t)h * S;
            for (uint32_t t = tid; t < HD; t += kStThreads) {
                float GM = -INFINITY;
                for (uint32_t q = 0; q < S; q++) GM = fmaxf(GM, __ldcg(hml + 2 * q));
                float GL = 0.0f, acc = 0.0f;
                for (uint32_t q = 0; q < S; q++) {
                    const float mk = __ldcg(hml + 2 * q);
                    if (mk != -INFINITY) {
                        const float f = expf(mk - GM);
                        GL += __ldcg(hml + 2 * q + 1) * f;
                        acc += __ldcg(ho + (size_t)q * HD + t) * f;
                    }
                }
                hq[t] = acc / GL;
            }
            __syncthreads();
            for (uint32_t b = warp; b < (uint32_t)HD / 32; b += kStWarps)
                qact_store_block(a.att, (int)nq, (int)(h * HD / 32 + b), hq[32 * b + lane], lane);
            if (tid == 0) head_cnt[h] = 0;
        }
        __syncthreads();
    }
}

// Phase G's rows: gate/up tile rows [0, 2 np) against Xx, then h = act(g) * u
// per pair (k_moe_decode's orders).
template <uint32_t GT>
__device__ __noinline__ void st_gate_up(const StackArgs &a, const uint8_t *W, float *part, XS Xx, uint64_t *bch,
                                        uint32_t par, uint32_t np, float *s_h) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t cpr = st_chunks64(a.d);
    const uint32_t gstride = 2 * a.maxpairs + 1;
    const uint32_t lpr = min(cpr, 32u), rps = 32 / lpr;
    const uint32_t sub = lane / lpr, nrows = 2 * np;
    if (sub < rps) {
        for (uint32_t cg = 0; cg < cpr; cg += lpr) {
            const uint32_t n = min(lpr, cpr - cg);
            if ((uint32_t)lane % lpr >= n) continue;
            const uint32_t cb = cg + spread_chunk((uint32_t)lane % lpr, n);
            XChunk xc;
            xchunk_load(Xx, 0, (int)cb, xc);
            const uint32_t step = kStWarps * rps;
            for (uint32_t r = warp * rps + sub; r < nrows; r += 2 * step) {
                const uint32_t rb = r + step < nrows ? r + step : r;
                const bool ok = st_wait(&bch[r / (2 * kStChunk)], par, a.dev_err) &
                                st_wait(&bch[rb / (2 * kStChunk)], par, a.dev_err);
                float ya = 0.0f, yb = 0.0f;
                if (ok) {
                    ya = dot64<GT>(W + (size_t)r * a.gpitch, (int)cb, (int)a.gnb, xc);
                    yb = dot64<GT>(W + (size_t)rb * a.gpitch, (int)cb, (int)a.gnb, xc);
                }
                part[cb * gstride + r] = ya;
                part[cb * gstride + rb] = yb;
            }
        }
    }
    __syncthreads();
    for (uint32_t lp = tid; lp < np; lp += kStThreads) {  // chunk partials summed in column order
        const uint32_t rg = 2 * kStChunk * (lp / kStChunk) + lp % kStChunk;
        const float *pg = part + rg, *pu = pg + kStChunk;
        float g = 0.0f, u = 0.0f;
        for (uint32_t i = 0; i < cpr; i++) {
            g += pg[i * gstride];
            u += pu[i * gstride];
        }
        s_h[lp] = act_apply(a.act, g) * u;
    }
}

// Phase D's rows: warps [s*wps, (s+1)*wps) take slot s; a lane owns one
// 64-column chunk of that slot's h; then y[s][r] from the chunk partials.
template <uint32_t DT>
__device__ __noinline__ void st_down(const StackArgs &a, const uint8_t *DN, uint8_t *XSr, float *part, float *s_y,
                                     uint64_t *bdn, uint32_t par, uint32_t nor, bool hok) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t cpr = st_chunks64(a.F);
    const uint32_t dstride = a.k * a.maxo + 1;
    const uint32_t lpr = min(cpr, 32u), rps = 32 / lpr;
    const uint32_t sub = lane / lpr;
    const uint32_t wps = max(1u, (uint32_t)kStWarps / a.k);
    const uint32_t s = warp / wps, ws = warp % wps;
    if (s < a.k && sub < rps && nor) {
        const bool ok = st_wait(&bdn[s], par, a.dev_err) && hok;
        const XS Xh = xs_carve(XSr + (size_t)s * a.img, 1, (int)a.di);
        for (uint32_t cg = 0; cg < cpr; cg += lpr) {
            const uint32_t n = min(lpr, cpr - cg);
            if ((uint32_t)lane % lpr >= n) continue;
            const uint32_t cb = cg + spread_chunk((uint32_t)lane % lpr, n);
            XChunk xc;
            xchunk_load(Xh, 0, (int)cb, xc);
            const uint32_t step = wps * rps;
            for (uint32_t r = ws * rps + sub; r < nor; r += 2 * step) {
                const uint32_t rb = r + step < nor ? r + step : r;
                const uint32_t ta = s * a.maxo + r, tb = s * a.maxo + rb;
                float ya = 0.0f, yb = 0.0f;
                if (ok) {
                    ya = dot64<DT>(DN + (size_t)ta * a.dpitch, (int)cb, (int)a.dnb, xc);
                    yb = dot64<DT>(DN + (size_t)tb * a.dpitch, (int)cb, (int)a.dnb, xc);
                }
                part[cb * dstride + ta] = ya;
                part[cb * dstride + tb] = yb;
            }
        }
    }
    __syncthreads();
    for (uint32_t w = tid; w < a.k * nor; w += kStThreads) {  // y[s][r]: chunk partials in column order
        const uint32_t s2 = w / nor, r = w - s2 * nor;
        const float *pp = part + s2 * a.maxo + r;
        float y = 0.0f;
        for (uint32_t i = 0; i < cpr; i++) y += pp[i * dstride];
        s_y[s2 * a.maxo + r] = y;
    }
}

// Thread 0: copy a layer's Q/K/V rows [q0, q0 + nqr), attn_norm and the Q/K
// norms into shared memory, all on barrier bq.
LT_DEVINL void st_issue_q(const StackArgs &a, const StLayout &L, uint8_t *smem, const StackLayerDev &Ly, uint32_t q0,
                          uint32_t nqr, uint64_t *bq) {
    const uint32_t hb = a.g.hd * 4;
    const uint32_t bytes = (uint32_t)(nqr * a.qpitch) + a.d * 4 + (Ly.q_norm ? hb : 0) + (Ly.k_norm ? hb : 0);
    mbar_arrive_expect_tx(bq, bytes);
    tma_load_1d(smem + L.w, Ly.wqkv + (uint64_t)q0 * a.qpitch, (uint32_t)(nqr * a.qpitch), bq);
    tma_load_1d(smem + L.an, Ly.attn_norm, a.d * 4, bq);
    if (Ly.q_norm) tma_load_1d(smem + L.qn, Ly.q_norm, hb, bq);
    if (Ly.k_norm) tma_load_1d(smem + L.kn, Ly.k_norm, hb, bq);
}

template <uint32_t QT, uint32_t OT, int HD, uint32_t GT, uint32_t DT>
__global__ void __launch_bounds__(kStThreads, 1) k_stack(const __grid_constant__ StackArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t G = gridDim.x, c = blockIdx.x;
    const StLayout L = st_layout(a);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *bq = bars, *bo = bars + 1, *brt = bars + 2, *bh = bars + 3;
    uint64_t *bdn = bars + 8, *bch = bars + 8 + kStMaxSlots;
    float *red = reinterpret_cast<float *>(smem + L.misc);                 // [16]
    uint32_t *s_sel = reinterpret_cast<uint32_t *>(smem + L.misc + 64);    // [16]
    float *s_w = reinterpret_cast<float *>(smem + L.misc + 128);           // [16]
    float *s_stat = reinterpret_cast<float *>(smem + L.misc + 192);        // rms, max, expsum
    float *s_ss = reinterpret_cast<float *>(smem + L.misc + 224);          // [4]
    uint64_t *s_launch = reinterpret_cast<uint64_t *>(smem + L.misc + 256);
    int *s_last = reinterpret_cast<int *>(smem + L.misc + 264);
    float *s_lg = reinterpret_cast<float *>(smem + L.lg);
    uint64_t *s_key = reinterpret_cast<uint64_t *>(smem + L.keys);
    uint32_t *s_cnt = reinterpret_cast<uint32_t *>(smem + L.cnt);
    uint8_t *W = smem + L.w, *DN = smem + L.dn;
    float *RT = reinterpret_cast<float *>(smem + L.rt);
    uint8_t *XSr = smem + L.xs;
    float *XF = reinterpret_cast<float *>(smem + L.xf);
    float *s_h = reinterpret_cast<float *>(smem + L.hs);
    float *s_y = reinterpret_cast<float *>(smem + L.ys);
    float *xres = reinterpret_cast<float *>(smem + L.xres);
    const StackLayerDev *s_lay = reinterpret_cast<const StackLayerDev *>(smem + L.lay);
    float *s_bias = reinterpret_cast<float *>(smem + L.bias);
    float *s_an = reinterpret_cast<float *>(smem + L.an), *s_fn = reinterpret_cast<float *>(smem + L.fn);
    float *s_qn = reinterpret_cast<float *>(smem + L.qn), *s_kn = reinterpret_cast<float *>(smem + L.kn);
    uint64_t *blay = bars + 4;
    unsigned long long *ctr_e = reinterpret_cast<unsigned long long *>(a.sync + kStEpoch);
    unsigned long long *ctr_b = reinterpret_cast<unsigned long long *>(a.sync + kStBar);
    unsigned long long *lslots = reinterpret_cast<unsigned long long *>(a.sync + kStLogits);
    uint32_t *head_cnt = reinterpret_cast<uint32_t *>(a.sync + kStHeadCnt);
    const uint32_t d = a.d;

    // this CTA's shares: Q/K/V rows [q0, q1); wo, down and residual rows
    // [o0, o1); gate/up pairs [p0, p1) of the k*F (slot, row) pairs in whole
    // 16-pair units
    const uint32_t q0 = (uint32_t)((uint64_t)c * a.qrows / G), q1 = (uint32_t)((uint64_t)(c + 1) * a.qrows / G);
    const uint32_t o0 = (uint32_t)((uint64_t)c * d / G), o1 = (uint32_t)((uint64_t)(c + 1) * d / G);
    const uint32_t nqr = q1 - q0, nor = o1 - o0;
    const uint32_t nunits = a.k * a.F / kStUnit;
    const uint32_t p0 = kStUnit * (uint32_t)((uint64_t)c * nunits / G);
    const uint32_t p1 = kStUnit * (uint32_t)((uint64_t)(c + 1) * nunits / G);
    const uint32_t np = p1 - p0, nchunks = np / kStChunk;
    const bool has_e = !a.dense && c < a.E;

    if (tid == 0) {
        mbar_init(bq, 1);
        mbar_init(bo, 1);
        mbar_init(brt, 1);
        mbar_init(bh, 1);
        mbar_init(blay, 1);
        for (uint32_t s = 0; s < a.k; s++) mbar_init(&bdn[s], 1);
        for (uint32_t j = 0; j < nchunks; j++) mbar_init(&bch[j], 1);
        fence_barrier_init();
        *s_launch = atomicAdd(ctr_e, 1ull) / G;  // every CTA adds 1 per launch
        // the layer table, then the first layer's static tiles
        const uint32_t lay_bytes = a.n_layers * (uint32_t)sizeof(StackLayerDev);
        mbar_arrive_expect_tx(blay, lay_bytes);
        tma_load_1d(smem + L.lay, a.layers, lay_bytes, blay);
        const StackLayerDev &L0 = a.layers[0];
        st_issue_q(a, L, smem, L0, q0, nqr, bq);
        if (has_e) {
            mbar_arrive_expect_tx(brt, d * 4);
            tma_load_1d(RT, L0.router + (size_t)c * d, d * 4, brt);
        }
        st_prefetch_rows(L0.wo, a.opitch, o0, nor);
    }
    if (tid < nqr) s_bias[tid] = a.layers[0].bias ? __ldg(a.layers[0].bias + q0 + tid) : 0.0f;
    if (tid == 0) st_wait(blay, 0, a.dev_err);
    __syncthreads();
    const uint64_t launch = *s_launch;
    uint32_t nb = 0;  // grid hand-offs passed in this launch
    auto gsync = [&]() {
        st_grid_sync(ctr_b, G, (uint64_t)launch * a.nbar + nb + 1, a.dev_err);
        nb++;
    };
    pdl_wait();
    const uint32_t pos = __ldcg(a.pos);
    const uint32_t seq = pos + 1, win = a.g.window ? min(seq, a.g.window) : seq, first = seq - win;
    const uint32_t S = min(a.splits, max(1u, (win + kStSplitPositions - 1) / kStSplitPositions));

    for (uint32_t l = 0; l < a.n_layers; l++) {
        const StackLayerDev *Ly = s_lay + l;
        const uint32_t par = l & 1;
        const bool more = l + 1 < a.n_layers;

        // ── Q ────────────────────────────────────────────────────────────────
        ST_MARK(0);
        if (tid == 0 && c < 2 && win > 1) {  // this layer's cached K (CTA 0) / V (CTA 1) rows into L2 for phase A
            const size_t row = (size_t)a.nkv * (a.g.kv_f16 ? 2 : 4);
            const uint8_t *base = static_cast<const uint8_t *>(c == 0 ? Ly->kc : Ly->vc);
            const uint32_t s0 = first % a.g.cap, n = win - 1, n0 = min(n, a.g.cap - s0);
            st_prefetch_rows(base, row, s0, n0);
            if (n > n0) st_prefetch_rows(base, row, 0, n - n0);
        }
        ab_load(XF, a.x, d);
        __syncthreads();
        ST_MARK(12);
        for (uint32_t r = tid; r < nor; r += kStThreads) xres[r] = XF[o0 + r];
        const bool qok = nqr && st_wait(bq, par, a.dev_err);  // the Q/K/V rows and the layer's norm weights
        {
            float ss = 0.0f;
            for (uint32_t i = tid; i < d; i += kStThreads) ss += XF[i] * XF[i];
            ss = ab_block_sum(ss, red);
            const float rms_inv = 1.0f / sqrtf(ss / (float)d + a.eps);
            for (uint32_t i = tid; i < d; i += kStThreads) XF[i] = XF[i] * rms_inv * s_an[i];
        }
        __syncthreads();
        ST_MARK(13);
        {
            const XS Xx = xs_carve(XSr, 1, (int)st_items(d));
            ab_quantise(Xx, XF, d, warp, lane);
            __syncthreads();
            ST_MARK(14);
            ST_MARK(15);
            if (qok) st_rows<QT>(W, a.qpitch, nqr, d, a.qnb, Xx, XF);
        }
        __syncthreads();
        ST_MARK(16);
        {
            const bool bias = Ly->bias != nullptr;
            for (uint32_t r = tid; r < nqr; r += kStThreads) a.qkv[q0 + r] = bias ? __fadd_rn(XF[r], s_bias[r]) : XF[r];
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // W is copied over next
        ST_MARK(1);
        gsync();
        ST_MARK(2);

        // ── A ────────────────────────────────────────────────────────────────
        if (tid == 0) {
            mbar_arrive_expect_tx(bo, (uint32_t)(nor * a.opitch) + d * 4);
            tma_load_1d(W, Ly->wo + (uint64_t)o0 * a.opitch, (uint32_t)(nor * a.opitch), bo);
            tma_load_1d(s_fn, Ly->ffn_norm, d * 4, bo);
        }
        st_attention<HD>(a, Ly->q_norm ? s_qn : nullptr, Ly->k_norm ? s_kn : nullptr, Ly->kc, Ly->vc, XF, red, s_last,
                         head_cnt, pos, S, win, first);
        ST_MARK(3);
        gsync();
        ST_MARK(4);

        // ── O ────────────────────────────────────────────────────────────────
        {
            const XS Xa = xs_carve(XSr, 1, (int)st_items(a.nq));
            ab_load_qact(Xa, a.att, a.nq);
            __syncthreads();
            ST_MARK(28);
            const bool ok = st_wait(bo, par, a.dev_err);  // the wo rows and ffn_norm
            ST_MARK(29);
            if (ok) st_rows<OT>(W, a.opitch, nor, a.nq, a.onb, Xa, XF);
        }
        __syncthreads();
        for (uint32_t r = tid; r < nor; r += kStThreads) {
            const float v = __fadd_rn(xres[r], XF[r]);
            a.x[o0 + r] = v;
            xres[r] = v;  // x' rows: the FFN block's residual
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // W takes the expert rows next
        ST_MARK(5);
        gsync();
        ST_MARK(6);

        // ── R ────────────────────────────────────────────────────────────────
        ab_load(XF, a.x, d);
        __syncthreads();
        ST_MARK(17);
        {  // rmsnorm(out, x, w, eps) with k_moe_decode's reduction order
            float ss = 0.0f;
            if (tid < kStNormThreads)
                for (uint32_t i = tid; i < d; i += kStNormThreads) ss += XF[i] * XF[i];
            ss = warp_sum(ss);
            if (lane == 0 && warp < kStNormThreads / 32) s_ss[warp] = ss;
            __syncthreads();
            if (tid == 0) {
                float t = 0.0f;
                for (int w = 0; w < kStNormThreads / 32; w++) t += s_ss[w];
                s_stat[0] = 1.0f / sqrtf(t / (float)d + a.eps);
            }
            __syncthreads();
            const float rms = s_stat[0];
            for (uint32_t i = tid; i < d; i += kStThreads) XF[i] = XF[i] * rms * s_fn[i];
        }
        __syncthreads();
        ST_MARK(18);
        const uint32_t tag = (uint32_t)(launch * 64 + l + 1);
        {
            const XS Xx = xs_carve(XSr, 1, (int)st_items(d));
            if (has_e && warp == 0) {
                st_wait(brt, par, a.dev_err);
                const float v = router_logit_sm(RT, XF, d, lane);
                if (lane == 0) st_relaxed_u64(lslots + c, ((uint64_t)tag << 32) | __float_as_uint(v));
            } else {
                const uint32_t w0 = has_e ? 1 : 0;
                for (uint32_t b = warp - w0; b < d / 32; b += kStWarps - w0)
                    qact_block_to_xs(Xx, 0, (int)b, XF[32 * b + lane], lane);
            }
        }
        ST_MARK(19);
        if (!a.dense && (uint32_t)tid < a.E) {  // poll expert tid's logit until it carries this layer's tag
            uint64_t v = ld_relaxed_u64(lslots + tid);
            if ((uint32_t)(v >> 32) != tag) {
                const uint64_t t0 = globaltimer_ns();
                for (;;) {
                    v = ld_relaxed_u64(lslots + tid);
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
        if (tid == 0) {
            s_key[a.E] = 0;
            if (a.dense) s_sel[0] = 0;
        }
        __syncthreads();
        ST_MARK(20);
        if (!a.dense) {
            if (warp == kStWarps - 1) {
                float mxv, es;
                router_softmax_stats(s_lg, a.E, lane, mxv, es);
                if (lane == 0) {
                    s_stat[1] = mxv;
                    s_stat[2] = es;
                }
            }
            router_rank_keys_split(s_key, a.E, a.k, s_sel, min(4u, (uint32_t)(kStThreads - 32) / a.E), s_cnt, tid);
        }
        __syncthreads();
        ST_MARK(7);

        // ── G ────────────────────────────────────────────────────────────────
        if (warp == 0) {  // one TMA chunk per lane: [8 gate rows][8 up rows] of pairs p0 + 8j..
            const uint8_t *gate = Ly->gate, *upt = Ly->up;
            for (uint32_t j = lane; j < nchunks; j += 32) {
                const uint32_t qq = p0 + j * kStChunk;
                const uint32_t s = qq / a.F, f0 = qq - s * a.F;
                const uint32_t e = min(s_sel[s], a.E - 1);
                const uint32_t bytes = (uint32_t)(kStChunk * a.gpitch);
                uint64_t grow, urow;
                const uint8_t *ub;
                if (upt) {
                    grow = (uint64_t)e * a.F + f0;
                    urow = grow;
                    ub = upt;
                } else {  // fused: gate rows [0,F), up rows [F,2F) (gemma4/forward.zig:469-471)
                    grow = (uint64_t)e * 2 * a.F + f0;
                    urow = grow + a.F;
                    ub = gate;
                }
                uint8_t *dst = W + (size_t)2 * j * kStChunk * a.gpitch;
                mbar_arrive_expect_tx(&bch[j], 2 * bytes);
                tma_load_1d(dst, gate + grow * a.gpitch, bytes, &bch[j]);
                tma_load_1d(dst + bytes, ub + urow * a.gpitch, bytes, &bch[j]);
            }
        } else if (warp == 1) {  // down rows [o0, o1) of each slot's expert
            if ((uint32_t)lane < a.k && nor) {
                const uint32_t e = min(s_sel[lane], a.E - 1);
                const uint32_t bytes = (uint32_t)(nor * a.dpitch);
                mbar_arrive_expect_tx(&bdn[lane], bytes);
                tma_load_1d(DN + (size_t)lane * a.maxo * a.dpitch, Ly->down + ((uint64_t)e * d + o0) * a.dpitch, bytes,
                            &bdn[lane]);
            }
        } else if (warp == 2 && lane == 0) {
            if (a.dense)
                s_w[0] = 1.0f;
            else
                router_weights(s_lg, s_sel, a.k, s_stat[1], s_stat[2], a.norm_topk, nullptr, s_w);
        }
        ST_MARK(22);
        st_gate_up<GT>(a, W, XF, xs_carve(XSr, 1, (int)st_items(d)), bch, par, np, s_h);
        __syncthreads();
        ST_MARK(23);
        // quantise this CTA's h values into their slots' images (32-blocks; a block may be half this CTA's)
        for (uint32_t b = p0 / 32 + warp; b * 32 < p1; b += kStWarps) {
            const uint32_t qq = 32 * b + lane;
            const bool own = qq >= p0 && qq < p1;
            const uint32_t s = (32 * b) / a.F, bs = (32 * b - s * a.F) / 32;
            const XS Xs = xs_carve(a.himg + (size_t)s * a.img, 1, (int)a.di);
            qact_block_to_xs(Xs, 0, (int)bs, own ? s_h[qq - p0] : 0.0f, lane, own);
        }
        ST_MARK(24);
        fence_proxy_async_global();  // the images are read by TMA after the hand-off
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // W, RT and XS are copied over next
        ST_MARK(8);
        gsync();
        ST_MARK(9);

        // ── D ────────────────────────────────────────────────────────────────
        if (tid == 0) {
            fence_proxy_async_global();
            mbar_arrive_expect_tx(bh, a.k * a.img);
            for (uint32_t s = 0; s < a.k; s++)
                tma_load_1d(XSr + (size_t)s * a.img, a.himg + (size_t)s * a.img, a.img, bh);
        }
        if (more && tid < nqr) s_bias[tid] = Ly[1].bias ? __ldg(Ly[1].bias + q0 + tid) : 0.0f;
        const bool hok = st_wait(bh, par, a.dev_err);
        // the next layer's Q/K/V rows, norm weights and router row, once the
        // slot images are in (queued behind them they would delay the images)
        if (tid == 0 && more) {
            st_issue_q(a, L, smem, Ly[1], q0, nqr, bq);
            if (has_e) {
                mbar_arrive_expect_tx(brt, d * 4);
                tma_load_1d(RT, Ly[1].router + (size_t)c * d, d * 4, brt);
            }
        }
        ST_MARK(25);
        st_down<DT>(a, DN, XSr, XF, s_y, bdn, par, nor, hok);
        __syncthreads();
        ST_MARK(26);
        for (uint32_t r = tid; r < nor; r += kStThreads) {
            float o = 0.0f;  // moe_buf is zeroed, then += scale * down, slot by slot
            for (uint32_t s = 0; s < a.k; s++) o += s_w[s] * s_y[s * a.maxo + r];
            a.x[o0 + r] = xres[r] + o;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // DN and XS are copied over next
        if (!more) pdl_launch_dependents();
        ST_MARK(10);
        gsync();
        ST_MARK(11);
    }
}

namespace {

// Global scratch of a plan: qkv rows, attention split partials, the quantised
// attention row, the slot images, then the sync block (each 256-aligned).
struct StScratch {
    size_t qkv, part, att, himg, sync, total;
};

StScratch st_scratch(const StackParams &p, uint32_t splits) {
    const AttnGeom &g = p.g;
    const uint32_t nq = g.n_heads * g.hd, qrows = nq + 2 * g.n_kv * g.hd;
    StScratch s;
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off += (b + 255) & ~(size_t)255;
        return o;
    };
    s.qkv = take((size_t)qrows * 4);
    s.part = take((size_t)g.n_heads * splits * (g.hd + 2) * 4);
    s.att = take(qact_pitch(nq));
    s.himg = take((size_t)p.k * xs_bytes(1, (int)st_items(p.F)));
    s.sync = take(kStackSyncBytes);
    s.total = off;
    return s;
}

}  // namespace

// The kernel's arguments without the per-call pointers: the one place both the
// plan (shared-memory size) and the launch take them from.  false: a shape the
// kernel does not take.
static bool st_args(const StackParams &p, int num_sms, StackArgs &a) {
    const AttnGeom &g = p.g;
    const uint32_t G = (uint32_t)num_sms;
    if (p.n_layers == 0 || p.n_layers > 63 || num_sms <= 0 || (uint32_t)num_sms > kStMaxCtas) return false;
    if (g.hd != 64 && g.hd != 128) return false;
    if (g.window != 0 || g.v_norm != 0 || g.n_kv == 0 || g.n_heads % g.n_kv != 0) return false;
    if (p.d % 256 != 0 && p.qtype != T_Q8_0) return false;
    if (p.d % 32 != 0 || p.F % 32 != 0 || p.d > 8192) return false;
    const uint32_t nq = g.n_heads * g.hd, nkv = g.n_kv * g.hd, qrows = nq + 2 * nkv;
    if (qrows < G || p.d < G || nq > 16384 || g.n_heads > 1024) return false;
    if (p.qtype != T_Q8_0 || p.otype != T_Q8_0) return false;
    if (p.dense) {
        if (p.gtype != T_Q8_0 || p.dtype != T_Q8_0 || p.k != 1 || p.E != 1) return false;
    } else {
        if (p.gtype != T_Q4_K || p.dtype != T_Q4_K || p.E > G || p.E > (uint32_t)kRouterMaxE) return false;
        if (p.k == 0 || p.k > kStMaxSlots || p.k > p.E) return false;
    }
    const uint32_t nunits = p.k * p.F / kStUnit;
    if (nunits < G || (p.k * p.F) % kStUnit) return false;
    a = StackArgs{};
    a.g = g;
    a.d = p.d;
    a.nq = nq;
    a.nkv = nkv;
    a.qrows = qrows;
    a.qpitch = p.qpitch;
    a.opitch = p.opitch;
    a.qnb = p.d / 32;
    a.onb = nq / 32;
    a.E = p.E;
    a.k = p.k;
    a.F = p.F;
    a.norm_topk = p.norm_topk;
    a.act = p.act;
    a.dense = p.dense;
    a.gpitch = p.gpitch;
    a.dpitch = p.dpitch;
    a.gnb = p.d / 32;
    a.dnb = p.F / 32;
    a.di = st_items(p.F);
    a.img = (uint32_t)xs_bytes(1, (int)a.di);
    a.eps = p.eps;
    a.n_layers = p.n_layers;
    a.nbar = 5 * p.n_layers;
    a.splits = max(1u, min(kStMaxSplits, G / g.n_heads));
    a.maxq = (qrows + G - 1) / G;
    a.maxo = (p.d + G - 1) / G;
    a.maxpairs = kStUnit * ((nunits + G - 1) / G);
    if (a.maxpairs / kStChunk > kStMaxChunks) return false;
    return st_layout(a).total <= kDecodeSmemLimit;
}

bool stack_plan(const StackParams &p, int num_sms, size_t *smem_out, size_t *scratch_bytes, size_t *sync_offset) {
    StackArgs a;
    if (!st_args(p, num_sms, a)) return false;
    if (smem_out) *smem_out = st_layout(a).total;
    if (scratch_bytes) *scratch_bytes = st_scratch(p, a.splits).total;
    if (sync_offset) *sync_offset = st_scratch(p, a.splits).sync;
    return true;
}

template <int HD, uint32_t GT, uint32_t DT>
static cudaError_t launch_stack_t(const LaunchCfg &c, const StackArgs &a, size_t smem) {
    return launch_k(c, "stack", k_stack<T_Q8_0, T_Q8_0, HD, GT, DT>, dim3((unsigned)c.num_sms), dim3(kStThreads),
                    smem, a);
}

#ifdef LT_STACK_TRACE
// Tuning builds only (not declared in the public header): copy the trace out.
extern "C" int lt_stack_trace_copy(void *dst, size_t bytes) {
    return (int)cudaMemcpyFromSymbol(dst, g_stack_trace, bytes);
}
#endif

cudaError_t launch_stack(const LaunchCfg &c, const StackParams &p, const void *dev_layers, float *x,
                         const uint32_t *pos, uint8_t *scratch) {
    StackArgs a;
    if (!st_args(p, c.num_sms, a)) return cudaErrorInvalidValue;
    const size_t smem = st_layout(a).total;  // the kernel carves exactly this layout from these arguments
    a.layers = static_cast<const StackLayerDev *>(dev_layers);
    a.x = x;
    a.pos = pos;
    const StScratch sc = st_scratch(p, a.splits);
    a.qkv = reinterpret_cast<float *>(scratch + sc.qkv);
    a.part = reinterpret_cast<float *>(scratch + sc.part);
    a.att = scratch + sc.att;
    a.himg = scratch + sc.himg;
    a.sync = scratch + sc.sync;
    a.dev_err = c.dev_err;
    if (p.dense) {
        if (p.g.hd == 64) return launch_stack_t<64, T_Q8_0, T_Q8_0>(c, a, smem);
        return launch_stack_t<128, T_Q8_0, T_Q8_0>(c, a, smem);
    }
    if (p.g.hd == 64) return launch_stack_t<64, T_Q4_K, T_Q4_K>(c, a, smem);
    return launch_stack_t<128, T_Q4_K, T_Q4_K>(c, a, smem);
}

}  // namespace lt
