// lt_internal.h — kernel launchers shared between the kernel files and the
// C ABI in lt_api.cu.  Not part of the public interface.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

struct lt_ctx;

namespace lt {

// The context's device and its current stream (lt_api.cu), for entry points
// implemented in other files.
int ctx_device(const lt_ctx *ctx);
cudaStream_t ctx_stream(const lt_ctx *ctx);

// A weight matrix as the kernels see it: GGUF rows at a 16-byte pitch.
struct DevMat {
    const uint8_t *data;
    uint32_t type;
    uint64_t rows;       // rows per expert (or all rows for 2-D)
    uint64_t cols;
    uint64_t row_bytes;
    uint64_t pitch;
    uint32_t n_experts;  // 0 for 2-D
};

// Routing plan built on the device for the grouped expert kernels.
struct MoePlan {
    uint32_t *n_active;   // [1]    experts with at least one token
    uint32_t *act_e;      // [E]    active expert ids, ascending
    uint32_t *act_off;    // [E]    first position of each active expert
    uint32_t *act_cnt;    // [E]    number of (token, slot) pairs routed to it
    uint32_t *pos_pair;   // [T*k]  position -> pair index (token*k + slot)
    uint32_t *pair_pos;   // [T*k]  pair index -> position
};

// Per-label kernel timing with CUDA events (the reference's GpuProfiler,
// src/gpu/context.zig:34-268).  Only active when enabled on the context.
struct Profiler {
    struct Rec {
        const char *label;
        cudaEvent_t a, b;
    };
    struct Agg {
        const char *label;
        uint64_t count;
        double total_ms, min_ms, max_ms;
    };
    bool on = false;
    Rec pending[4096];
    int n_pending = 0;
    cudaEvent_t pool[8192];
    int n_pool = 0;
    Agg agg[64];
    int n_agg = 0;

    cudaEvent_t get_event();
    void begin(const char *label, cudaStream_t s, Rec &r);
    void end(Rec &r, cudaStream_t s);
    cudaError_t flush();  // waits for pending events and accumulates
    void reset();
    void destroy();
};

struct LaunchCfg {
    cudaStream_t stream;
    bool pdl;        // launch with programmatic stream serialization
    int *dev_err;    // device error word (DEV_ERR_*)
    int num_sms;
    Profiler *prof;  // nullptr or disabled: no timing
};

constexpr int kRouterMaxE = 256;  // experts per router (top-k runs in one warp)

bool type_supported(uint32_t t);
uint64_t row_bytes_of(uint32_t t, uint64_t cols);
uint32_t block_elems_of(uint32_t t);

cudaError_t launch_dequant(const LaunchCfg &c, const DevMat &m, uint64_t row0, uint64_t nrows,
                           float *out);
cudaError_t launch_quantize_q8_1(const LaunchCfg &c, const float *x, uint64_t n, int x4, uint8_t *out);
cudaError_t launch_dequant_q8_1(const LaunchCfg &c, const uint8_t *q, uint64_t n, int x4, float *out);
cudaError_t launch_rmsnorm(const LaunchCfg &c, const float *x, const float *w, float eps, uint32_t n,
                           uint32_t ntok, float *y);
cudaError_t launch_softmax(const LaunchCfg &c, float *x, uint32_t n, uint32_t ntok);
// tokens != nullptr (ntok == 1): greedy step of a decode graph -- with
// p = *pos, tokens[p + 1] = argmax when p + 1 >= *n_prompt, then *pos = p + 1.
cudaError_t launch_argmax(const LaunchCfg &c, const float *x, uint32_t n, uint32_t ntok,
                          uint32_t *idx, float *scratch_val, uint32_t *scratch_idx,
                          uint32_t *counters, uint32_t *tokens = nullptr, uint32_t *pos = nullptr,
                          const uint32_t *n_prompt = nullptr);
cudaError_t launch_fill_f32(cudaStream_t s, float *p, size_t n, float v);
// sample.zig:27-183 as a decode-step op (lt_sample.cu); probs: n floats of scratch.
cudaError_t launch_sample(const LaunchCfg &c, const float *logits, uint32_t n, float temperature, uint32_t top_k,
                          float top_p, unsigned long long *rng, uint32_t *tokens, uint32_t *pos,
                          const uint32_t *n_prompt, float *probs);
// Gemma 4 layer glue (lt_glue.cu), ntok rows of n values.
cudaError_t launch_scale(const LaunchCfg &c, float *x, uint32_t n, uint32_t ntok, float s);
cudaError_t launch_add_rmsnorm(const LaunchCfg &c, const float *y, const float *w, float eps, uint32_t n,
                               uint32_t ntok, float *x);
cudaError_t launch_norm_pair(const LaunchCfg &c, const float *x, const float *w, const float *g, float gs, float eps,
                             uint32_t n, uint32_t ntok, float *a, float *b);
cudaError_t launch_ffn_tail(const LaunchCfg &c, const float *f, const float *w1, float *m, const float *w2,
                            const float *w, float los, float eps, uint32_t n, uint32_t ntok, float *x);
cudaError_t launch_softcap(const LaunchCfg &c, float *x, size_t n, float cap);
cudaError_t launch_selftest_wait(const LaunchCfg &c, int kind, uint64_t limit_ns);
// out = dequantised row tokens[*pos] of m (embedLookup); rows >= m.rows set
// DEV_ERR_BAD_INDEX and read row 0.
cudaError_t launch_embed(const LaunchCfg &c, const DevMat &m, const uint32_t *tokens, const uint32_t *pos,
                         float *out);

// Decode attention (lt_attn.cu).  KV cache per layer: [cap][n_kv * hd] f32
// for K and for V; position slot = pos % cap.
struct AttnGeom {
    uint32_t n_heads, n_kv, hd;
    uint32_t rope_neox;  // 0: consecutive pairs (rope.zig:14), 1: halves (rope.zig:56)
    float theta, eps, scale;
    uint32_t cap;
    uint32_t window;  // 0: every cached position; else the last `window`
    uint32_t v_norm;  // 1: RMSNorm without weights on each V head before caching (gemma4/forward.zig:269)
    uint32_t kv_f16;  // 1: caches hold f16 elements, else f32
};
uint32_t attn_splits(const AttnGeom &g, int num_sms);
size_t attn_scratch_floats(const AttnGeom &g, int num_sms);
cudaError_t launch_attn_prep(const LaunchCfg &c, const AttnGeom &g, float *qkv, const float *q_norm,
                             const float *k_norm, const uint32_t *pos, void *kc, void *vc);
cudaError_t launch_attn_decode(const LaunchCfg &c, const AttnGeom &g, const float *q, const void *kc,
                               const void *vc, const uint32_t *pos, float *out, float *part, uint32_t *counters);

// The attention half of a decoder layer for one token in one persistent
// kernel (lt_attn_block.cu): out = x + wo . attention(rope(norm(W_qkv .
// rmsnorm(x) + bias))), KV append included.  Grid = num_sms, all resident.
struct AttnBlockParams {
    AttnGeom g;
    uint32_t d;
    const float *x, *norm_w;
    float eps;
    // Q/K/V rows: one stacked tensor [nq + 2 nkv][d] (nseg 1), or wq, wk and wv
    // (nseg 3), or wq and wk with V = the raw K head (nseg 2, v_is_k)
    DevMat seg[3];
    uint32_t nseg = 1;
    int v_is_k = 0;
    DevMat wo;
    const float *bias, *q_norm, *k_norm;
    const float *post_norm = nullptr;  // out = x + rmsnorm(wo . att) * post_norm instead of x + wo . att
    // non-null tail_f: x is first replaced by the previous layer's FFN tail of it (launch_ffn_tail's arguments)
    const float *tail_f = nullptr, *tail_w1 = nullptr, *tail_m = nullptr, *tail_w2 = nullptr, *tail_w = nullptr;
    float tail_los = 1.0f, tail_eps = 0.0f;
    const uint32_t *pos;
    void *kc, *vc;  // f32 or f16 elements (AttnGeom::kv_f16)
    float *out;            // may alias x
    float *scratch;        // the floats attn_block_plan gives
    uint8_t *sync;         // kAttnSyncBytes zero-initialised, this kernel only
    const uint8_t *pf[2];  // optional L2 prefetch ranges (the next kernel's weights)
    uint64_t pf_bytes[2];
};
constexpr size_t kAttnSyncBytes = 8192;  // counters, one merge counter per head (<= 1024), hand-off counters
// Whether the persistent kernel takes this shape (and fits in shared memory);
// its global scratch in floats.
bool attn_block_plan(const AttnBlockParams &p, int num_sms, size_t *scratch_floats);
cudaError_t launch_attn_block(const LaunchCfg &c, const AttnBlockParams &p);

// Bytes of one quantised activation row (lt_qact.cuh) of `cols` values.
size_t qact_row_pitch(uint64_t cols);
// nrows f32 rows of `cols` -> quantised activation rows at q (pitch qpitch).
cudaError_t launch_quantize(const LaunchCfg &c, const float *x, uint32_t cols, uint32_t nrows, uint8_t *q,
                            uint64_t qpitch);

// y[tok][rows] = W[expert] . x[tok].  Quantised types read the activations
// from xq (quantised rows); f32/f16 matrices read x directly.
// add != nullptr: y = W . x + add (same shape as y; may alias y).
// CTAs of a quantised matvec over m's rows (each quantises a one-token input
// itself when launch_qmatvec gets no pre-quantised rows).
uint32_t qmv_ctas(const DevMat &m);
// Whether launch_qmatvec runs this matvec as the persistent streaming kernel
// (one token over a large matrix; it quantises the f32 row itself).
bool qmv_streams(const DevMat &m, uint32_t ntok, int num_sms);
// n <= 4 one-token matvecs y[s] = m[s] . x (x normalised by norm_w first when
// given) in one launch; the matrices share cols and may differ in type.
cudaError_t launch_qmatvec_multi(const LaunchCfg &c, uint32_t n, const DevMat *const *m, const float *x,
                                 const float *norm_w, float eps, float *const *y);
cudaError_t launch_qmatvec(const LaunchCfg &c, const DevMat &m, uint32_t expert, const uint8_t *xq,
                           uint64_t xq_pitch, const float *x, float *y, uint32_t ntok,
                           const float *add = nullptr);

// Router over f32 weights [E][cols] (row stride w_ld floats); logits scratch
// [ntok][E]; counters zero-initialised, one per token group (reset by the
// kernel).  norm_w != nullptr routes rmsnorm(x) * norm_w.  xq != nullptr also
// writes the (normalised) input as quantised rows for the expert kernels.
cudaError_t launch_router(const LaunchCfg &c, const float *w, uint32_t E, uint32_t cols, uint32_t w_ld,
                          const float *x, const float *norm_w, float eps, uint32_t ntok, uint32_t k,
                          int norm_topk, const float *escale, uint32_t *ids, float *wout, float *logits,
                          uint32_t *counters, uint8_t *xq, uint64_t xq_pitch, float *xn = nullptr);
uint32_t router_token_groups(uint32_t ntok);

cudaError_t launch_moe_plan(const LaunchCfg &c, const uint32_t *ids, uint32_t ntok, uint32_t k,
                            uint32_t E, const MoePlan &p);
// hq[pos] = quantised act(gate_e . x_tok) * (up_e . x_tok).  direct: ntok == 1
// and ids are the plan (position = slot).  up.data == nullptr: fused gate_up.
// hf: f32 h rows [ntok*k][F]; hcnt: [ntok*k][F/32] counters that must be zero
// on entry (the kernel leaves them zero).
cudaError_t launch_moe_gate_up(const LaunchCfg &c, const DevMat &gate, const DevMat &up, int act,
                               const uint8_t *xq, uint64_t xq_pitch, uint32_t ntok, uint32_t k,
                               const uint32_t *ids, bool direct, const MoePlan &p, float *hf,
                               uint32_t *hcnt, uint8_t *hq, uint64_t hq_pitch);
constexpr size_t kMoeCounterBase = 4096;  // MoE block counters start here in the context's counter array
// out[t][d] = (resid ? resid[t][d] : 0) + sum_s w[t][s] * (down_e(s) . h[pos(t,s)])
cudaError_t launch_moe_down(const LaunchCfg &c, const DevMat &down, const uint8_t *hq, uint64_t hq_pitch,
                            uint32_t ntok, uint32_t k, const uint32_t *ids, const float *w, bool direct,
                            const MoePlan &p, const float *resid, float *out);


// One token through a whole MoE block in one persistent kernel (one CTA per
// SM, grid barriers): RMSNorm (norm_w != nullptr), router, top-k, gate/up,
// down, combine, residual (residual != 0: out = x + moe).  out may alias x.
struct DecodeParams {
    const float *router;  // F32 [E][router_ld]; nullptr: a dense FFN (E = k = 1, weight 1)
    uint32_t E, d, router_ld;
    const float *x, *norm_w;
    // nullable: the router takes x * rms_inv * router_gs * router_scale, the
    // experts rmsnorm(x) * norm_w (Gemma 4's rmsnormWeightedAndRawScaled)
    const float *router_scale = nullptr;
    float router_gs = 1.0f;
    float eps;
    uint32_t k;
    int norm_topk;
    const float *escale;
    uint32_t *ids;
    float *w;
    DevMat gate;
    const uint8_t *up_data;  // nullptr: fused gate_up
    DevMat down;
    uint32_t F;
    int act;
    uint8_t *himg;  // [k][moe_decode_img_bytes(F)] scratch
    int residual;
    float *out;
    // kDecodeSyncBytes, zero-initialised, used by no other kernel and only
    // with grid = num_sms: epoch and barrier counters, tagged logits
    uint8_t *sync;
    // optional L2 prefetch ranges issued at kernel start (the next kernel's weights)
    const uint8_t *pf[2] = {nullptr, nullptr};
    uint64_t pf_bytes[2] = {0, 0};
};
constexpr size_t kDecodeSyncBytes = 36864;

// Grouped expert GEMM on the tensor cores (lt_moe_gemm.cu) for multi-token
// batches with Q4_K gate/up/down (K <= 2048).  x: [T][d] expert input (already
// normalised), w: [T][k] slot weights, p: dispatch plan of the T*k pairs;
// out = (resid ? resid : 0) + sum_s w_s * down(act(gate x) * up x).
bool moe_gemm_supported(const DevMat &gate, const DevMat &down, uint64_t F);
size_t moe_gemm_scratch(uint32_t T, uint32_t k, uint32_t E, uint64_t d, uint64_t F);
cudaError_t launch_moe_gemm_ffn(const LaunchCfg &c, const DevMat &gate, const uint8_t *up, const DevMat &down, int act,
                                const float *x, uint32_t T, uint32_t k, const float *w, const MoePlan &p,
                                const float *resid, float *out, uint8_t *scratch);
size_t moe_decode_img_bytes(uint64_t F);
constexpr size_t kDecodeSmemLimit = 227 * 1024;
// Whether the persistent kernel's per-CTA share fits in shared memory.
bool moe_decode_fits(const DecodeParams &p, int num_sms);
cudaError_t launch_moe_decode(const LaunchCfg &c, const DecodeParams &p);

// Every decoder layer of one token in one persistent kernel (lt_stack.cu):
// attention (stacked Q8_0 Q/K/V rows, optional bias and Q/K norms, RoPE,
// f32/f16 KV, Q8_0 wo) and a Q4_K MoE or Q8_0 dense SwiGLU FFN per layer,
// x updated in place.  One descriptor per layer, in device memory.
struct StackLayerDev {
    const uint8_t *wqkv, *wo;
    const float *attn_norm, *ffn_norm, *q_norm, *k_norm, *bias;
    void *kc, *vc;
    const float *router;              // nullptr: a dense FFN (gate/up/down are 2-D)
    const uint8_t *gate, *up, *down;  // up == nullptr: fused gate_up
    uint64_t reserved;                // 112 bytes: the table is copied to shared memory by TMA
};
static_assert(sizeof(StackLayerDev) % 16 == 0, "layer descriptor size");
struct StackParams {
    AttnGeom g;
    uint32_t d, E, k, F;
    int norm_topk, act, dense;
    float eps;
    uint32_t n_layers;
    uint32_t qtype, otype, gtype, dtype;
    uint64_t qpitch, opitch, gpitch, dpitch;
};
constexpr size_t kStackSyncBytes = 16384;
// Whether the stack kernel takes this shape: its shared memory and global
// scratch bytes (the sync block at sync_offset must be zeroed once, before
// the first launch, and used by no other kernel).
bool stack_plan(const StackParams &p, int num_sms, size_t *smem, size_t *scratch_bytes, size_t *sync_offset);
cudaError_t launch_stack(const LaunchCfg &c, const StackParams &p, const void *dev_layers, float *x,
                         const uint32_t *pos, uint8_t *scratch);

// out[t] = (resid ? resid[t] : 0) + sum_s w[t][s] * y[pair_pos[t*k + s]]  (slot order), D columns.
cudaError_t launch_combine(const LaunchCfg &c, const float *y, uint64_t D, const uint32_t *pair_pos, const float *w,
                           uint32_t ntok, uint32_t k, const float *resid, float *out);

// Expert parallelism (lt_ep.cu): experts [r*E/nranks, (r+1)*E/nranks) live on rank r.
cudaError_t launch_ep_dispatch(const LaunchCfg &c, const uint32_t *ids, uint32_t ntok, uint32_t k, uint32_t E,
                               uint32_t nranks, uint32_t *send_counts, uint32_t *send_token, uint32_t *send_local,
                               uint32_t *pair_pos);
cudaError_t launch_gather_rows(const LaunchCfg &c, const float *src, uint64_t cols, const uint32_t *idx, uint32_t n,
                               float *dst);

}  // namespace lt
