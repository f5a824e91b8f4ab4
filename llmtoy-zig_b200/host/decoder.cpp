// decoder.cpp — host decode loop over the C ABI (see decoder.h).
//
// One step is forwardOneModel (src/model/forward.zig:229-316) with the
// device position word standing in for its `pos` argument:
//   x = embedLookup(tokens[pos])                               (:319-341)
//   per layer: xb = rmsnorm(x); qkv = W_qkv xb (+ bias)        (:272-287)
//              per-head Q/K norm, RoPE, K/V into the cache     (:289-292)
//              att = sdpAttn per head                          (:294-302)
//              x = x + wo att                                  (:304-305)
//              x = x + ffn(rmsnorm(x))  dense or MoE block     (:307-312)
//   logits = lm_head rmsnorm(x); tokens[pos+1] = greedy; pos++ (:314-316)
#include "decoder.h"

#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

struct lth_decoder {
    lt_ctx *ctx = nullptr;
    lth_model m{};
    std::vector<lth_layer> layers;
    lt_attn_cfg attn{};
    float *x = nullptr, *xb = nullptr, *logits = nullptr;
    uint8_t *kcache = nullptr, *vcache = nullptr;
    size_t kv_esize = 4;         // bytes per cache element: 4 (f32) or 2 (f16)
    std::vector<size_t> kv_off;  // per layer: offset of its cache (elements)
    // Gemma 4: dense FFN, MoE accumulator, expert and router inputs, routing
    float *fbuf = nullptr, *mbuf = nullptr, *moe_in = nullptr, *router_in = nullptr;
    uint32_t *ids = nullptr;
    float *wts = nullptr;
    uint32_t *ids_zero = nullptr;  // {0}: row index of a one-row gather
    uint32_t *tokens = nullptr;  // [kv_cap + 1]
    uint32_t *state = nullptr;   // {pos, n_prompt}
    lt_graph *graph = nullptr;   // the full step
    lt_graph *pgraph = nullptr;  // a prompt step: no logits
    float *one = nullptr;        // a one-element logits row for the prompt step's position advance
    uint32_t host_pos = 0, n_prompt = 0;  // the host's copy of the position (steps enqueued)
    bool warmed = false;
    lt_sample_params sampling{0.0f, 0, 1.0f};  // temperature 0: greedy
    uint64_t *rng = nullptr;                   // xoshiro256++ state (device)
    lt_stack *stack = nullptr;                 // all layers in one launch, when the kernel takes the shape
};

namespace {

template <class T>
lt_status alloc(lth_decoder *d, T **p, size_t count) {
    void *v = nullptr;
    lt_status st = lt_device_alloc(d->ctx, count * sizeof(T), &v);
    *p = static_cast<T *>(v);
    return st;
}

#define LTH_TRY(expr)                        \
    do {                                     \
        lt_status st_ = (expr);              \
        if (st_ != LT_OK) return st_;        \
    } while (0)

lt_status layer_step(lth_decoder *d, uint32_t l) {
    const lth_model &m = d->m;
    const lth_layer &L = d->layers[l];
    lt_ctx *c = d->ctx;
    const uint32_t *pos = d->state;
    void *kc = d->kcache + d->kv_off[l] * d->kv_esize, *vc = d->vcache + d->kv_off[l] * d->kv_esize;
    const lth_layer *next = l + 1 < m.n_layers ? &d->layers[l + 1] : nullptr;
    // the whole attention half in one launch; warm this layer's router (or FFN) in L2 meanwhile
    LTH_TRY(lt_prefetch_next(c, L.router ? L.router : L.ffn_gate, L.router ? nullptr : L.ffn_up));
    if (L.wqkv)
        LTH_TRY(lt_attn_block(c, &d->attn, d->x, L.attn_norm, m.eps, L.wqkv, L.qkv_bias, L.q_norm, L.k_norm, pos,
                              kc, vc, L.wo, d->x));
    else
        LTH_TRY(lt_attn_block_split(c, &d->attn, d->x, L.attn_norm, m.eps, L.wq, L.wk, L.wv, L.qkv_bias, L.q_norm,
                                    L.k_norm, pos, kc, vc, L.wo, nullptr, nullptr, d->x));
    // the FFN block warms the next layer's attention weights in L2
    if (next) LTH_TRY(lt_prefetch_next(c, next->wqkv ? next->wqkv : next->wq, next->wo));
    if (L.router) {
        return lt_moe_block(c, L.router, L.exp_gate, L.exp_up, L.exp_down, (int)m.act, (int)m.norm_topk, nullptr,
                            L.ffn_norm, m.eps, d->x, 1, m.n_used, d->x, nullptr, nullptr);
    }
    return lt_ffn_block(c, L.ffn_gate, L.ffn_up, L.ffn_down, (int)m.act, L.ffn_norm, m.eps, d->x, 1, 1, d->x);
}

// One Gemma 4 layer (gemma4/forward.zig:195-533, the CPU branches).
// The end of layer l (forward.zig:520-532): x = (x + rmsnorm(f' + m') * w) * los.
lt_ffn_tail_in gemma_tail(const lth_decoder *d, uint32_t l) {
    const lth_layer &L = d->layers[l];
    return lt_ffn_tail_in{d->fbuf, L.post_ffw_norm_1, d->mbuf, L.post_ffw_norm_2, L.post_ffw_norm,
                          L.layer_output_scale, d->m.eps};
}

// Layer l up to its FFN tail, which the next layer's attention block (or the
// step, after the last layer) applies.
lt_status gemma_layer(lth_decoder *d, uint32_t l) {
    const lth_model &m = d->m;
    const lth_layer &L = d->layers[l];
    lt_ctx *c = d->ctx;
    const uint32_t *pos = d->state;
    const uint32_t hd = L.head_dim ? L.head_dim : m.head_dim, nkvh = L.n_kv_heads ? L.n_kv_heads : m.n_kv_heads;
    lt_attn_cfg a{};
    a.n_heads = m.n_heads;
    a.n_kv_heads = nkvh;
    a.head_dim = hd;
    a.rope_neox = 1;  // applyRopeNeox / applyRopeFreqsNeox
    a.rope_theta = L.is_swa ? m.rope_theta_swa : m.rope_theta;
    a.eps = m.eps;
    a.scale = 1.0f;  // per-head Q/K norms control the magnitude (forward.zig:324)
    a.kv_cap = L.is_swa ? m.sliding_window : m.kv_cap;
    a.window = L.is_swa ? m.sliding_window : 0;
    a.v_norm = 1;
    a.kv_f16 = m.kv_f16 ? 1u : 0u;
    void *kc = d->kcache + d->kv_off[l] * d->kv_esize, *vc = d->vcache + d->kv_off[l] * d->kv_esize;
    // norm, Q/K/V (without wv, V = K before the norms: forward.zig:250), Q/K/V norms, RoPE, attention,
    // wo and the post-attention norm into the residual (:329-333) in one launch
    // and first the previous layer's FFN tail
    const lt_ffn_tail_in prev = l ? gemma_tail(d, l - 1) : lt_ffn_tail_in{};
    LTH_TRY(lt_attn_block_split(c, &a, d->x, L.attn_norm, m.eps, L.wq, L.wk, L.wv, nullptr, L.q_norm, L.k_norm, pos,
                                kc, vc, L.wo, L.post_attention_norm, l ? &prev : nullptr, d->x));
    // dense GeGLU FFN (:390-396; its post_ffw_norm_1 is applied in the tail)
    LTH_TRY(lt_ffn_block(c, L.ffn_gate, L.ffn_up, L.ffn_down, LT_ACT_GELU_TANH, L.ffn_norm, m.eps, d->x, 1, 0,
                         d->fbuf));
    // MoE: weighted and raw-scaled norms of x, router, experts (:401-494) in one launch
    return lt_moe_block_scaled(c, L.router, L.exp_gate, L.exp_up, L.exp_down, LT_ACT_GELU_TANH, 0, L.down_exps_scale,
                               L.pre_ffw_norm_2, L.router_scale, 1.0f / __builtin_sqrtf((float)m.d_model), m.eps,
                               d->x, 1, m.n_used, 0, d->mbuf, d->ids, d->wts);
}

lt_status step(lth_decoder *d, bool logits) {
    const lth_model &m = d->m;
    LTH_TRY(lt_embed(d->ctx, m.token_emb, d->tokens, d->state, d->x));
    if (m.family == LTH_GEMMA4) {
        LTH_TRY(lt_scale(d->ctx, d->x, m.d_model, 1, __builtin_sqrtf((float)m.d_model)));  // forward.zig:117-120
        for (uint32_t l = 0; l < m.n_layers; l++) LTH_TRY(gemma_layer(d, l));
        const lt_ffn_tail_in t = gemma_tail(d, m.n_layers - 1);
        LTH_TRY(lt_ffn_tail(d->ctx, t.dev_f, t.dev_w1, d->mbuf, t.dev_w2, t.dev_w, t.los, t.eps, m.d_model, 1, d->x));
    } else if (d->stack) {
        LTH_TRY(lt_stack_run(d->ctx, d->stack, d->x, d->state));
    } else {
        for (uint32_t l = 0; l < m.n_layers; l++) LTH_TRY(layer_step(d, l));
    }
    // a prompt position before the last: no logits, the position advances (tokens[pos+1] is a prompt id)
    if (!logits) return lt_greedy_step(d->ctx, d->one, 1, d->tokens, d->state, d->state + 1);
    LTH_TRY(lt_rmsnorm(d->ctx, d->x, m.out_norm, m.eps, m.d_model, 1, d->xb));
    LTH_TRY(lt_qmatvec(d->ctx, m.lm_head, 0, d->xb, d->logits, 1));
    if (m.family == LTH_GEMMA4 && m.logit_softcap != 0.0f)
        LTH_TRY(lt_softcap(d->ctx, d->logits, m.vocab, m.logit_softcap));
    if (d->sampling.temperature != 0.0f)
        return lt_sample_step(d->ctx, d->logits, m.vocab, &d->sampling, d->rng, d->tokens, d->state, d->state + 1);
    return lt_greedy_step(d->ctx, d->logits, m.vocab, d->tokens, d->state, d->state + 1);
}

// The whole-stack kernel for a LTH_LLAMA model whose layers it takes (stacked
// Q/K/V, same FFN kind and types everywhere), when LLMTOY_STACK=1.  Off by
// default: on config 2 it measured 2.45 ms per token against 2.29 for the
// per-layer kernels (one launch per half-layer).  Any refusal leaves d->stack
// null: the per-layer path runs.
void try_stack(lth_decoder *d) {
    const lth_model &m = d->m;
    const char *env = getenv("LLMTOY_STACK");
    if (m.family != LTH_LLAMA || !env || env[0] != '1') return;
    std::vector<lt_stack_layer> sl(m.n_layers);
    for (uint32_t l = 0; l < m.n_layers; l++) {
        const lth_layer &L = d->layers[l];
        if (!L.wqkv) return;
        lt_stack_layer &o = sl[l];
        o.wqkv = L.wqkv;
        o.wo = L.wo;
        o.attn_norm = L.attn_norm;
        o.ffn_norm = L.ffn_norm;
        o.q_norm = L.q_norm;
        o.k_norm = L.k_norm;
        o.qkv_bias = L.qkv_bias;
        o.k_cache = d->kcache + d->kv_off[l] * d->kv_esize;
        o.v_cache = d->vcache + d->kv_off[l] * d->kv_esize;
        o.router = L.router;
        o.gate = L.router ? L.exp_gate : L.ffn_gate;
        o.up = L.router ? L.exp_up : L.ffn_up;
        o.down = L.router ? L.exp_down : L.ffn_down;
    }
    lt_stack *s = nullptr;
    if (lt_stack_create(d->ctx, &d->attn, m.d_model, sl.data(), m.n_layers, m.n_used, (int)m.act, (int)m.norm_topk,
                        m.eps, &s) == LT_OK)
        d->stack = s;
}

void release(lth_decoder *d) {
    if (d->stack) lt_stack_free(d->ctx, d->stack);
    if (d->graph) lt_graph_free(d->ctx, d->graph);
    if (d->pgraph) lt_graph_free(d->ctx, d->pgraph);
    void *bufs[] = {d->x,    d->xb,     d->logits,    d->kcache, d->vcache,
                    d->fbuf,   d->mbuf,      d->moe_in,    d->router_in, d->ids,    d->wts,
                    d->ids_zero, d->tokens, d->state, d->rng, d->one};
    for (void *b : bufs)
        if (b) lt_device_free(d->ctx, b);
}

}  // namespace

extern "C" {

lt_status lth_decoder_create(lt_ctx *ctx, const lth_model *m, lth_decoder **out) {
    if (!ctx || !m || !out || !m->layers || !m->token_emb || !m->lm_head || !m->out_norm) return LT_EINVAL;
    *out = nullptr;
    if (m->n_layers == 0 || m->n_heads == 0 || m->n_kv_heads == 0 || m->kv_cap == 0 || m->vocab == 0) return LT_EINVAL;
    lth_decoder *d = new (std::nothrow) lth_decoder;
    if (!d) return LT_ENOMEM;
    d->ctx = ctx;
    d->m = *m;
    d->layers.assign(m->layers, m->layers + m->n_layers);
    d->m.layers = nullptr;
    d->attn.n_heads = m->n_heads;
    d->attn.n_kv_heads = m->n_kv_heads;
    d->attn.head_dim = m->head_dim;
    d->attn.rope_neox = m->rope_neox;
    d->attn.rope_theta = m->rope_theta;
    d->attn.eps = m->eps;
    d->attn.scale = 1.0f / __builtin_sqrtf((float)m->head_dim);  // forward.zig:300
    d->attn.kv_cap = m->kv_cap;
    d->attn.window = 0;
    d->attn.kv_f16 = m->kv_f16 ? 1u : 0u;
    d->kv_esize = m->kv_f16 ? 2 : 4;
    // per-layer caches: the model's heads and kv_cap positions, or (Gemma 4)
    // this layer's heads and, for sliding-window layers, a ring of the window
    size_t cache = 0;
    for (uint32_t l = 0; l < m->n_layers; l++) {
        const lth_layer &L = m->layers[l];
        const bool g4 = m->family == LTH_GEMMA4;
        const size_t hd = g4 && L.head_dim ? L.head_dim : m->head_dim;
        const size_t nkv = (g4 && L.n_kv_heads ? L.n_kv_heads : m->n_kv_heads) * hd;
        const size_t cap = g4 && L.is_swa ? m->sliding_window : m->kv_cap;
        if (g4 && L.is_swa && (m->sliding_window == 0 || m->sliding_window > m->kv_cap)) {
            delete d;
            return LT_EINVAL;
        }
        d->kv_off.push_back(cache);
        cache += cap * nkv;
    }
    const size_t dm = m->d_model;
    lt_status st;
    if ((st = alloc(d, &d->x, dm)) != LT_OK || (st = alloc(d, &d->xb, dm)) != LT_OK ||
        (st = alloc(d, &d->logits, m->vocab)) != LT_OK || (st = alloc(d, &d->kcache, cache * d->kv_esize)) != LT_OK ||
        (st = alloc(d, &d->vcache, cache * d->kv_esize)) != LT_OK || (st = alloc(d, &d->tokens, (size_t)m->kv_cap + 1)) != LT_OK ||
        (st = alloc(d, &d->state, 2)) != LT_OK || (st = alloc(d, &d->ids_zero, 4)) != LT_OK ||
        (st = alloc(d, &d->rng, 4)) != LT_OK || (st = alloc(d, &d->one, 1)) != LT_OK ||
        (m->family == LTH_GEMMA4 &&
         ((st = alloc(d, &d->fbuf, dm)) != LT_OK ||
          (st = alloc(d, &d->mbuf, dm)) != LT_OK || (st = alloc(d, &d->moe_in, dm)) != LT_OK ||
          (st = alloc(d, &d->router_in, dm)) != LT_OK || (st = alloc(d, &d->ids, 16)) != LT_OK ||
          (st = alloc(d, &d->wts, 16)) != LT_OK))) {
        release(d);
        delete d;
        return st;
    }
    try_stack(d);
    *out = d;
    return LT_OK;
}

void lth_decoder_free(lth_decoder *d) {
    if (!d) return;
    release(d);
    delete d;
}

lt_status lth_decoder_start(lth_decoder *d, const uint32_t *prompt, uint32_t n_prompt) {
    if (!d || !prompt || n_prompt == 0 || n_prompt > d->m.kv_cap) return LT_EINVAL;
    const uint32_t state[2] = {0, n_prompt};
    const float zero = 0.0f;
    LTH_TRY(lt_copy_to_device(d->ctx, d->tokens, prompt, (size_t)n_prompt * 4));
    LTH_TRY(lt_copy_to_device(d->ctx, d->state, state, sizeof state));
    LTH_TRY(lt_copy_to_device(d->ctx, d->one, &zero, sizeof zero));
    d->host_pos = 0;
    d->n_prompt = n_prompt;
    return lt_sync(d->ctx);  // the host arrays may go away after this call
}

lt_status lth_decoder_step(lth_decoder *d) {
    if (!d) return LT_EINVAL;
    LTH_TRY(step(d, true));
    d->warmed = true;
    d->host_pos++;
    return LT_OK;
}

lt_status lth_decoder_run_layers(lth_decoder *d) {
    if (!d) return LT_EINVAL;
    if (d->m.family != LTH_LLAMA) return LT_EINVAL;
    if (d->stack) return lt_stack_run(d->ctx, d->stack, d->x, d->state);
    for (uint32_t l = 0; l < d->m.n_layers; l++) LTH_TRY(layer_step(d, l));
    return LT_OK;
}

int lth_decoder_uses_stack(const lth_decoder *d) { return d && d->stack ? 1 : 0; }

lt_status lth_decoder_capture(lth_decoder *d) {
    if (!d) return LT_EINVAL;
    if (d->graph) return LT_OK;
    if (!d->warmed) return LT_EINVAL;  // an eager step first sizes the scratch buffers
    for (int full = 1; full >= 0; full--) {
        LTH_TRY(lt_capture_begin(d->ctx));
        lt_status st = step(d, full != 0);
        lt_graph *g = nullptr;
        lt_status st2 = lt_capture_end(d->ctx, &g);
        if (st != LT_OK || st2 != LT_OK) {
            if (g) lt_graph_free(d->ctx, g);
            if (d->pgraph) lt_graph_free(d->ctx, d->pgraph);
            if (d->graph) lt_graph_free(d->ctx, d->graph);
            d->graph = d->pgraph = nullptr;
            return st != LT_OK ? st : st2;
        }
        (full ? d->graph : d->pgraph) = g;
    }
    return LT_OK;
}

lt_status lth_decoder_replay(lth_decoder *d, uint32_t n_steps) {
    if (!d) return LT_EINVAL;
    if (!d->graph || !d->pgraph) return LT_EINVAL;
    for (uint32_t i = 0; i < n_steps; i++, d->host_pos++)
        LTH_TRY(lt_graph_launch(d->ctx, d->host_pos + 1 < d->n_prompt ? d->pgraph : d->graph));
    return LT_OK;
}

const float *lth_decoder_logits(const lth_decoder *d) { return d ? d->logits : nullptr; }

lt_status lth_decoder_set_sampling(lth_decoder *d, float temperature, uint32_t top_k, float top_p, uint64_t seed) {
    if (!d || !(temperature >= 0.0f) || !(top_p >= 0.0f)) return LT_EINVAL;
    d->sampling.temperature = temperature;
    d->sampling.top_k = top_k;
    d->sampling.top_p = top_p;
    uint64_t st[4];
    lt_rng_seed(seed, st);
    LTH_TRY(lt_copy_to_device(d->ctx, d->rng, st, sizeof st));
    LTH_TRY(lt_sync(d->ctx));
    if (d->graph) {  // the step's last op changed
        lt_graph_free(d->ctx, d->graph);
        d->graph = nullptr;
    }
    if (d->pgraph) {
        lt_graph_free(d->ctx, d->pgraph);
        d->pgraph = nullptr;
    }
    return LT_OK;
}

lt_status lth_decoder_tokens(lth_decoder *d, uint32_t *host_out, uint32_t n) {
    if (!d || !host_out || n > d->m.kv_cap + 1) return LT_EINVAL;
    LTH_TRY(lt_copy_to_host(d->ctx, host_out, d->tokens, (size_t)n * 4));
    return lt_sync(d->ctx);
}

lt_status lth_generate(lth_decoder *d, const uint32_t *prompt, uint32_t n_prompt, uint32_t n_gen, uint32_t *out) {
    if (!d || !out || n_gen == 0 || (size_t)n_prompt + n_gen > d->m.kv_cap) return LT_EINVAL;
    LTH_TRY(lth_decoder_start(d, prompt, n_prompt));
    const uint32_t steps = n_prompt + n_gen - 1;
    uint32_t done = 0;
    if (!d->graph) {  // first use: one eager step sizes the scratch, then capture
        LTH_TRY(lth_decoder_step(d));
        done = 1;
        LTH_TRY(lth_decoder_capture(d));
    }
    LTH_TRY(lth_decoder_replay(d, steps - done));
    std::vector<uint32_t> all((size_t)n_prompt + n_gen);
    LTH_TRY(lth_decoder_tokens(d, all.data(), n_prompt + n_gen));
    std::memcpy(out, all.data() + n_prompt, (size_t)n_gen * 4);
    return LT_OK;
}

}  // extern "C"
