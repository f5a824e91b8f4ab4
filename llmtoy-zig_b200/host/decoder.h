/*
 * decoder.h — C API of the host decode loop (libllmtoy_host.so).
 *
 * The reference's forward loop is host code (src/model/forward.zig:229-316,
 * forwardOneModel; the generate loop of src/main.zig) that calls its ops per
 * token.  This is that loop restated in C++ on top of the C ABI alone
 * (include/llmtoy_cuda.h), as a Zig host would bind it: weights are lt_tensor
 * handles, norms and caches device buffers from lt_device_alloc.  One decode
 * step is captured once as a CUDA graph and replayed per token; the position
 * and the token stream live on the device, so a whole generation runs without
 * a host round trip.
 *
 * Model shapes covered (per layer): RMSNorm -> Q/K/V (stacked or separate,
 * optional biases) -> optional per-head Q/K RMSNorm -> RoPE -> KV cache ->
 * attention -> wo + residual -> FFN block (dense SwiGLU, or the MoE block with
 * router/top-k/experts) + residual; then the final norm, lm_head, greedy.
 */
#ifndef LLMTOY_HOST_DECODER_H
#define LLMTOY_HOST_DECODER_H

#include "llmtoy_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lth_layer {
    const float *attn_norm, *ffn_norm;   /* device [d_model]                           */
    const lt_tensor *wqkv;               /* [nq + 2 nkv][d] stacked rows, or NULL:      */
    const lt_tensor *wq, *wk, *wv;       /*   separate [nq][d], [nkv][d], [nkv][d]      */
    const lt_tensor *wo;                 /* [d][nq]                                     */
    const float *qkv_bias;               /* device [nq + 2 nkv] or NULL (forward.zig:285) */
    const float *q_norm, *k_norm;        /* device [head_dim] or NULL (per-head RMSNorm) */
    const lt_tensor *ffn_gate, *ffn_up, *ffn_down;         /* dense FFN (router NULL)   */
    const lt_tensor *router, *exp_gate, *exp_up, *exp_down; /* MoE FFN                 */
    /* family LTH_GEMMA4 only (src/model/gemma4/weights.zig): exp_up NULL, exp_gate
     * is the fused gate_up tensor; wv NULL means V = K */
    const float *post_attention_norm, *pre_ffw_norm_2, *post_ffw_norm_1, *post_ffw_norm_2, *post_ffw_norm;
    const float *router_scale;           /* device [d_model] */
    const float *down_exps_scale;        /* device [n_experts] */
    float layer_output_scale;
    uint32_t is_swa;                     /* sliding-window layer */
    uint32_t n_kv_heads, head_dim;       /* this layer's (0: the model's) */
} lth_layer;

enum { LTH_LLAMA = 0, LTH_GEMMA4 = 1 };

typedef struct lth_model {
    uint32_t n_layers, d_model, n_heads, n_kv_heads, head_dim, vocab;
    uint32_t n_used;       /* experts per token (MoE layers) */
    uint32_t norm_topk;    /* renormalise the selected weights */
    uint32_t rope_neox;    /* 0: rope.zig:14 pairs, 1: rope.zig:56 halves */
    uint32_t act;          /* lt_act of the FFN */
    float eps, rope_theta;
    uint32_t kv_cap;       /* positions per sequence */
    const lt_tensor *token_emb, *lm_head;
    const float *out_norm; /* device [d_model] */
    const lth_layer *layers;
    /* LTH_LLAMA: forwardOneModel (src/model/forward.zig:229-316) with the MoE
     * block option; LTH_GEMMA4: gemma4/forward.zig:37-567 (embedding scale,
     * SWA ring caches, post norms, dense + MoE GeGLU FFNs, logit soft-cap) */
    uint32_t family;
    float rope_theta_swa, logit_softcap;
    uint32_t sliding_window;
    uint32_t kv_f16;       /* 1: f16 KV caches (the reference's GPU cache format), 0: f32 */
} lth_model;

typedef struct lth_decoder lth_decoder;

/* The model description is copied; tensors and device buffers it points to
 * must outlive the decoder. */
lt_status lth_decoder_create(lt_ctx *ctx, const lth_model *m, lth_decoder **out);
void lth_decoder_free(lth_decoder *d);
/* Start a sequence: prompt into the device token stream, position 0. */
lt_status lth_decoder_start(lth_decoder *d, const uint32_t *prompt, uint32_t n_prompt);
/* Enqueue one step with eager launches (the first call also sizes every
 * scratch buffer, so a capture afterwards allocates nothing).  Every eager
 * step computes the logits, prompt positions included. */
lt_status lth_decoder_step(lth_decoder *d);
/* Capture the step as graphs (done on first use by lth_generate): the full
 * step, and the prompt step without the output norm, lm_head and sampling
 * (main.zig:1916-1919 asks for logits only at the last prompt position). */
lt_status lth_decoder_capture(lth_decoder *d);
/* LTH_LLAMA only: the decoder layers alone at the current position (no
 * embedding, logits or position advance) -- x is updated in place and the
 * layer caches' slot at the position rewritten.  For timing the layer stack. */
lt_status lth_decoder_run_layers(lth_decoder *d);
/* 1 when the steps run every layer in one launch (lt_stack_run), else 0. */
int lth_decoder_uses_stack(const lth_decoder *d);
/* Replay n_steps steps (asynchronous): the prompt graph while the next
 * position is still a prompt position, the full step after. */
lt_status lth_decoder_replay(lth_decoder *d, uint32_t n_steps);
/* Device address of the last step's logits [vocab]. */
const float *lth_decoder_logits(const lth_decoder *d);
/* Copy tokens[0, n) of the device token stream to the host (synchronises). */
lt_status lth_decoder_tokens(lth_decoder *d, uint32_t *host_out, uint32_t n);
/* Sampling for the following steps (src/model/sample.zig; temperature 0:
 * greedy), the generator seeded as DefaultPrng.init(seed).  Re-captures the
 * step graph on its next use. */
lt_status lth_decoder_set_sampling(lth_decoder *d, float temperature, uint32_t top_k, float top_p, uint64_t seed);
/* Prompt -> n_gen tokens into out (n_prompt + n_gen - 1 steps). */
lt_status lth_generate(lth_decoder *d, const uint32_t *prompt, uint32_t n_prompt, uint32_t n_gen,
                       uint32_t *out);

#ifdef __cplusplus
}
#endif
#endif
