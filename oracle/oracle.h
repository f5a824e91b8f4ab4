/*
 * oracle.h — CPU restatement of llmtoy-zig's quantized MoE forward path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path and the timed CPU baseline in bench.py.  Nothing in the product
 * (llmtoy-zig_b200/) links, loads or calls it.
 *
 * Every function restates one reference function, in the same float
 * evaluation order, compiled with -ffp-contract=off so that no multiply-add
 * is fused (Zig's default float mode is strict; the reference never calls
 * @setFloatMode).  Citations are path:line inside the llmtoy-zig tree.
 *
 * Assumptions that cannot be checked here (no Zig toolchain):
 *   - @reduce(.Add, v) on f32 vectors is the LLVM ordered reduction
 *     ((((-0 + v0) + v1) + v2) ...), which is what strict float mode lowers to.
 *   - @exp on f32 resolves to the C library's expf; tanh is std.math.tanh
 *     (musl-derived), restated here with the C library's tanhf.
 *   Both only affect last-ulp rounding of activations and softmax weights,
 *   never the dequantised values or the router's selected ids.
 */
#ifndef LLMTOY_ORACLE_H
#define LLMTOY_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GgmlType codes, src/gguf/types.zig:23-52 */
enum {
    ORC_F32 = 0, ORC_F16 = 1, ORC_Q5_0 = 6, ORC_Q5_1 = 7, ORC_Q8_0 = 8, ORC_Q3_K = 11, ORC_Q4_K = 12,
    ORC_Q5_K = 13, ORC_Q6_K = 14, ORC_IQ4_NL = 20
};

/* f16 bits -> f32, exact (src/quant/dequant.zig:302-305) */
float orc_f16_to_f32(uint16_t h);
/* round-to-nearest-even f32 -> f16 bits (used only by fixture generators) */
uint16_t orc_f32_to_f16(float f);

/* rowBytes, src/ops/math.zig:194-208.  Returns 0 for an unsupported type. */
size_t orc_row_bytes(uint32_t type, size_t cols);

/* Block codecs, src/quant/dequant.zig */
void orc_dequant_f32(const uint8_t *data, float *out, size_t n);   /* :17  */
void orc_dequant_f16(const uint8_t *data, float *out, size_t n);   /* :24  */
void orc_dequant_q8_0(const uint8_t *data, float *out, size_t n);  /* :42  */
void orc_dequant_q4_k(const uint8_t *data, float *out, size_t n);  /* :157 */
void orc_dequant_q6_k(const uint8_t *data, float *out, size_t n);  /* :237 */
float orc_dot_q8_0(const uint8_t *data, const float *vec, size_t n); /* :59 */
void orc_dequant_q5_0(const uint8_t *data, float *out, size_t n);   /* :201 */
float orc_dot_q5_0(const uint8_t *data, const float *vec, size_t n); /* :92  */
void orc_dequant_q5_1(const uint8_t *data, float *out, size_t n);   /* :469 */
void orc_dequant_q5_k(const uint8_t *data, float *out, size_t n);   /* :324 */
void orc_dequant_q3_k(const uint8_t *data, float *out, size_t n);   /* :388 */
void orc_dequant_iq4_nl(const uint8_t *data, float *out, size_t n); /* :623 */
float orc_dot_iq4_nl(const uint8_t *data, const float *vec, size_t n); /* :642 */
/* Q8_1 activation blocks (36 B: f16 d, f16 s = d * sum q, 32 x i8) and the
 * 4-block x4 layout, dequant.zig:508-613.  n is a multiple of 32. */
void orc_quantize_q8_1(const float *in, uint8_t *out, size_t n);    /* :517 */
void orc_dequant_q8_1(const uint8_t *data, float *out, size_t n);   /* :549 */
void orc_pack_q8_1_x4(const uint8_t *basic, size_t n_blocks, uint8_t *x4);   /* :569 */
void orc_unpack_q8_1_x4(const uint8_t *x4, size_t n_groups, uint8_t *basic); /* :588 */

/* dequantRow, src/ops/math.zig:211-225.  Returns -1 for an unsupported type. */
int orc_dequant_row(const uint8_t *data, float *out, size_t n, uint32_t type);

/* src/ops/math.zig */
void  orc_matvec(float *out, const float *mat, const float *vec, size_t rows, size_t cols); /* :8 */
float orc_dotf32(const float *a, const float *b, size_t n);                                /* :96 */
int   orc_quant_matvec(float *out, const uint8_t *mat, uint32_t type, const float *vec,
                       size_t rows, size_t cols, float *row_buf);                          /* :133 */
void  orc_rmsnorm(float *out, const float *x, const float *w, size_t n, float eps);        /* :20 */
void  orc_rmsnorm_raw(float *out, const float *x, size_t n, float eps);                    /* :43 */
void  orc_softmax(float *x, size_t n);                                                     /* :29 */
float orc_silu(float x);                                                                   /* :38 */
float orc_gelu(float x);                                                                   /* :85 */

/* Persistent worker pool, src/ops/thread_pool.zig:15-112 */
typedef struct orc_pool orc_pool;
orc_pool *orc_pool_create(int n_threads);
void      orc_pool_destroy(orc_pool *pool);
int       orc_pool_threads(const orc_pool *pool);

/* quantMatvecPar, src/ops/math.zig:277-320 (scratch: threads*cols floats) */
int orc_quant_matvec_par(float *out, const uint8_t *mat, uint32_t type, const float *vec,
                         size_t rows, size_t cols, float *scratch, orc_pool *pool);

/* Router, src/model/gemma4/forward.zig */
typedef struct { float max; float exp_sum; } orc_softmax_stats;
orc_softmax_stats orc_topk_with_softmax_stats(const float *scores, size_t n,
                                              uint32_t *out, size_t k);            /* :598 */
void orc_softmax_topk(float *scores, size_t n, uint32_t *out, size_t k);           /* :637 */
orc_softmax_stats orc_topk_matvec_f32(const float *w, const float *vec, size_t rows, size_t cols,
                                      uint32_t *out, float *selected, size_t k);   /* :672 */
orc_softmax_stats orc_topk_matvec_f32_par(const float *w, const float *vec, size_t rows,
                                          size_t cols, uint32_t *out, float *selected,
                                          size_t k, orc_pool *pool);               /* :769 */
/* routerTopKSoftmax (:648): writes softmax probabilities of the k selected
 * experts into scores[idx] and the ids (descending, lowest index on ties). */
void orc_router_topk_softmax(float *scores, uint32_t *out, size_t k, const float *router_w,
                             size_t rows, size_t cols, const float *router_in, orc_pool *pool);
/* topK of the generic MoE (src/ops/moe.zig:80-91) */
void orc_moe_topk(const float *scores, size_t n, uint32_t *out, size_t k);

/* Generic moeForward, src/ops/moe.zig:18-77: softmax over all router logits,
 * topK, fused gate_up tensor (gate rows [0,F), up rows [F,2F)), SiLU, no
 * renormalisation.  out must be zeroed by the caller. */
int orc_moe_forward(float *out, const float *router_w, size_t n_experts,
                    const uint8_t *gate_up, uint32_t gate_up_type,
                    const uint8_t *down, uint32_t down_type,
                    const float *x, size_t d_model, size_t n_used, size_t d_expert,
                    orc_pool *pool);

/*
 * One MoE FFN layer over T tokens: router + selected experts + weighted
 * combine.  The router is routerTopKSoftmax (gemma4/forward.zig:648-668);
 * the expert loop is gemma4/forward.zig:463-479 with a selectable
 * activation.
 *   up == NULL      -> `gate` is the fused gate_up tensor (forward.zig:469-471)
 *   norm_topk != 0  -> weights renormalised over the k selected (Qwen3-MoE;
 *                      NEW oracle code, the reference has no such mode)
 *   expert_scale    -> multiplied in as down_exps_scale[e] * w (forward.zig:477)
 *   act             -> 0 = SiLU (math.zig:38), 1 = GELU tanh (math.zig:85)
 * ids_out / w_out (T*k) receive the selected ids and final weights.
 */
int orc_moe_layer(float *out, const float *x, size_t n_tok, size_t d_model,
                  const float *router_w, size_t n_experts, size_t k, int norm_topk,
                  const float *expert_scale,
                  const uint8_t *gate, const uint8_t *up, uint32_t gate_type,
                  const uint8_t *down, uint32_t down_type, size_t d_expert, int act,
                  orc_pool *pool, uint32_t *ids_out, float *w_out);

/* greedy, src/model/sample.zig:11-17 (lowest index among equal maxima) */
uint32_t orc_greedy(const float *logits, size_t n);

/* RoPE on one head vector, src/ops/rope.zig:14-31 (consecutive pairs) and
 * :56-75 (NeoX halves, neox != 0). */
void orc_rope(float *vec, size_t len, size_t pos, float theta, int neox);

/* sdpAttn, src/ops/attn.zig:13-42: one query over seq_len cached rows. */
void orc_sdp_attn(float *out, const float *q, const float *ks, const float *vs, size_t seq_len,
                  size_t head_dim, float scale);

/*
 * One token of a decoder: forwardOneModel (src/model/forward.zig:229-316).
 * Per layer: rmsnorm -> Q/K/V matvecs (+ optional biases, :285-287) ->
 * optional per-head Q/K RMSNorm (the style of gemma4/forward.zig:267-268) ->
 * RoPE (rope_neox selects rope.zig:56 over :14) -> KV store at pos ->
 * sdpAttn per head with scale 1/sqrt(hd) -> wo + residual -> FFN block:
 * dense SwiGLU (router == NULL, forward.zig:307-312) or the MoE layer of
 * orc_moe_layer (norm_topk renormalisation, SiLU) -> residual.  Then the final
 * rmsnorm, lm_head and logits.  The Qwen3-MoE assembly (QK norm + NeoX RoPE +
 * MoE block) is NEW oracle code: the reference has no such model.
 * KV caches: [n_layers][kv_cap][n_kv*hd] f32, slot = pos (pos < kv_cap).
 */
typedef struct orc_layer {
    const float *attn_norm, *ffn_norm;          /* [d] */
    const uint8_t *wq, *wk, *wv, *wo;
    uint32_t wq_type, wk_type, wv_type, wo_type;
    const float *q_bias, *k_bias, *v_bias;      /* nullable */
    const float *q_norm, *k_norm;               /* [hd], nullable */
    /* dense FFN: gate/up [d_ffn][d], down [d][d_ffn] */
    const uint8_t *w_gate, *w_up, *w_down;
    uint32_t ffn_gate_type, ffn_down_type;
    /* MoE FFN when router != NULL */
    const float *router;                        /* [n_experts][d] */
    const uint8_t *e_gate, *e_up, *e_down;
    uint32_t e_gate_type, e_down_type;
} orc_layer;

typedef struct orc_model {
    size_t n_layers, d_model, n_heads, n_kv_heads, head_dim, d_ffn, vocab;
    size_t n_experts, k, d_expert;
    int norm_topk, rope_neox;
    float eps, rope_theta;
    const uint8_t *token_emb; uint32_t emb_type;
    const float *out_norm;
    const uint8_t *lm_head; uint32_t lm_type;
    const orc_layer *layers;
    int kv_f16;  /* cache K and V rounded to f16 (the reference's GPU cache format) */
} orc_model;

int orc_model_step(const orc_model *m, float *k_cache, float *v_cache, size_t kv_cap, uint32_t token,
                   size_t pos, float *logits, orc_pool *pool);

/*
 * One token of the Gemma 4 decoder: forwardOne's CPU path
 * (src/model/gemma4/forward.zig:37-567).  Per layer: attention with per-head
 * Q/K norms, raw V norm and NeoX RoPE (sliding-window layers: theta_swa and
 * a ring of `sliding_window` positions; global layers: the rope_freqs table,
 * or 1/1e6^(2i/hd) when absent, loader.zig:225-233), scale 1; post-attention
 * norm + residual; dense GeGLU FFN + post_ffw_norm_1; MoE (fused gate_up,
 * GELU, router on the raw-scaled norm, weights down_exps_scale[e] * p_e) +
 * post_ffw_norm_2; post_ffw_norm of their sum + residual; layer_output_scale.
 * Then the final norm, lm_head and the tanh soft-cap.
 * KV caches: layer l at offset sum_{j<l} cap_j * nkv_j floats, cap_l =
 * sliding_window for SWA layers, global_cap otherwise.
 */
typedef struct orc_gemma_layer {
    int is_swa;
    size_t n_kv_heads;
    const float *attn_norm, *post_attention_norm, *q_norm, *k_norm, *ffn_norm;
    const float *pre_ffw_norm_2, *post_ffw_norm_1, *post_ffw_norm_2, *post_ffw_norm;
    float layer_output_scale;
    const uint8_t *wq, *wk, *wv, *wo;   /* wv NULL: V = K (forward.zig:250) */
    uint32_t wq_type, wk_type, wv_type, wo_type;
    const uint8_t *w_gate, *w_up, *w_down;
    uint32_t gate_type, up_type, down_type;
    const float *router_w, *router_scale, *down_exps_scale;
    const uint8_t *gate_up_exps, *down_exps;
    uint32_t gu_type, dn_type;
} orc_gemma_layer;

typedef struct orc_gemma {
    size_t n_layers, d_model, n_heads, head_dim_swa, head_dim_global, d_ffn, d_expert, n_experts, k;
    size_t vocab, sliding_window;
    float eps, rope_theta_swa, logit_softcap;
    const float *rope_freqs;            /* [head_dim_global / 2] or NULL */
    const uint8_t *token_emb; uint32_t emb_type;
    const float *out_norm;
    const uint8_t *lm_head; uint32_t lm_type;
    const orc_gemma_layer *layers;
} orc_gemma;

/*
 * Sampling, src/model/sample.zig:27-183, with std.Random.DefaultPrng
 * (xoshiro256++ seeded through SplitMix64) and Random.float(f32) restated
 * from the published algorithms (no Zig compiler here to confirm the stream).
 * The full path's top-p sort is unstable in the reference (ties in an
 * unspecified order); here ties keep index order.
 */
typedef struct orc_rng { uint64_t s[4]; } orc_rng;
void orc_rng_seed(orc_rng *r, uint64_t seed);
float orc_rng_float(orc_rng *r);
uint32_t orc_sample(float *logits, size_t n, float temperature, uint32_t top_k, float top_p, orc_rng *rng);

int orc_gemma_step(const orc_gemma *m, float *k_cache, float *v_cache, size_t global_cap, uint32_t token,
                   size_t pos, float *logits, orc_pool *pool);

#ifdef __cplusplus
}
#endif
#endif
