/*
 * llmtoy_cuda.h — C ABI of the B200 (sm_100a) backend for llmtoy-zig's
 * quantized MoE forward path.
 *
 * The reference has no FFI; its operator API is Zig (src/ops, src/quant,
 * src/model/gemma4/forward.zig) and its device seam is GpuWeights in
 * src/model/gemma4/gpu_weights.zig, which returns Zig error unions.  Each
 * entry point below names the reference function it replaces.  Everything is
 * plain C: fixed-width integers, raw pointers and sizes, no CUDA or torch
 * types, so a Zig `extern fn`, a C++ host or Python ctypes can bind it.
 *
 * Conventions
 *   - Weights are uploaded once (lt_upload) and owned by the context, like
 *     GpuWeights.init (gpu_weights.zig:373).  GGUF bytes go up unchanged
 *     except that each row is padded to a 16-byte pitch on the device so
 *     every row starts 16-byte aligned; lt_tensor_download undoes it.
 *   - "dev_" pointers are device memory owned by the caller.  Device ops are
 *     asynchronous on the context's stream (lt_set_stream); lt_sync joins.
 *   - Errors are returned as lt_status, never by abort; lt_last_error gives
 *     the message.  There is no CPU fallback: a missing device is
 *     LT_ENODEV, an unsupported GGUF type LT_EUNSUPPORTED_TYPE (the
 *     reference panics there, src/ops/math.zig:206,223).
 *   - One context per GPU; a context is not re-entrant across host threads.
 *   - ggml_type uses the GGUF enum (src/gguf/types.zig:23-52): F32=0,
 *     F16=1, Q5_0=6, Q5_1=7, Q8_0=8, Q3_K=11, Q4_K=12, Q5_K=13, Q6_K=14,
 *     IQ4_NL=20 -- the types src/ops/math.zig:194-225 (rowBytes, dequantRow)
 *     handle.  K-quants (Q3_K..Q6_K) need cols % 256 == 0, the rest cols % 32.
 *     The fused single-token kernels (lt_attn_block, the T = 1 MoE block) take
 *     Q8_0/Q4_K/Q6_K weights; the other types run through the separate ops.
 */
#ifndef LLMTOY_CUDA_H
#define LLMTOY_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LT_API_VERSION 1

typedef enum lt_status {
    LT_OK = 0,
    LT_EINVAL = 1,              /* bad argument, shape or size              */
    LT_EUNSUPPORTED_TYPE = 2,   /* a ggml type outside the list above      */
    LT_ENOMEM = 3,              /* device allocation failed                 */
    LT_ECUDA = 4,               /* a CUDA runtime call failed               */
    LT_ETIMEOUT = 5,            /* a bounded device-side wait gave up       */
    LT_ENODEV = 6               /* no usable sm_100 device                  */
} lt_status;

typedef enum lt_ggml_type {
    LT_TYPE_F32 = 0,
    LT_TYPE_F16 = 1,
    LT_TYPE_Q5_0 = 6,
    LT_TYPE_Q5_1 = 7,
    LT_TYPE_Q8_0 = 8,
    LT_TYPE_Q3_K = 11,
    LT_TYPE_Q4_K = 12,
    LT_TYPE_Q5_K = 13,
    LT_TYPE_Q6_K = 14,
    LT_TYPE_IQ4_NL = 20
} lt_ggml_type;

typedef enum lt_act {
    LT_ACT_SILU = 0,            /* x / (1 + e^-x), src/ops/math.zig:38-40    */
    LT_ACT_GELU_TANH = 1        /* tanh GELU, src/ops/math.zig:85-88         */
} lt_act;

typedef struct lt_ctx lt_ctx;
typedef struct lt_tensor lt_tensor;

/* Shape of an uploaded tensor. */
typedef struct lt_tensor_desc {
    uint32_t ggml_type;
    uint32_t n_experts;     /* 0 for a plain 2-D matrix                       */
    uint64_t rows;          /* rows per expert (or total rows when 2-D)       */
    uint64_t cols;
    uint64_t row_bytes;     /* rowBytes(type, cols), src/ops/math.zig:194     */
    uint64_t row_pitch;     /* device row stride: row_bytes rounded up to 16  */
} lt_tensor_desc;

/* ── context ──────────────────────────────────────────────────────────────
 * Replaces GpuContext.init/deinit (src/gpu/context.zig:270-960).          */
int         lt_api_version(void);
lt_status   lt_init(int device, lt_ctx **out);
void        lt_free(lt_ctx *ctx);
/* Use an existing cudaStream_t (passed as void*); NULL selects the
 * context's own stream (non-blocking).  The legacy default stream is
 * cudaStreamLegacy ((void *)1), the per-thread one cudaStreamPerThread
 * ((void *)2); on those two the kernels launch without programmatic
 * dependent launch. */
lt_status   lt_set_stream(lt_ctx *ctx, void *cuda_stream);
lt_status   lt_sync(lt_ctx *ctx);
const char *lt_last_error(const lt_ctx *ctx);
const char *lt_status_string(lt_status status);
/* Pre-size the context's scratch arena for up to max_tokens tokens, so that
 * later ops allocate nothing (needed before CUDA graph capture). */
lt_status   lt_reserve(lt_ctx *ctx, uint32_t max_tokens, uint32_t max_k,
                       uint64_t max_d_model, uint64_t max_d_expert);

/* ── tensors ──────────────────────────────────────────────────────────────
 * RawMatrix{data,type_,rows,cols} (src/model/model_weights.zig:17-22) with
 * the 3-D expert flattening of src/model/gemma4/loader.zig:277-292:
 * n_experts > 0 means `rows` rows per expert, experts back to back.       */
uint64_t    lt_row_bytes(uint32_t ggml_type, uint64_t cols);   /* == rowBytes */
lt_status   lt_upload(lt_ctx *ctx, const void *host_bytes, size_t nbytes,
                      uint32_t ggml_type, uint64_t rows, uint64_t cols,
                      uint32_t n_experts, lt_tensor **out);
/* Same as lt_upload with the GGUF bytes already in device memory. */
lt_status   lt_upload_from_device(lt_ctx *ctx, const void *dev_bytes, size_t nbytes,
                                  uint32_t ggml_type, uint64_t rows, uint64_t cols,
                                  uint32_t n_experts, lt_tensor **out);
lt_status   lt_tensor_download(lt_ctx *ctx, const lt_tensor *t, void *host_bytes,
                               size_t nbytes);
lt_status   lt_tensor_describe(const lt_tensor *t, lt_tensor_desc *out);
lt_status   lt_tensor_free(lt_ctx *ctx, lt_tensor *t);

/* ── device ops (asynchronous on the context stream) ───────────────────── */

/* dequantRow over rows [row0, row0+nrows) (src/ops/math.zig:211-225 and
 * src/quant/dequant.zig:17-277).  Bit-exact with the reference CPU codecs.
 * dev_out holds nrows*cols f32.  Expert tensors: row0 counts over all
 * experts' rows. */
lt_status lt_dequant(lt_ctx *ctx, const lt_tensor *t, uint64_t row0, uint64_t nrows,
                     float *dev_out);

/* quantizeQ8_1 (src/quant/dequant.zig:517-547): n f32 values (n % 32 == 0)
 * into n/32 Q8_1 blocks of 36 bytes (f16 d = amax/127, f16 s = d*sum(q),
 * 32 int8 q rounded half away from zero), bit-exact with the reference; with
 * x4 != 0 in the block_q8_1_x4 layout instead (packQ8_1_x4, :569-586: 144
 * bytes per 4 blocks, a partial last group zero-padded, so dev_out holds
 * ceil(n/128)*144 bytes).  The reference's GPU activation format; the
 * matvecs here quantise activations their own way (qact, exact products). */
lt_status lt_quantize_q8_1(lt_ctx *ctx, const float *dev_x, uint64_t n, int x4, uint8_t *dev_out);
/* dequantQ8_1 (src/quant/dequant.zig:549-558) of n values, either layout. */
lt_status lt_dequant_q8_1(lt_ctx *ctx, const uint8_t *dev_q, uint64_t n, int x4, float *dev_out);

/* quantMatvec / quantMatvecPar (src/ops/math.zig:133-171, :277-320) for ntok
 * input vectors: dev_y[tok][rows] = W[expert] . dev_x[tok][cols].
 * expert selects one expert of a 3-D tensor (ignored for 2-D). */
lt_status lt_qmatvec(lt_ctx *ctx, const lt_tensor *w, uint32_t expert,
                     const float *dev_x, float *dev_y, uint32_t ntok);

/* rmsnorm (src/ops/math.zig:20-26) of ntok rows of length n. */
lt_status lt_rmsnorm(lt_ctx *ctx, const float *dev_x, const float *dev_w, float eps,
                     uint32_t n, uint32_t ntok, float *dev_y);

/* In-place softmax (src/ops/math.zig:29-35) of ntok rows of length n. */
lt_status lt_softmax(lt_ctx *ctx, float *dev_x, uint32_t n, uint32_t ntok);

/* Router: routerTopKSoftmax (src/model/gemma4/forward.zig:648-668).
 * f32 router logits, top-k with the lowest index winning ties
 * (forward.zig:598-629), softmax probabilities of the selected experts.
 * norm_topk != 0 renormalises the k weights to sum 1 (Qwen3-MoE; the
 * reference has no such mode).  dev_expert_scale (nullable) multiplies in
 * down_exps_scale[e] (forward.zig:477).  The logits reproduce dotf32's
 * summation order (src/ops/math.zig:96-116) exactly, so ids match the CPU
 * path bit for bit.  Outputs: dev_ids[ntok][k], dev_w[ntok][k]. */
lt_status lt_moe_route(lt_ctx *ctx, const lt_tensor *router, const float *dev_x,
                       uint32_t ntok, uint32_t k, int norm_topk,
                       const float *dev_expert_scale, uint32_t *dev_ids, float *dev_w);

/* Dispatch + grouped expert FFN + weighted combine: the expert loop of
 * src/model/gemma4/forward.zig:463-479 and src/ops/moe.zig:61-76.
 * gate: [E][F][d] (or the fused gate_up [E][2F][d] when up == NULL),
 * up: [E][F][d], down: [E][d][F].  dev_out[tok][d] is overwritten with
 * sum_i w[tok][i] * down_e(act(gate_e.x) * (up_e.x)), summed in slot order. */
lt_status lt_moe_ffn(lt_ctx *ctx, const lt_tensor *gate, const lt_tensor *up,
                     const lt_tensor *down, int act, const float *dev_x, uint32_t ntok,
                     const uint32_t *dev_ids, const float *dev_w, uint32_t k,
                     float *dev_out);

/* moeForward (src/ops/moe.zig:18-77) generalised to the routing modes above:
 * lt_moe_route followed by lt_moe_ffn.  dev_ids / dev_w may be NULL. */
lt_status lt_moe_forward(lt_ctx *ctx, const lt_tensor *router, const lt_tensor *gate,
                         const lt_tensor *up, const lt_tensor *down, int act,
                         int norm_topk, const float *dev_expert_scale,
                         const float *dev_x, uint32_t ntok, uint32_t k, float *dev_out,
                         uint32_t *dev_ids, float *dev_w);

/* The whole MoE FFN block of a decoder layer on device vectors:
 *   dev_out = dev_x + moe(rmsnorm(dev_x) * dev_norm_w)
 * i.e. the pre-FFN rmsnorm (src/ops/math.zig:20-26, src/model/forward.zig:304),
 * the router and experts of lt_moe_forward on the normalised vector, and the
 * residual add (src/model/forward.zig:309).  The norm and the residual are
 * fused into the router and down kernels (one persistent launch at one
 * token).  dev_out may alias dev_x. */
lt_status lt_moe_block(lt_ctx *ctx, const lt_tensor *router, const lt_tensor *gate,
                       const lt_tensor *up, const lt_tensor *down, int act, int norm_topk,
                       const float *dev_expert_scale, const float *dev_norm_w, float eps,
                       const float *dev_x, uint32_t ntok, uint32_t k, float *dev_out,
                       uint32_t *dev_ids, float *dev_w);

/* Gemma 4's MoE half (src/model/gemma4/forward.zig:401-494): the experts take
 * rmsnorm(dev_x) * dev_norm_w, the router dev_x * rms_inv * router_gs *
 * dev_router_scale (rmsnormWeightedAndRawScaled, src/ops/math.zig:51-82)
 * with dev_expert_scale[e] on the selected weights;
 *   dev_out = (residual ? dev_x : 0) + moe(...)
 * One persistent launch at one token (lt_norm_pair + lt_moe_route +
 * lt_moe_ffn otherwise, with the same results).  dev_out may alias dev_x. */
lt_status lt_moe_block_scaled(lt_ctx *ctx, const lt_tensor *router, const lt_tensor *gate,
                              const lt_tensor *up, const lt_tensor *down, int act, int norm_topk,
                              const float *dev_expert_scale, const float *dev_norm_w,
                              const float *dev_router_scale, float router_gs, float eps,
                              const float *dev_x, uint32_t ntok, uint32_t k, int residual,
                              float *dev_out, uint32_t *dev_ids, float *dev_w);

/* greedy (src/model/sample.zig:11-17): index of the first maximum of each of
 * ntok rows of length n (the argmax shader, src/gpu/shaders/argmax.glsl). */
lt_status lt_argmax(lt_ctx *ctx, const float *dev_x, uint32_t n, uint32_t ntok,
                    uint32_t *dev_idx);

/* Self-test of the bounded device waits (no reference counterpart: the
 * reference has no device-side timeouts; on a GPU error its forward loop falls
 * back to the CPU, src/model/gemma4/forward.zig:456-480).  Launches two CTAs
 * that run the library's own wait helpers with a limit of limit_us
 * (1..2000000):
 *   kind 0 -- a grid barrier every CTA reaches: lt_sync returns LT_OK;
 *   kind 1 -- a grid barrier expecting one arrival more than the grid gives;
 *   kind 2 -- an mbarrier expecting one arrival more than it gets.
 * Kinds 1 and 2 give up after the limit, record the code in the device error
 * word and return, so lt_sync returns LT_ETIMEOUT and the context stays
 * usable.  The persistent kernels' waits use the same helpers with a 2 s limit. */
lt_status lt_selftest_wait(lt_ctx *ctx, uint32_t kind, uint32_t limit_us);

/* ── kernel timing ────────────────────────────────────────────────────────
 * GpuProfiler (src/gpu/context.zig:34-268, LLMTOY_GPU_PROFILE): when on,
 * every kernel launch is bracketed by CUDA events on its stream and its
 * duration is aggregated per kernel label (count/total/min/max in ms).
 * Timing serialises launches (no programmatic overlap), so take throughput
 * numbers with it off. */
lt_status lt_profile_enable(lt_ctx *ctx, int on);
/* Entry `index` of the aggregate (waits for pending events first);
 * LT_EINVAL once index is past the last label.  label stays valid for the
 * life of the library. */
lt_status lt_profile_read(lt_ctx *ctx, uint32_t index, const char **label, uint64_t *count,
                          double *total_ms, double *min_ms, double *max_ms);
lt_status lt_profile_reset(lt_ctx *ctx);

/* ── CUDA graph capture ───────────────────────────────────────────────────
 * Records the device ops issued between begin and end on the context stream
 * into a graph that lt_graph_launch replays (one launch per decode token
 * instead of one per kernel).  The stream must not be the legacy default
 * stream; call lt_reserve first so no op allocates while capturing. */
typedef struct lt_graph lt_graph;
lt_status lt_capture_begin(lt_ctx *ctx);
lt_status lt_capture_end(lt_ctx *ctx, lt_graph **out);
lt_status lt_graph_launch(lt_ctx *ctx, const lt_graph *graph);
lt_status lt_graph_free(lt_ctx *ctx, lt_graph *graph);

/* ── allocation-free MoE FFN ─────────────────────────────────────────────────
 * No counterpart in the reference (its CPU path allocates per call and its
 * Vulkan path owns its buffers).  For callers that cannot allocate device
 * memory themselves -- an embedding runtime or pool hands them every buffer,
 * or another owner drives the allocator -- this runs the same dispatch +
 * grouped gate/up + down + weighted combine as lt_moe_ffn without a context
 * and without allocating: weights, x, ids, w and out are the caller's device
 * pointers, and the intermediate activations live in a fixed 8 MiB device
 * array inside the library (held by every GPU that loads it until exit).
 *   - Weights are GGUF rows used in place: gate [E][F or 2F][d] (fused
 *     gate_up when up == NULL), up [E][F][d], down [E][d][F]; every row's
 *     byte size and every weight pointer must be a multiple of 16 (true for
 *     Q4_K/Q6_K/Q8_0 rows of 2048 or 768 columns).
 *   - Capacity: 256 + ntok*qact(d) + ntok*k*(qact(F) + 4*F + F/8)
 *     + (3*E + 2*ntok*k + 1)*4 bytes, each term rounded up to 256, with
 *     qact(n) = 3.375*n rounded up to 16; larger requests return LT_EINVAL.
 *     (ntok=16, k=8, d=2048, F=768 uses 0.9 MiB.)
 *   - Asynchronous on cuda_stream (NULL = legacy default stream).  The first
 *     call on each device looks up the array's device address; make that
 *     first call before any stream capture.
 *   - Calls share the array: calls that overlap on the GPU race.
 *   - The array's address is kept per device for the life of the process:
 *     after a cudaDeviceReset of a device it ran on, unload the library.
 * Returns LT_EINVAL / LT_EUNSUPPORTED_TYPE for bad arguments, LT_ECUDA if a
 * launch fails.  Faults the kernels detect on the device (an id >= n_experts,
 * whose token's output is then unspecified; a copy that timed out) are not in
 * this return value: lt_noalloc_status reports them. */
lt_status lt_moe_ffn_noalloc(void *cuda_stream, const void *gate, const void *up,
                             const void *down, uint32_t gate_type, uint32_t down_type,
                             uint32_t n_experts, uint64_t d_model, uint64_t d_expert, int act,
                             const float *dev_x, uint32_t ntok, const uint32_t *dev_ids,
                             const float *dev_w, uint32_t k, float *dev_out);

/* The device-detected fault of the lt_moe_ffn_noalloc calls issued on
 * cuda_stream since the last call started (each call clears the word first):
 * waits for the stream, then returns LT_OK, LT_EINVAL (an expert id past
 * n_experts) or LT_ETIMEOUT (a device-side wait gave up), and clears it.
 * Allocates nothing; not for use during stream capture. */
lt_status lt_noalloc_status(void *cuda_stream);

/* ── expert-parallel MoE layer ───────────────────────────────────────────────
 * No counterpart in the reference, whose MoE runs on one device (the seam it
 * plugs into is GpuWeights.runExpertBatch, src/model/gemma4/gpu_weights.zig:
 * 2748).  Rank r of nranks holds experts [r*E/nranks, (r+1)*E/nranks) of each
 * layer; the exchange runs over NCCL, which is loaded at run time
 * (libnccl.so.2; LT_ENODEV when absent).
 *
 * lt_ep_unique_id: on one rank, the 128-byte id the host hands to every rank
 * (its own channel: a store, MPI, a file).  lt_ep_init: every rank, one ep per
 * context; the context's stream at this point is the ep's stream for life.
 * timeout_ms bounds every host-side wait of a call: when it runs out the
 * communicator is aborted (its kernels return) and the call returns
 * LT_ETIMEOUT, as does every later call on that ep; an error NCCL reports
 * aborts it too (LT_ECUDA). */
typedef struct lt_ep lt_ep;
lt_status lt_ep_unique_id(uint8_t id_out[128]);
lt_status lt_ep_init(lt_ctx *ctx, uint32_t nranks, uint32_t rank, const uint8_t id[128], uint32_t timeout_ms,
                     lt_ep **out);
lt_status lt_ep_free(lt_ep *ep);

/* One MoE layer over this rank's ntok tokens, expert-parallel (every rank
 * calls it for the same layer, in the same order): router [E][d] replicated;
 * gate/up/down this rank's E/nranks experts (up NULL: fused gate_up);
 * dev_out[ntok][d] = dev_x + moe(rmsnorm(dev_x) * dev_norm_w) when dev_norm_w
 * is given, else moe(dev_x) -- the same result as lt_moe_block / lt_moe_forward
 * over all E experts on one device.  Synchronises with the stream twice (the
 * split sizes, then the end of the exchanges): not capturable. */
lt_status lt_moe_ffn_ep(lt_ctx *ctx, lt_ep *ep, const lt_tensor *router, const lt_tensor *gate,
                        const lt_tensor *up, const lt_tensor *down, int act, int norm_topk,
                        const float *dev_expert_scale, const float *dev_norm_w, float eps,
                        const float *dev_x, uint32_t ntok, uint32_t k, float *dev_out);

/* ── expert parallelism building blocks ──────────────────────────────────────
 * No counterpart in the reference, whose MoE runs on one device: these let a
 * host shard the experts across ranks (experts [r*E/n, (r+1)*E/n) on rank r)
 * and exchange tokens with an all-to-all of its own (NCCL, or any transport).
 * Per layer: lt_moe_route -> lt_ep_dispatch -> lt_gather_rows (send buffer)
 * -> all-to-all (rows and local ids) -> lt_moe_ffn on the received rows with
 * k = 1 and weight 1 -> all-to-all back -> lt_moe_combine. */

/* Stable sort of the ntok*k (token, slot) pairs of ids [ntok][k] by
 * destination rank.  Outputs (device): send_counts[nranks] pairs per rank,
 * and per send position send_token (the pair's token) and send_local (its
 * expert index on the destination rank); pair_pos[ntok*k] is the send
 * position of each pair.  n_experts % nranks == 0, nranks <= 8. */
lt_status lt_ep_dispatch(lt_ctx *ctx, const uint32_t *dev_ids, uint32_t ntok, uint32_t k,
                         uint32_t n_experts, uint32_t nranks, uint32_t *dev_send_counts,
                         uint32_t *dev_send_token, uint32_t *dev_send_local,
                         uint32_t *dev_pair_pos);

/* dev_dst[i][:] = dev_src[dev_idx[i]][:] for i < n rows of cols floats
 * (cols % 4 == 0). */
lt_status lt_gather_rows(lt_ctx *ctx, const float *dev_src, uint64_t cols, const uint32_t *dev_idx,
                         uint32_t n, float *dev_dst);

/* Weighted combine in slot order (forward.zig:463-479):
 * out[t][:] = (resid ? resid[t][:] : 0) + sum_s w[t][s] * y[pair_pos[t*k + s]][:]. */
lt_status lt_moe_combine(lt_ctx *ctx, const float *dev_y, uint64_t cols, const uint32_t *dev_pair_pos,
                         const float *dev_w, uint32_t ntok, uint32_t k, const float *dev_resid,
                         float *dev_out);

/* ── device buffers ──────────────────────────────────────────────────────────
 * For hosts without a CUDA runtime of their own (the Zig forward loop, the
 * C++ host in this package): activation buffers, KV caches and token streams.
 * Copies are asynchronous on the context stream; lt_sync joins. */
lt_status lt_device_alloc(lt_ctx *ctx, size_t bytes, void **dev_out);  /* zero-filled */
lt_status lt_device_free(lt_ctx *ctx, void *dev);
lt_status lt_copy_to_device(lt_ctx *ctx, void *dev_dst, const void *host_src, size_t bytes);
lt_status lt_copy_to_host(lt_ctx *ctx, void *host_dst, const void *dev_src, size_t bytes);

/* ── decode-step ops ─────────────────────────────────────────────────────────
 * The pieces of one token of forwardOneModel (src/model/forward.zig:229-316)
 * beyond the matvecs and the MoE block.  Each reads the token position from
 * a device word (dev_pos), so one captured graph (lt_capture_begin) serves
 * every step of a generation: the host writes the prompt into a device token
 * stream once and replays the graph. */

/* Geometry of one attention layer. */
typedef struct lt_attn_cfg {
    uint32_t n_heads, n_kv_heads, head_dim;   /* head_dim 64, 128 or 256 */
    uint32_t rope_neox;  /* 0: consecutive pairs (rope.zig:14), 1: NeoX halves (rope.zig:56) */
    float rope_theta;
    float eps;           /* per-head Q/K RMSNorm epsilon */
    float scale;         /* score scale: 1/sqrt(head_dim) (forward.zig:300), 1 for Gemma 4 */
    uint32_t kv_cap;     /* positions per layer cache; slot = pos % kv_cap */
    uint32_t window;     /* 0: attend to every position; else the last `window` (sliding) */
    uint32_t v_norm;     /* 1: RMSNorm without weights on each V head (gemma4/forward.zig:269) */
    uint32_t kv_f16;     /* 1: the caches hold IEEE f16 elements (stored rounded to nearest even, as the
                            reference's GPU cache does); 0: f32 (its CPU KvCache) */
} lt_attn_cfg;

/* embedLookup (src/model/forward.zig:319-341): dev_out[cols] = dequantised
 * row dev_tokens[*dev_pos] of emb.  An id beyond the table is reported by
 * lt_sync as LT_EINVAL (the row read is row 0). */
lt_status lt_embed(lt_ctx *ctx, const lt_tensor *emb, const uint32_t *dev_tokens,
                   const uint32_t *dev_pos, float *dev_out);

/* Up to four one-token quantMatvec calls on the same input vector in one
 * launch, e.g. a layer's separate Q, K and V projections (forward.zig:278-281):
 * dev_y[i] = w[i] . xn with xn = dev_x, or rmsnorm(dev_x) * dev_norm_w when
 * dev_norm_w is given (the pre-attention norm folded in, math.zig:20-26).
 * The tensors share cols and may differ in type. */
lt_status lt_qmatvec_multi(lt_ctx *ctx, uint32_t n, const lt_tensor *const *w, const float *dev_x,
                           const float *dev_norm_w, float eps, float *const *dev_y);

/* quantMatvec plus an addend of y's shape: y = W . x + add -- the residual
 * `x += wo . attn` (forward.zig:304-305) or the Q/K/V biases (:285-287).
 * dev_add may alias dev_y. */
lt_status lt_qmatvec_add(lt_ctx *ctx, const lt_tensor *w, uint32_t expert, const float *dev_x,
                         const float *dev_add, float *dev_y, uint32_t ntok);

/* dev_qkv = [q (n_heads*hd) | k (n_kv*hd) | v (n_kv*hd)] of this position:
 * per-head RMSNorm of q and k when their weights (head_dim floats) are
 * given (gemma4/forward.zig:267-268), RoPE on q and k (rope.zig), q updated in
 * place; k and v written to the caches at slot *dev_pos % kv_cap.  Caches are
 * [kv_cap][n_kv*hd] elements, f32 or f16 (cfg->kv_f16). */
lt_status lt_attn_prep(lt_ctx *ctx, const lt_attn_cfg *cfg, float *dev_qkv, const float *dev_q_norm,
                       const float *dev_k_norm, const uint32_t *dev_pos, void *dev_k_cache,
                       void *dev_v_cache);

/* sdpAttn (src/ops/attn.zig:13-42) of every query head over the cached
 * positions max(0, pos+1-window) .. pos (query head h reads KV head
 * h / (n_heads / n_kv_heads)); dev_out[n_heads*hd]. */
lt_status lt_attn_decode(lt_ctx *ctx, const lt_attn_cfg *cfg, const float *dev_q,
                         const void *dev_k_cache, const void *dev_v_cache,
                         const uint32_t *dev_pos, float *dev_out);

/* The attention half of a decoder layer for one token (forward.zig:272-305
 * with the per-head Q/K norms of gemma4/forward.zig:267-268):
 *   xn = rmsnorm(x) * norm_w;  qkv = wqkv . xn (+ bias);  per-head Q/K norm,
 *   RoPE, K/V into the caches at *dev_pos;  att = attention per head;
 *   out = x + wo . att.
 * wqkv holds the Q, K and V rows stacked ([nq + 2 nkv][d]).  On one GPU this
 * runs as a single persistent kernel (one CTA per SM, grid-wide hand-offs,
 * weight tiles loaded before the previous kernel ends); shapes it does not
 * cover run as the separate ops.  dev_out may alias dev_x. */
lt_status lt_attn_block(lt_ctx *ctx, const lt_attn_cfg *cfg, const float *dev_x, const float *dev_norm_w,
                        float eps, const lt_tensor *wqkv, const float *dev_qkv_bias,
                        const float *dev_q_norm, const float *dev_k_norm, const uint32_t *dev_pos,
                        void *dev_k_cache, void *dev_v_cache, const lt_tensor *wo, float *dev_out);

/* The end of a Gemma 4 layer (lt_ffn_tail's inputs, gemma4/forward.zig:520-532):
 * x' = (x + rmsnorm(f' + rmsnorm(m) * w2) * w) * los, f' = rmsnorm(f) * w1
 * (w1 nullable: f' = f); rmsnorm with eps.  m is only read. */
typedef struct lt_ffn_tail_in {
    const float *dev_f, *dev_w1, *dev_m, *dev_w2, *dev_w;
    float los, eps;
} lt_ffn_tail_in;

/* lt_attn_block over separate Q, K and V tensors ([nq][d], [nkv][d], [nkv][d];
 * the types may differ).  wv NULL: V is the K projection before the norms
 * (gemma4/forward.zig:250), and dev_qkv_bias (nullable) then holds nq + nkv
 * entries.  dev_post_norm non-NULL: out = x + rmsnorm(wo . att) * post_norm
 * (gemma4/forward.zig:329-333) instead of x + wo . att.  tail non-NULL: the
 * block's input is the previous layer's tail of dev_x (x' above) instead of
 * dev_x itself, in the same launch; dev_x is not written (unless it is
 * dev_out). */
lt_status lt_attn_block_split(lt_ctx *ctx, const lt_attn_cfg *cfg, const float *dev_x, const float *dev_norm_w,
                              float eps, const lt_tensor *wq, const lt_tensor *wk, const lt_tensor *wv,
                              const float *dev_qkv_bias, const float *dev_q_norm, const float *dev_k_norm,
                              const uint32_t *dev_pos, void *dev_k_cache, void *dev_v_cache,
                              const lt_tensor *wo, const float *dev_post_norm, const lt_ffn_tail_in *tail,
                              float *dev_out);

/* ── whole-stack decode ─────────────────────────────────────────────────────
 * Every decoder layer of one token in one launch: the per-layer loop of
 * forwardOneModel (src/model/forward.zig:260-316) -- for each layer
 * lt_attn_block (stacked Q/K/V) followed by lt_moe_block (router + Q4_K
 * experts) or lt_ffn_block (dense SwiGLU) -- as one persistent kernel.  The
 * layers hand over inside the kernel and the next layer's static weights are
 * copied while the current one runs, so a batch-1 step pays no kernel
 * boundary per half-layer.  Same results as the per-layer entry points (bit
 * for bit up to 256 cached positions, where no head is split across CTAs).
 * Measured on one B200 (config 2): 2.45 ms per token against 2.29 ms for the
 * per-layer entry points, whose phases run shorter; kept as an alternative
 * path (the host decoder uses it with LLMTOY_STACK=1).
 *
 * Shapes the kernel takes (otherwise lt_stack_create returns
 * LT_EUNSUPPORTED_TYPE and the caller keeps the per-layer calls): head_dim 64
 * or 128, no sliding window and no V norm; Q8_0 wqkv and wo; a MoE FFN with an
 * F32 router over at most num_SMs experts and Q4_K gate/up/down, or a dense
 * FFN with Q8_0 gate/up/down; every layer the same kind, types and shapes. */
typedef struct lt_stack lt_stack;
typedef struct lt_stack_layer {
    const lt_tensor *wqkv;                 /* [nq + 2 nkv][d] stacked Q, K, V rows */
    const lt_tensor *wo;                   /* [d][nq] */
    const float *attn_norm, *ffn_norm;     /* device [d] */
    const float *q_norm, *k_norm;          /* device [head_dim] or NULL */
    const float *qkv_bias;                 /* device [nq + 2 nkv] or NULL */
    void *k_cache, *v_cache;               /* this layer's caches, [kv_cap][nkv] (cfg->kv_f16: f16) */
    const lt_tensor *router;               /* F32 [E][d]; NULL: a dense FFN */
    const lt_tensor *gate, *up, *down;     /* [E][F][d], [E][F][d], [E][d][F] (2-D when dense) */
} lt_stack_layer;

/* Checks the layers, copies their descriptors to the device and allocates the
 * stack's scratch (not while capturing).  k: experts per token (MoE);
 * norm_topk: renormalise the selected weights; eps: the layer RMSNorms'. */
lt_status lt_stack_create(lt_ctx *ctx, const lt_attn_cfg *cfg, uint32_t d_model, const lt_stack_layer *layers,
                          uint32_t n_layers, uint32_t k, int act, int norm_topk, float eps, lt_stack **out);
/* dev_x[d] <- the stack applied to dev_x at position *dev_pos (asynchronous on
 * the context's stream; capturable).  One stack's launches must not overlap. */
lt_status lt_stack_run(lt_ctx *ctx, const lt_stack *stack, float *dev_x, const uint32_t *dev_pos);
lt_status lt_stack_free(lt_ctx *ctx, lt_stack *stack);

/* L2 prefetch hint: the next lt_attn_block, or single-token lt_moe_block /
 * lt_moe_forward, launched on this context starts by prefetching these
 * tensors into L2 (a later op's weights, fetched while this one waits on its
 * own dependency chain).  Either may be NULL; the hint is used once. */
lt_status lt_prefetch_next(lt_ctx *ctx, const lt_tensor *a, const lt_tensor *b);

/* The dense FFN block of a decoder layer (forward.zig:307-312):
 * out = (residual ? x : 0) + down . (act(gate . xn) * (up . xn)),
 * xn = rmsnorm(x) * norm_w, for 2-D gate/up [F][d] and down [d][F].
 * dev_out may alias dev_x. */
lt_status lt_ffn_block(lt_ctx *ctx, const lt_tensor *gate, const lt_tensor *up, const lt_tensor *down,
                       int act, const float *dev_norm_w, float eps, const float *dev_x, uint32_t ntok,
                       int residual, float *dev_out);

/* Gemma 4 layer glue on ntok rows of n values (src/model/gemma4/forward.zig):
 *   lt_scale        x *= s                                   (:117-120 embedding, :531 layer_output_scale)
 *   lt_add_rmsnorm  x += rmsnorm(y) * w                      (:329-333 post_attention_norm)
 *   lt_norm_pair    a = rmsnorm(x) * w, b = x * rms_inv * gs * g   (:401-410, math.zig:51-82)
 *   lt_ffn_tail     m = rmsnorm(m) * w2; x = (x + rmsnorm(f' + m) * w) * los   (:520-532),
 *                   f' = rmsnorm(f) * w1 (post_ffw_norm_1, :396), or f when w1 is NULL
 *   lt_softcap      x = tanh(x / cap) * cap over n values   (:560-564) */
lt_status lt_scale(lt_ctx *ctx, float *dev_x, uint32_t n, uint32_t ntok, float s);
lt_status lt_add_rmsnorm(lt_ctx *ctx, const float *dev_y, const float *dev_w, float eps, uint32_t n,
                         uint32_t ntok, float *dev_x);
lt_status lt_norm_pair(lt_ctx *ctx, const float *dev_x, const float *dev_w, const float *dev_g, float gs,
                       float eps, uint32_t n, uint32_t ntok, float *dev_a, float *dev_b);
lt_status lt_ffn_tail(lt_ctx *ctx, const float *dev_f, const float *dev_w1, float *dev_m, const float *dev_w2,
                      const float *dev_w, float los, float eps, uint32_t n, uint32_t ntok, float *dev_x);
lt_status lt_softcap(lt_ctx *ctx, float *dev_x, uint64_t n, float cap);

/* greedy (sample.zig:11-17) as the last op of a decode step: with
 * p = *dev_pos, dev_tokens[p + 1] = argmax(logits) unless p + 1 is still a
 * prompt position (< *dev_n_prompt); then *dev_pos = p + 1. */
lt_status lt_greedy_step(lt_ctx *ctx, const float *dev_logits, uint32_t n, uint32_t *dev_tokens,
                         uint32_t *dev_pos, const uint32_t *dev_n_prompt);

/* sample (src/model/sample.zig:27-183) as the last op of a decode step, like
 * lt_greedy_step: temperature 0 is greedy; top_k in 1..256 takes the
 * reference's fast path (sampleTopK) with optional top_p; otherwise softmax,
 * top-k threshold, top-p cut, renormalisation and a multinomial draw.  The
 * generator is std.Random.DefaultPrng (xoshiro256++, four 64-bit words in
 * dev_rng_state, seeded by lt_rng_seed) with Random.float(f32); it advances
 * only on sampled positions.  Scratch: n floats of the context arena. */
typedef struct lt_sample_params {
    float temperature;   /* 0: greedy */
    uint32_t top_k;      /* 0: off */
    float top_p;         /* 1: off */
} lt_sample_params;
lt_status lt_sample_step(lt_ctx *ctx, const float *dev_logits, uint32_t n, const lt_sample_params *params,
                         uint64_t *dev_rng_state, uint32_t *dev_tokens, uint32_t *dev_pos,
                         const uint32_t *dev_n_prompt);
/* DefaultPrng.init(seed): the four xoshiro256++ words from SplitMix64 (host). */
void lt_rng_seed(uint64_t seed, uint64_t state_out[4]);

/* ── host-buffer entry points (synchronous) ─────────────────────────────────
 * Same semantics with HOST vectors, copies included: the shape of the
 * reference's own CPU calls, for callers that keep activations on the host. */

/* quantMatvec(out, mat_data, mat_type, vec, rows, cols, row_buf)
 * (src/ops/math.zig:133): host vec[cols] -> host out[rows]. */
lt_status lt_quant_matvec_host(lt_ctx *ctx, float *out, const lt_tensor *mat,
                               uint32_t expert, const float *vec, uint64_t rows,
                               uint64_t cols);

/* moeForward on host vectors: x[ntok][d] -> out[ntok][d]; ids/w nullable. */
lt_status lt_moe_forward_host(lt_ctx *ctx, const lt_tensor *router, const lt_tensor *gate,
                              const lt_tensor *up, const lt_tensor *down, int act,
                              int norm_topk, const float *expert_scale_host,
                              const float *x, uint32_t ntok, uint32_t k, float *out,
                              uint32_t *ids, float *w);

#ifdef __cplusplus
}
#endif
#endif
