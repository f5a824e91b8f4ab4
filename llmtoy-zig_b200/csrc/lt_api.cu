// lt_api.cu — the C ABI declared in include/llmtoy_cuda.h.
//
// Host side of the backend: context and stream, weight upload (GGUF rows at a
// 16-byte device pitch), a scratch arena for intermediate activations, argument
// checking, and the op entry points that launch the kernels in lt_kernels.cu.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "llmtoy_cuda.h"
#include "lt_common.cuh"
#include "lt_internal.h"

struct lt_tensor {
    lt::DevMat m;
    void *dev;
    size_t dev_bytes;
    uint64_t total_rows;
};

struct lt_ctx {
    int device = 0;
    cudaStream_t own = nullptr;
    cudaStream_t stream = nullptr;
    std::string err;
    int num_sms = 0;
    bool pdl = true;
    bool decode_kernel = true;       // single-token MoE blocks run as one persistent kernel
    uint32_t tc_min_tokens = 64;     // batches of at least this many tokens use the tensor-core expert GEMM
    int *dev_err = nullptr;          // device error word written by kernels
    uint8_t *dec_sync = nullptr;     // counters and tagged logits of the persistent decode kernel
    uint8_t *attn_sync = nullptr;    // epoch and barrier counters of the attention-block kernel
    bool attn_block = true;          // single-token attention halves run as one persistent kernel
    const uint8_t *pf[2] = {nullptr, nullptr};  // L2 prefetch hint for the next block kernel
    uint64_t pf_bytes[2] = {0, 0};
    float *ones = nullptr;           // n_const slot weights of 1 (dense FFN blocks)
    uint32_t *zeros = nullptr;       // n_const expert ids of 0
    size_t n_const = 0;
    uint8_t *scratch = nullptr;      // activation scratch arena
    size_t scratch_bytes = 0;
    uint32_t *counters = nullptr;    // zero-initialised, kernels leave them zero
    size_t n_counters = 0;
    uint8_t *pinned = nullptr;       // pinned staging for the host-buffer entry points
    size_t pinned_bytes = 0;
    bool capturing = false;          // between lt_capture_begin and lt_capture_end
    cudaStream_t cap_user = nullptr; // the caller's stream while a capture runs on `own`
    cudaEvent_t cap_ev = nullptr;    // joins `own` to the caller's stream for such a capture
    lt::Profiler prof;
};

struct lt_graph {
    cudaGraph_t graph;
    cudaGraphExec_t exec;
};

int lt::ctx_device(const lt_ctx *ctx) { return ctx->device; }
cudaStream_t lt::ctx_stream(const lt_ctx *ctx) { return ctx->stream; }

struct lt_stack {
    lt::StackParams p;
    void *dev_layers = nullptr;  // lt::StackLayerDev[n_layers]
    uint8_t *scratch = nullptr;  // activations between phases, then the zeroed sync block
    size_t scratch_bytes = 0;
};

namespace {

lt_status fail(lt_ctx *ctx, lt_status st, const char *fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        ctx->err = buf;
    }
    return st;
}

lt_status cuda_fail(lt_ctx *ctx, cudaError_t e, const char *what) {
    if (e == cudaErrorMemoryAllocation)
        return fail(ctx, LT_ENOMEM, "%s: %s", what, cudaGetErrorString(e));
    return fail(ctx, LT_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define LT_CUDA(ctx, call, what)                              \
    do {                                                      \
        cudaError_t e_ = (call);                              \
        if (e_ != cudaSuccess) return cuda_fail(ctx, e_, what); \
    } while (0)

lt::LaunchCfg cfg_of(lt_ctx *ctx) {
    lt::LaunchCfg c;
    c.stream = ctx->stream;
    // No programmatic dependent launch on the default streams (legacy or
    // per-thread): only on explicit streams.
    c.pdl = ctx->pdl && ctx->stream != cudaStreamLegacy && ctx->stream != cudaStreamPerThread &&
            ctx->stream != nullptr;
    c.dev_err = ctx->dev_err;
    c.num_sms = ctx->num_sms;
    c.prof = &ctx->prof;
    return c;
}

lt_status enter(lt_ctx *ctx) {
    if (!ctx) return LT_EINVAL;
    ctx->err.clear();
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaSetDevice");
    return LT_OK;
}

// Entry points that copy or synchronise cannot be recorded into a graph.
lt_status enter_uncaptured(lt_ctx *ctx, const char *what) {
    lt_status st = enter(ctx);
    if (st == LT_OK && ctx->capturing) return fail(ctx, LT_EINVAL, "%s: not allowed while capturing", what);
    return st;
}

// Grow the scratch arena; waits for the stream first so nothing in flight
// still uses the old buffer.
lt_status ensure_scratch(lt_ctx *ctx, size_t bytes) {
    if (bytes <= ctx->scratch_bytes) return LT_OK;
    if (ctx->capturing)
        return fail(ctx, LT_EINVAL, "op needs %zu scratch bytes while capturing: call lt_reserve first", bytes);
    LT_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    if (ctx->scratch) cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
    bytes = (bytes + (1u << 20) - 1) & ~((size_t)(1u << 20) - 1);
    LT_CUDA(ctx, cudaMalloc(&ctx->scratch, bytes), "cudaMalloc(scratch)");
    ctx->scratch_bytes = bytes;
    return LT_OK;
}

lt_status ensure_counters(lt_ctx *ctx, size_t n) {
    if (n <= ctx->n_counters) return LT_OK;
    if (ctx->capturing) return fail(ctx, LT_EINVAL, "op needs more counters while capturing: call lt_reserve first");
    LT_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    if (ctx->counters) cudaFree(ctx->counters);
    ctx->counters = nullptr;
    ctx->n_counters = 0;
    n = (n + 4095) & ~(size_t)4095;
    LT_CUDA(ctx, cudaMalloc(&ctx->counters, n * 4), "cudaMalloc(counters)");
    LT_CUDA(ctx, cudaMemset(ctx->counters, 0, n * 4), "cudaMemset(counters)");
    ctx->n_counters = n;
    return LT_OK;
}

void clear_prefetch(lt_ctx *ctx) {
    ctx->pf[0] = ctx->pf[1] = nullptr;
    ctx->pf_bytes[0] = ctx->pf_bytes[1] = 0;
}

// Constant slot weights (1) and expert ids (0) for n tokens.
lt_status ensure_consts(lt_ctx *ctx, size_t n) {
    if (n <= ctx->n_const) return LT_OK;
    if (ctx->capturing) return fail(ctx, LT_EINVAL, "dense FFN for %zu tokens while capturing: run it once first", n);
    LT_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    if (ctx->ones) cudaFree(ctx->ones);
    if (ctx->zeros) cudaFree(ctx->zeros);
    ctx->ones = nullptr;
    ctx->zeros = nullptr;
    ctx->n_const = 0;
    n = (n + 1023) & ~(size_t)1023;
    LT_CUDA(ctx, cudaMalloc(&ctx->ones, n * 4), "cudaMalloc(ones)");
    LT_CUDA(ctx, cudaMalloc(&ctx->zeros, n * 4), "cudaMalloc(zeros)");
    LT_CUDA(ctx, cudaMemsetAsync(ctx->zeros, 0, n * 4, ctx->stream), "cudaMemsetAsync");
    LT_CUDA(ctx, lt::launch_fill_f32(ctx->stream, ctx->ones, n, 1.0f), "fill");
    ctx->n_const = n;
    return LT_OK;
}

lt_status ensure_pinned(lt_ctx *ctx, size_t bytes) {
    if (bytes <= ctx->pinned_bytes) return LT_OK;
    if (ctx->pinned) cudaFreeHost(ctx->pinned);
    ctx->pinned = nullptr;
    ctx->pinned_bytes = 0;
    bytes = (bytes + 65535) & ~(size_t)65535;
    LT_CUDA(ctx, cudaMallocHost(&ctx->pinned, bytes), "cudaMallocHost");
    ctx->pinned_bytes = bytes;
    return LT_OK;
}

size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

bool quantized(uint32_t t) { return lt::is_quant_type(t); }

lt_status check_kernel_shape(lt_ctx *ctx, const lt::DevMat &m, const char *what) {
    if (quantized(m.type)) {
        if (lt::is_k_type(m.type) && m.cols % 256 != 0)
            return fail(ctx, LT_EINVAL, "%s: K-quant cols %llu not a multiple of 256", what,
                        (unsigned long long)m.cols);
        if (m.cols % 32 != 0)
            return fail(ctx, LT_EINVAL, "%s: cols %llu not a multiple of 32", what, (unsigned long long)m.cols);
        if (m.cols > 65536) return fail(ctx, LT_EINVAL, "%s: cols %llu too large", what, (unsigned long long)m.cols);
    }
    return LT_OK;
}

// MoE scratch layout for T tokens, k slots, E experts, model width d and
// expert width F: router outputs, the quantised expert input xq [T] and the
// quantised expert activations hq [T*k], the dispatch plan.
struct MoeScratch {
    uint32_t *ids;
    float *w;
    float *logits;
    uint8_t *xq;
    uint64_t xq_pitch;
    uint8_t *hq;
    uint64_t hq_pitch;
    float *hf;  // f32 h rows, staged before quantisation
    uint8_t *himg;  // single-token decode kernel: quantised h slot images
    float *xn;      // f32 normalised expert input rows (tensor-core path)
    uint8_t *gemm;  // tensor-core path scratch (lt_moe_gemm.cu)
    lt::MoePlan plan;
    size_t bytes;
    size_t counters;  // block counters needed past kMoeCounterBase
};

MoeScratch moe_layout(uint8_t *base, uint32_t T, uint32_t k, uint32_t E, uint64_t d, uint64_t F,
                      size_t gemm_bytes = 0) {
    MoeScratch s;
    size_t off = 0;
    auto take = [&](size_t b) {
        uint8_t *p = base ? base + off : nullptr;
        off += al256(b);
        return p;
    };
    const size_t P = (size_t)T * k;
    s.xq_pitch = lt::qact_row_pitch(d);
    s.hq_pitch = lt::qact_row_pitch(F);
    s.ids = (uint32_t *)take(P * 4);
    s.w = (float *)take(P * 4);
    s.xq = take((size_t)T * s.xq_pitch);
    s.hq = take(P * s.hq_pitch);
    s.hf = (float *)take(P * F * 4);
    s.himg = take(P * lt::moe_decode_img_bytes(F));
    s.xn = gemm_bytes ? (float *)take((size_t)T * d * 4) : nullptr;
    s.gemm = gemm_bytes ? take(gemm_bytes) : nullptr;
    s.counters = P * (F / 32);
    s.logits = (float *)take((size_t)T * E * 4);
    s.plan.n_active = (uint32_t *)take(4);
    s.plan.act_e = (uint32_t *)take((size_t)E * 4);
    s.plan.act_off = (uint32_t *)take((size_t)E * 4);
    s.plan.act_cnt = (uint32_t *)take((size_t)E * 4);
    s.plan.pos_pair = (uint32_t *)take(P * 4);
    s.plan.pair_pos = (uint32_t *)take(P * 4);
    s.bytes = off;
    return s;
}

lt_status launched(lt_ctx *ctx, cudaError_t e, const char *what) {
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(ctx, e, what);
    return LT_OK;
}

}  // namespace

extern "C" {

int lt_api_version(void) { return LT_API_VERSION; }

const char *lt_status_string(lt_status s) {
    switch (s) {
    case LT_OK: return "ok";
    case LT_EINVAL: return "invalid argument";
    case LT_EUNSUPPORTED_TYPE: return "unsupported ggml type";
    case LT_ENOMEM: return "out of device memory";
    case LT_ECUDA: return "CUDA error";
    case LT_ETIMEOUT: return "device wait timed out";
    case LT_ENODEV: return "no sm_100 device";
    }
    return "unknown status";
}

const char *lt_last_error(const lt_ctx *ctx) { return ctx ? ctx->err.c_str() : "null context"; }

lt_status lt_init(int device, lt_ctx **out) {
    if (!out) return LT_EINVAL;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return LT_ENODEV;
    }
    if (device < 0 || device >= n) return LT_ENODEV;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return LT_ENODEV;
    if (prop.major != 10) return LT_ENODEV;  // kernels are built for sm_100a only
    lt_ctx *ctx = new lt_ctx();
    ctx->device = device;
    ctx->num_sms = prop.multiProcessorCount;
    const char *pdl = getenv("LLMTOY_PDL");
    ctx->pdl = !(pdl && strcmp(pdl, "0") == 0);
    const char *dk = getenv("LLMTOY_DECODE_KERNEL");
    ctx->decode_kernel = !(dk && strcmp(dk, "0") == 0);
    const char *ab = getenv("LLMTOY_ATTN_BLOCK");  // 0: attention halves as separate kernels
    ctx->attn_block = !(ab && strcmp(ab, "0") == 0);
    const char *tc = getenv("LLMTOY_TC_MIN_TOKENS");  // 0 turns the tensor-core expert GEMM off
    if (tc) ctx->tc_min_tokens = (uint32_t)strtoul(tc, nullptr, 10);
    lt_status st = LT_OK;
    if (cudaSetDevice(device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ctx->own, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&ctx->dev_err, 4) != cudaSuccess || cudaMemset(ctx->dev_err, 0, 4) != cudaSuccess ||
        cudaMalloc(&ctx->dec_sync, lt::kDecodeSyncBytes) != cudaSuccess ||
        cudaMemset(ctx->dec_sync, 0, lt::kDecodeSyncBytes) != cudaSuccess ||
        cudaMalloc(&ctx->attn_sync, lt::kAttnSyncBytes) != cudaSuccess ||
        cudaMemset(ctx->attn_sync, 0, lt::kAttnSyncBytes) != cudaSuccess) {
        st = LT_ECUDA;
    }
    ctx->stream = ctx->own;
    if (st == LT_OK) st = ensure_counters(ctx, 4096);
    if (st != LT_OK) {
        lt_free(ctx);
        return st;
    }
    *out = ctx;
    return LT_OK;
}

void lt_free(lt_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->capturing) {
        cudaGraph_t g = nullptr;
        cudaStreamEndCapture(ctx->stream, &g);
        if (g) cudaGraphDestroy(g);
    }
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    ctx->prof.destroy();
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->counters) cudaFree(ctx->counters);
    if (ctx->dev_err) cudaFree(ctx->dev_err);
    if (ctx->dec_sync) cudaFree(ctx->dec_sync);
    if (ctx->attn_sync) cudaFree(ctx->attn_sync);
    if (ctx->ones) cudaFree(ctx->ones);
    if (ctx->zeros) cudaFree(ctx->zeros);
    if (ctx->pinned) cudaFreeHost(ctx->pinned);
    if (ctx->cap_ev) cudaEventDestroy(ctx->cap_ev);
    if (ctx->own) cudaStreamDestroy(ctx->own);
    delete ctx;
}

lt_status lt_set_stream(lt_ctx *ctx, void *cuda_stream) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    ctx->stream = cuda_stream ? (cudaStream_t)cuda_stream : ctx->own;
    return LT_OK;
}

lt_status lt_profile_enable(lt_ctx *ctx, int on) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (ctx->capturing) return fail(ctx, LT_EINVAL, "lt_profile_enable: not while capturing");
    ctx->prof.on = on != 0;
    return LT_OK;
}

lt_status lt_profile_read(lt_ctx *ctx, uint32_t index, const char **label, uint64_t *count, double *total_ms,
                          double *min_ms, double *max_ms) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (ctx->capturing) return fail(ctx, LT_EINVAL, "lt_profile_read: not while capturing");
    LT_CUDA(ctx, ctx->prof.flush(), "profile events");
    if (index >= (uint32_t)ctx->prof.n_agg) return LT_EINVAL;
    const lt::Profiler::Agg &a = ctx->prof.agg[index];
    if (label) *label = a.label;
    if (count) *count = a.count;
    if (total_ms) *total_ms = a.total_ms;
    if (min_ms) *min_ms = a.min_ms;
    if (max_ms) *max_ms = a.max_ms;
    return LT_OK;
}

lt_status lt_profile_reset(lt_ctx *ctx) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    LT_CUDA(ctx, ctx->prof.flush(), "profile events");
    ctx->prof.reset();
    return LT_OK;
}

lt_status lt_capture_begin(lt_ctx *ctx) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (ctx->capturing) return fail(ctx, LT_EINVAL, "lt_capture_begin: already capturing");
    if (ctx->prof.on) return fail(ctx, LT_EINVAL, "lt_capture_begin: turn profiling off first");
    ctx->cap_user = nullptr;
    if (ctx->stream == cudaStreamLegacy || ctx->stream == cudaStreamPerThread) {
        // the default streams cannot be captured: capture on the context's own
        // stream, ordered after the caller's work; the graph launches on any stream
        if (!ctx->cap_ev) LT_CUDA(ctx, cudaEventCreateWithFlags(&ctx->cap_ev, cudaEventDisableTiming), "cudaEventCreate");
        LT_CUDA(ctx, cudaEventRecord(ctx->cap_ev, ctx->stream), "cudaEventRecord");
        LT_CUDA(ctx, cudaStreamWaitEvent(ctx->own, ctx->cap_ev, 0), "cudaStreamWaitEvent");
        ctx->cap_user = ctx->stream;
        ctx->stream = ctx->own;
    }
    cudaError_t e = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) {
        if (ctx->cap_user) ctx->stream = ctx->cap_user;
        ctx->cap_user = nullptr;
        return cuda_fail(ctx, e, "cudaStreamBeginCapture");
    }
    ctx->capturing = true;
    return LT_OK;
}

lt_status lt_capture_end(lt_ctx *ctx, lt_graph **out) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!ctx->capturing) return fail(ctx, LT_EINVAL, "lt_capture_end: not capturing");
    ctx->capturing = false;
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(ctx->stream, &g);
    if (ctx->cap_user) ctx->stream = ctx->cap_user;
    ctx->cap_user = nullptr;
    LT_CUDA(ctx, ce, "cudaStreamEndCapture");
    if (!out) {
        cudaGraphDestroy(g);
        return fail(ctx, LT_EINVAL, "lt_capture_end: null output");
    }
    cudaGraphExec_t ex = nullptr;
    cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
    if (e != cudaSuccess) {
        cudaGraphDestroy(g);
        return cuda_fail(ctx, e, "cudaGraphInstantiate");
    }
    *out = new lt_graph{g, ex};
    return LT_OK;
}

lt_status lt_graph_launch(lt_ctx *ctx, const lt_graph *graph) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!graph) return fail(ctx, LT_EINVAL, "lt_graph_launch: null graph");
    LT_CUDA(ctx, cudaGraphLaunch(graph->exec, ctx->stream), "cudaGraphLaunch");
    return LT_OK;
}

lt_status lt_graph_free(lt_ctx *ctx, lt_graph *graph) {
    if (!graph) return LT_OK;
    if (ctx) cudaSetDevice(ctx->device);
    cudaGraphExecDestroy(graph->exec);
    cudaGraphDestroy(graph->graph);
    delete graph;
    return LT_OK;
}

lt_status lt_sync(lt_ctx *ctx) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (ctx->capturing) return fail(ctx, LT_EINVAL, "lt_sync: not while capturing");
    LT_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    int h = 0;
    LT_CUDA(ctx, cudaMemcpy(&h, ctx->dev_err, 4, cudaMemcpyDeviceToHost), "read device error word");
    if (h != 0) {
        cudaMemset(ctx->dev_err, 0, 4);
        if (h == lt::DEV_ERR_BAD_INDEX) return fail(ctx, LT_EINVAL, "a device-side index was out of range");
        return fail(ctx, LT_ETIMEOUT, "a device-side wait gave up (code %d)", h);
    }
    return LT_OK;
}

lt_status lt_reserve(lt_ctx *ctx, uint32_t max_tokens, uint32_t max_k, uint64_t max_d_model,
                     uint64_t max_d_expert) {
    lt_status st = enter_uncaptured(ctx, "lt_reserve");
    if (st != LT_OK) return st;
    const size_t gemm = max_tokens > 1 ? lt::moe_gemm_scratch(max_tokens, max_k, lt::kRouterMaxE, max_d_model,
                                                               max_d_expert)
                                       : 0;
    const size_t moe =
        moe_layout(nullptr, max_tokens, max_k, lt::kRouterMaxE, max_d_model, max_d_expert, gemm).bytes;
    const size_t io = 2 * al256((size_t)max_tokens * max_d_model * 4) + 2 * al256((size_t)max_tokens * max_k * 4) +
                      al256((size_t)lt::kRouterMaxE * 4);
    const size_t qmv = al256((size_t)max_tokens * lt::qact_row_pitch(max_d_model > max_d_expert ? max_d_model
                                                                                                : max_d_expert));
    st = ensure_scratch(ctx, (moe + io > qmv ? moe + io : qmv));
    if (st != LT_OK) return st;
    return ensure_counters(ctx, lt::kMoeCounterBase + (size_t)max_tokens * max_k * (max_d_expert / 32) + max_tokens);
}

uint64_t lt_row_bytes(uint32_t ggml_type, uint64_t cols) {
    if (!lt::type_supported(ggml_type)) return 0;
    return lt::row_bytes_of(ggml_type, cols);
}

static lt_status upload_impl(lt_ctx *ctx, const void *src, bool src_on_device, size_t nbytes, uint32_t type,
                             uint64_t rows, uint64_t cols, uint32_t n_experts, lt_tensor **out) {
    lt_status st = enter_uncaptured(ctx, "lt_upload");
    if (st != LT_OK) return st;
    if (!out || !src) return fail(ctx, LT_EINVAL, "lt_upload: null pointer");
    *out = nullptr;
    if (!lt::type_supported(type)) return fail(ctx, LT_EUNSUPPORTED_TYPE, "lt_upload: ggml type %u", type);
    const uint32_t be = lt::block_elems_of(type);
    if (rows == 0 || cols == 0 || cols % be != 0)
        return fail(ctx, LT_EINVAL, "lt_upload: cols %llu not a multiple of the %u-element block",
                    (unsigned long long)cols, be);
    const uint64_t total_rows = rows * (n_experts ? n_experts : 1);
    const uint64_t rb = lt::row_bytes_of(type, cols);
    if ((uint64_t)nbytes != total_rows * rb)
        return fail(ctx, LT_EINVAL, "lt_upload: %zu bytes given, shape needs %llu", nbytes,
                    (unsigned long long)(total_rows * rb));
    const uint64_t pitch = (rb + 15) & ~(uint64_t)15;
    lt_tensor *t = new lt_tensor();
    t->total_rows = total_rows;
    t->dev_bytes = (size_t)(total_rows * pitch) + 256;  // slack: decoders read a little past a row
    cudaError_t e = cudaMalloc(&t->dev, t->dev_bytes);
    if (e != cudaSuccess) {
        delete t;
        return cuda_fail(ctx, e, "cudaMalloc(tensor)");
    }
    e = cudaMemsetAsync(t->dev, 0, t->dev_bytes, ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpy2DAsync(t->dev, pitch, src, rb, rb, total_rows,
                              src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        cudaFree(t->dev);
        delete t;
        return cuda_fail(ctx, e, "upload copy");
    }
    t->m.data = (const uint8_t *)t->dev;
    t->m.type = type;
    t->m.rows = rows;
    t->m.cols = cols;
    t->m.row_bytes = rb;
    t->m.pitch = pitch;
    t->m.n_experts = n_experts;
    *out = t;
    return LT_OK;
}

lt_status lt_upload(lt_ctx *ctx, const void *host_bytes, size_t nbytes, uint32_t ggml_type, uint64_t rows,
                    uint64_t cols, uint32_t n_experts, lt_tensor **out) {
    return upload_impl(ctx, host_bytes, false, nbytes, ggml_type, rows, cols, n_experts, out);
}

lt_status lt_upload_from_device(lt_ctx *ctx, const void *dev_bytes, size_t nbytes, uint32_t ggml_type,
                                uint64_t rows, uint64_t cols, uint32_t n_experts, lt_tensor **out) {
    return upload_impl(ctx, dev_bytes, true, nbytes, ggml_type, rows, cols, n_experts, out);
}

lt_status lt_tensor_download(lt_ctx *ctx, const lt_tensor *t, void *host_bytes, size_t nbytes) {
    lt_status st = enter_uncaptured(ctx, "lt_tensor_download");
    if (st != LT_OK) return st;
    if (!t || !host_bytes) return fail(ctx, LT_EINVAL, "lt_tensor_download: null pointer");
    if ((uint64_t)nbytes != t->total_rows * t->m.row_bytes)
        return fail(ctx, LT_EINVAL, "lt_tensor_download: buffer is %zu bytes, tensor %llu", nbytes,
                    (unsigned long long)(t->total_rows * t->m.row_bytes));
    LT_CUDA(ctx,
            cudaMemcpy2DAsync(host_bytes, t->m.row_bytes, t->dev, t->m.pitch, t->m.row_bytes, t->total_rows,
                              cudaMemcpyDeviceToHost, ctx->stream),
            "download copy");
    LT_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    return LT_OK;
}

lt_status lt_tensor_describe(const lt_tensor *t, lt_tensor_desc *out) {
    if (!t || !out) return LT_EINVAL;
    out->ggml_type = t->m.type;
    out->n_experts = t->m.n_experts;
    out->rows = t->m.rows;
    out->cols = t->m.cols;
    out->row_bytes = t->m.row_bytes;
    out->row_pitch = t->m.pitch;
    return LT_OK;
}

lt_status lt_tensor_free(lt_ctx *ctx, lt_tensor *t) {
    if (!t) return LT_OK;
    if (ctx) {
        cudaSetDevice(ctx->device);
        cudaStreamSynchronize(ctx->stream);
    }
    cudaFree(t->dev);
    delete t;
    return LT_OK;
}

lt_status lt_dequant(lt_ctx *ctx, const lt_tensor *t, uint64_t row0, uint64_t nrows, float *dev_out) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!t || (!dev_out && nrows)) return fail(ctx, LT_EINVAL, "lt_dequant: null pointer");
    if (row0 + nrows > t->total_rows || row0 + nrows < row0)
        return fail(ctx, LT_EINVAL, "lt_dequant: rows [%llu,+%llu) out of %llu", (unsigned long long)row0,
                    (unsigned long long)nrows, (unsigned long long)t->total_rows);
    return launched(ctx, lt::launch_dequant(cfg_of(ctx), t->m, row0, nrows, dev_out), "dequant");
}

lt_status lt_quantize_q8_1(lt_ctx *ctx, const float *dev_x, uint64_t n, int x4, uint8_t *dev_out) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (n % 32 != 0) return fail(ctx, LT_EINVAL, "lt_quantize_q8_1: n=%llu not a multiple of 32", (unsigned long long)n);
    if (n && (!dev_x || !dev_out)) return fail(ctx, LT_EINVAL, "lt_quantize_q8_1: null pointer");
    return launched(ctx, lt::launch_quantize_q8_1(cfg_of(ctx), dev_x, n, x4 != 0, dev_out), "quantize_q8_1");
}

lt_status lt_dequant_q8_1(lt_ctx *ctx, const uint8_t *dev_q, uint64_t n, int x4, float *dev_out) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (n % 32 != 0) return fail(ctx, LT_EINVAL, "lt_dequant_q8_1: n=%llu not a multiple of 32", (unsigned long long)n);
    if (n && (!dev_q || !dev_out)) return fail(ctx, LT_EINVAL, "lt_dequant_q8_1: null pointer");
    return launched(ctx, lt::launch_dequant_q8_1(cfg_of(ctx), dev_q, n, x4 != 0, dev_out), "dequant_q8_1");
}

static lt_status qmatvec_impl(lt_ctx *ctx, const lt_tensor *w, uint32_t expert, const float *dev_x, float *dev_y,
                              uint32_t ntok, const float *dev_add) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!w || !dev_x || !dev_y) return fail(ctx, LT_EINVAL, "lt_qmatvec: null pointer");
    if (ntok == 0) return LT_OK;
    if (expert >= (w->m.n_experts ? w->m.n_experts : 1u))
        return fail(ctx, LT_EINVAL, "lt_qmatvec: expert %u out of range", expert);
    if ((st = check_kernel_shape(ctx, w->m, "lt_qmatvec")) != LT_OK) return st;
    if (w->m.rows > 0xffffffffull) return fail(ctx, LT_EINVAL, "lt_qmatvec: too many rows");
    const lt::LaunchCfg c = cfg_of(ctx);
    // f32/f16 rows; or one token over few enough CTAs that each quantising it
    // costs less than a separate quantiser launch; or the persistent streaming
    // kernel (one CTA per SM) for a large matrix such as an lm_head
    if (!quantized(w->m.type) ||
        (ntok == 1 && (lt::qmv_ctas(w->m) <= 2u * (uint32_t)ctx->num_sms ||
                       lt::qmv_streams(w->m, 1, ctx->num_sms))))
        return launched(ctx, lt::launch_qmatvec(c, w->m, expert, nullptr, 0, dev_x, dev_y, ntok, dev_add), "qmatvec");
    const uint64_t qp = lt::qact_row_pitch(w->m.cols);
    if ((st = ensure_scratch(ctx, al256((size_t)ntok * qp))) != LT_OK) return st;
    uint8_t *xq = ctx->scratch;
    st = launched(ctx, lt::launch_quantize(c, dev_x, (uint32_t)w->m.cols, ntok, xq, qp), "quantize");
    if (st != LT_OK) return st;
    return launched(ctx, lt::launch_qmatvec(c, w->m, expert, xq, qp, dev_x, dev_y, ntok, dev_add), "qmatvec");
}

lt_status lt_qmatvec_multi(lt_ctx *ctx, uint32_t n, const lt_tensor *const *w, const float *dev_x,
                           const float *dev_norm_w, float eps, float *const *dev_y) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (n == 0 || n > 4 || !w || !dev_x || !dev_y) return fail(ctx, LT_EINVAL, "lt_qmatvec_multi: bad argument");
    const lt::DevMat *m[4];
    for (uint32_t i = 0; i < n; i++) {
        if (!w[i] || !dev_y[i]) return fail(ctx, LT_EINVAL, "lt_qmatvec_multi: null tensor or output %u", i);
        if (!quantized(w[i]->m.type)) return fail(ctx, LT_EUNSUPPORTED_TYPE, "lt_qmatvec_multi: tensor %u not block-quantised", i);
        if (w[i]->m.n_experts) return fail(ctx, LT_EINVAL, "lt_qmatvec_multi: tensor %u is an expert tensor", i);
        if (w[i]->m.cols != w[0]->m.cols) return fail(ctx, LT_EINVAL, "lt_qmatvec_multi: column counts differ");
        if ((st = check_kernel_shape(ctx, w[i]->m, "lt_qmatvec_multi")) != LT_OK) return st;
        m[i] = &w[i]->m;
    }
    return launched(ctx, lt::launch_qmatvec_multi(cfg_of(ctx), n, m, dev_x, dev_norm_w, eps, dev_y), "qmatvec multi");
}

lt_status lt_qmatvec(lt_ctx *ctx, const lt_tensor *w, uint32_t expert, const float *dev_x, float *dev_y,
                     uint32_t ntok) {
    return qmatvec_impl(ctx, w, expert, dev_x, dev_y, ntok, nullptr);
}

lt_status lt_rmsnorm(lt_ctx *ctx, const float *dev_x, const float *dev_w, float eps, uint32_t n, uint32_t ntok,
                     float *dev_y) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_x || !dev_w || !dev_y || n == 0) return fail(ctx, LT_EINVAL, "lt_rmsnorm: bad argument");
    if (ntok == 0) return LT_OK;
    return launched(ctx, lt::launch_rmsnorm(cfg_of(ctx), dev_x, dev_w, eps, n, ntok, dev_y), "rmsnorm");
}

lt_status lt_softmax(lt_ctx *ctx, float *dev_x, uint32_t n, uint32_t ntok) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_x || n == 0) return fail(ctx, LT_EINVAL, "lt_softmax: bad argument");
    if (ntok == 0) return LT_OK;
    return launched(ctx, lt::launch_softmax(cfg_of(ctx), dev_x, n, ntok), "softmax");
}

lt_status lt_argmax(lt_ctx *ctx, const float *dev_x, uint32_t n, uint32_t ntok, uint32_t *dev_idx) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_x || !dev_idx || n == 0) return fail(ctx, LT_EINVAL, "lt_argmax: bad argument");
    if (ntok == 0) return LT_OK;
    const size_t part = (size_t)ntok * 64;
    if ((st = ensure_scratch(ctx, al256(part * 4) * 2)) != LT_OK) return st;
    if ((st = ensure_counters(ctx, ntok)) != LT_OK) return st;
    float *pv = (float *)ctx->scratch;
    uint32_t *pi = (uint32_t *)(ctx->scratch + al256(part * 4));
    return launched(ctx, lt::launch_argmax(cfg_of(ctx), dev_x, n, ntok, dev_idx, pv, pi, ctx->counters), "argmax");
}

lt_status lt_selftest_wait(lt_ctx *ctx, uint32_t kind, uint32_t limit_us) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (kind > 2 || limit_us == 0 || limit_us > 2000000) return fail(ctx, LT_EINVAL, "lt_selftest_wait: bad argument");
    return launched(ctx, lt::launch_selftest_wait(cfg_of(ctx), (int)kind, (uint64_t)limit_us * 1000ull),
                    "selftest_wait");
}

// ── device buffers ─────────────────────────────────────────────────────────

lt_status lt_device_alloc(lt_ctx *ctx, size_t bytes, void **dev_out) {
    lt_status st = enter_uncaptured(ctx, "lt_device_alloc");
    if (st != LT_OK) return st;
    if (!dev_out) return fail(ctx, LT_EINVAL, "lt_device_alloc: null output");
    *dev_out = nullptr;
    if (bytes == 0) return fail(ctx, LT_EINVAL, "lt_device_alloc: zero bytes");
    void *p = nullptr;
    LT_CUDA(ctx, cudaMalloc(&p, bytes), "cudaMalloc");
    cudaError_t e = cudaMemsetAsync(p, 0, bytes, ctx->stream);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(ctx, e, "cudaMemsetAsync");
    }
    *dev_out = p;
    return LT_OK;
}

lt_status lt_device_free(lt_ctx *ctx, void *dev) {
    lt_status st = enter_uncaptured(ctx, "lt_device_free");
    if (st != LT_OK) return st;
    if (!dev) return LT_OK;
    LT_CUDA(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    LT_CUDA(ctx, cudaFree(dev), "cudaFree");
    return LT_OK;
}

lt_status lt_copy_to_device(lt_ctx *ctx, void *dev_dst, const void *host_src, size_t bytes) {
    lt_status st = enter_uncaptured(ctx, "lt_copy_to_device");
    if (st != LT_OK) return st;
    if (bytes == 0) return LT_OK;
    if (!dev_dst || !host_src) return fail(ctx, LT_EINVAL, "lt_copy_to_device: null pointer");
    LT_CUDA(ctx, cudaMemcpyAsync(dev_dst, host_src, bytes, cudaMemcpyHostToDevice, ctx->stream), "cudaMemcpyAsync");
    return LT_OK;
}

lt_status lt_copy_to_host(lt_ctx *ctx, void *host_dst, const void *dev_src, size_t bytes) {
    lt_status st = enter_uncaptured(ctx, "lt_copy_to_host");
    if (st != LT_OK) return st;
    if (bytes == 0) return LT_OK;
    if (!host_dst || !dev_src) return fail(ctx, LT_EINVAL, "lt_copy_to_host: null pointer");
    LT_CUDA(ctx, cudaMemcpyAsync(host_dst, dev_src, bytes, cudaMemcpyDeviceToHost, ctx->stream), "cudaMemcpyAsync");
    return LT_OK;
}

// ── decode-step ops ────────────────────────────────────────────────────────

lt_status lt_embed(lt_ctx *ctx, const lt_tensor *emb, const uint32_t *dev_tokens, const uint32_t *dev_pos,
                   float *dev_out) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!emb || !dev_tokens || !dev_pos || !dev_out) return fail(ctx, LT_EINVAL, "lt_embed: null pointer");
    if (emb->m.n_experts != 0) return fail(ctx, LT_EINVAL, "lt_embed: 3-D tensor");
    return launched(ctx, lt::launch_embed(cfg_of(ctx), emb->m, dev_tokens, dev_pos, dev_out), "embed");
}

lt_status lt_qmatvec_add(lt_ctx *ctx, const lt_tensor *w, uint32_t expert, const float *dev_x, const float *dev_add,
                         float *dev_y, uint32_t ntok) {
    if (!dev_add) {
        lt_status st = enter(ctx);
        return st != LT_OK ? st : fail(ctx, LT_EINVAL, "lt_qmatvec_add: null addend");
    }
    return qmatvec_impl(ctx, w, expert, dev_x, dev_y, ntok, dev_add);
}

static lt_status attn_geom(lt_ctx *ctx, const lt_attn_cfg *cfg, lt::AttnGeom &g, const char *what) {
    if (!cfg) return fail(ctx, LT_EINVAL, "%s: null cfg", what);
    if (cfg->head_dim != 64 && cfg->head_dim != 128 && cfg->head_dim != 256)
        return fail(ctx, LT_EINVAL, "%s: head_dim %u (64, 128 or 256)", what, cfg->head_dim);
    if (cfg->n_heads == 0 || cfg->n_kv_heads == 0 || cfg->n_heads % cfg->n_kv_heads != 0 || cfg->n_heads > 1024)
        return fail(ctx, LT_EINVAL, "%s: %u query heads over %u KV heads", what, cfg->n_heads, cfg->n_kv_heads);
    if (cfg->kv_cap == 0) return fail(ctx, LT_EINVAL, "%s: kv_cap 0", what);
    if (cfg->window > cfg->kv_cap) return fail(ctx, LT_EINVAL, "%s: window %u > kv_cap %u", what, cfg->window, cfg->kv_cap);
    g.n_heads = cfg->n_heads;
    g.n_kv = cfg->n_kv_heads;
    g.hd = cfg->head_dim;
    g.rope_neox = cfg->rope_neox ? 1u : 0u;
    g.theta = cfg->rope_theta;
    g.eps = cfg->eps;
    g.scale = cfg->scale;
    g.cap = cfg->kv_cap;
    g.window = cfg->window;
    g.v_norm = cfg->v_norm ? 1u : 0u;
    g.kv_f16 = cfg->kv_f16 ? 1u : 0u;
    return LT_OK;
}

lt_status lt_attn_prep(lt_ctx *ctx, const lt_attn_cfg *cfg, float *dev_qkv, const float *dev_q_norm,
                       const float *dev_k_norm, const uint32_t *dev_pos, void *dev_k_cache, void *dev_v_cache) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    lt::AttnGeom g;
    if ((st = attn_geom(ctx, cfg, g, "lt_attn_prep")) != LT_OK) return st;
    if (!dev_qkv || !dev_pos || !dev_k_cache || !dev_v_cache) return fail(ctx, LT_EINVAL, "lt_attn_prep: null pointer");
    return launched(ctx, lt::launch_attn_prep(cfg_of(ctx), g, dev_qkv, dev_q_norm, dev_k_norm, dev_pos, dev_k_cache,
                                              dev_v_cache),
                    "attn prep");
}

lt_status lt_attn_decode(lt_ctx *ctx, const lt_attn_cfg *cfg, const float *dev_q, const void *dev_k_cache,
                         const void *dev_v_cache, const uint32_t *dev_pos, float *dev_out) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    lt::AttnGeom g;
    if ((st = attn_geom(ctx, cfg, g, "lt_attn_decode")) != LT_OK) return st;
    if (!dev_q || !dev_k_cache || !dev_v_cache || !dev_pos || !dev_out)
        return fail(ctx, LT_EINVAL, "lt_attn_decode: null pointer");
    if ((st = ensure_scratch(ctx, lt::attn_scratch_floats(g, ctx->num_sms) * 4)) != LT_OK) return st;
    if ((st = ensure_counters(ctx, g.n_heads)) != LT_OK) return st;
    return launched(ctx, lt::launch_attn_decode(cfg_of(ctx), g, dev_q, dev_k_cache, dev_v_cache, dev_pos, dev_out,
                                                (float *)ctx->scratch, ctx->counters),
                    "attn decode");
}

lt_status lt_prefetch_next(lt_ctx *ctx, const lt_tensor *a, const lt_tensor *b) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    const lt_tensor *t[2] = {a, b};
    for (int i = 0; i < 2; i++) {
        ctx->pf[i] = t[i] ? t[i]->m.data : nullptr;
        ctx->pf_bytes[i] = t[i] ? (t[i]->dev_bytes & ~(size_t)15) : 0;
    }
    return LT_OK;
}

// The attention half of a layer: the persistent kernel when it takes the
// shape, else the same computation as separate kernels.  seg: the stacked
// Q/K/V tensor (nseg 1), or wq, wk and wv (3), or wq and wk with V = K (2).
static lt_status attn_block_impl(lt_ctx *ctx, const char *who, const lt_attn_cfg *cfg, const float *dev_x,
                                 const float *dev_norm_w, float eps, const lt_tensor *const *seg, uint32_t nseg,
                                 const float *dev_qkv_bias, const float *dev_q_norm, const float *dev_k_norm,
                                 const uint32_t *dev_pos, void *dev_k_cache, void *dev_v_cache, const lt_tensor *wo,
                                 const float *dev_post_norm, const lt_ffn_tail_in *tail, float *dev_out) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    struct Clear {
        lt_ctx *c;
        ~Clear() { clear_prefetch(c); }
    } clear{ctx};
    lt::AttnGeom g;
    if ((st = attn_geom(ctx, cfg, g, who)) != LT_OK) return st;
    if (!dev_x || !dev_norm_w || !wo || !dev_pos || !dev_k_cache || !dev_v_cache || !dev_out)
        return fail(ctx, LT_EINVAL, "%s: null argument", who);
    for (uint32_t s = 0; s < nseg; s++)
        if (!seg[s]) return fail(ctx, LT_EINVAL, "%s: null Q/K/V tensor", who);
    if (tail && (!tail->dev_f || !tail->dev_m || !tail->dev_w2 || !tail->dev_w))
        return fail(ctx, LT_EINVAL, "%s: null tail input", who);
    const uint32_t nq = g.n_heads * g.hd, nkv = g.n_kv * g.hd;
    const bool v_is_k = nseg == 2;
    const uint64_t d = wo->m.rows;
    const uint64_t want[3] = {nseg == 1 ? (uint64_t)nq + 2 * nkv : nq, nkv, nkv};
    for (uint32_t s = 0; s < nseg; s++) {
        const lt::DevMat &m = seg[s]->m;
        if (m.n_experts || m.rows != want[s] || m.cols != d)
            return fail(ctx, LT_EINVAL, "%s: Q/K/V tensor %u is %llux%llu, the heads want %llux%llu", who, s,
                        (unsigned long long)m.rows, (unsigned long long)m.cols, (unsigned long long)want[s],
                        (unsigned long long)d);
        if ((st = check_kernel_shape(ctx, m, who)) != LT_OK) return st;
    }
    if (wo->m.n_experts || wo->m.cols != nq)
        return fail(ctx, LT_EINVAL, "%s: wo %llux%llu does not fit the heads", who, (unsigned long long)wo->m.rows,
                    (unsigned long long)wo->m.cols);
    if ((st = check_kernel_shape(ctx, wo->m, who)) != LT_OK) return st;
    lt::AttnBlockParams p;
    p.g = g;
    p.d = (uint32_t)d;
    p.x = dev_x;
    p.norm_w = dev_norm_w;
    p.eps = eps;
    for (uint32_t s = 0; s < nseg; s++) p.seg[s] = seg[s]->m;
    p.nseg = nseg;
    p.v_is_k = v_is_k ? 1 : 0;
    p.wo = wo->m;
    p.bias = dev_qkv_bias;
    p.q_norm = dev_q_norm;
    p.k_norm = dev_k_norm;
    p.post_norm = dev_post_norm;
    if (tail) {
        p.tail_f = tail->dev_f;
        p.tail_w1 = tail->dev_w1;
        p.tail_m = tail->dev_m;
        p.tail_w2 = tail->dev_w2;
        p.tail_w = tail->dev_w;
        p.tail_los = tail->los;
        p.tail_eps = tail->eps;
    }
    p.pos = dev_pos;
    p.kc = dev_k_cache;
    p.vc = dev_v_cache;
    p.out = dev_out;
    size_t sf = 0;
    if (ctx->attn_block && lt::attn_block_plan(p, ctx->num_sms, &sf)) {
        if ((st = ensure_scratch(ctx, sf * 4 + 1024)) != LT_OK) return st;
        p.scratch = (float *)ctx->scratch;
        p.sync = ctx->attn_sync;
        for (int i = 0; i < 2; i++) {
            p.pf[i] = ctx->pf[i];
            p.pf_bytes[i] = ctx->pf_bytes[i];
        }
        return launched(ctx, lt::launch_attn_block(cfg_of(ctx), p), "attn block");
    }
    // the same computation as separate kernels: norm, Q/K/V, prep, attention, wo + residual (or + normed wo)
    const size_t xb_b = al256((size_t)d * 4), qkv_b = al256(((size_t)nq + 2 * nkv) * 4), att_b = al256((size_t)nq * 4);
    // [0, base): the quantised activation row of each matvec, then the attention partials
    const size_t attn_sc = lt::attn_scratch_floats(g, ctx->num_sms) * 4;
    const size_t qrow = lt::qact_row_pitch(d > nq ? d : nq);
    const size_t base = al256(attn_sc > qrow ? attn_sc : qrow);
    if ((st = ensure_scratch(ctx, base + 4 * xb_b + qkv_b + att_b)) != LT_OK) return st;
    float *xb = (float *)(ctx->scratch + base), *qkv = (float *)(ctx->scratch + base + xb_b);
    float *att = (float *)(ctx->scratch + base + xb_b + qkv_b);
    float *yb = (float *)(ctx->scratch + base + xb_b + qkv_b + att_b);
    const lt::LaunchCfg c = cfg_of(ctx);
    if (tail) {  // the tail of copies of x and m (neither is written): the block's input
        float *xt = (float *)(ctx->scratch + base + 2 * xb_b + qkv_b + att_b), *mt = xt + xb_b / 4;
        if ((st = launched(ctx, cudaMemcpyAsync(xt, dev_x, d * 4, cudaMemcpyDeviceToDevice, ctx->stream), "copy")) !=
                LT_OK ||
            (st = launched(ctx, cudaMemcpyAsync(mt, tail->dev_m, d * 4, cudaMemcpyDeviceToDevice, ctx->stream),
                           "copy")) != LT_OK ||
            (st = launched(ctx, lt::launch_ffn_tail(c, tail->dev_f, tail->dev_w1, mt, tail->dev_w2, tail->dev_w,
                                                    tail->los, tail->eps, (uint32_t)d, 1, xt),
                           "ffn_tail")) != LT_OK)
            return st;
        dev_x = xt;
    }
    if (nseg > 1 && !dev_qkv_bias) {  // the norm and the projections in one launch (V = K: K once more)
        const lt::DevMat *m[3] = {&seg[0]->m, &seg[1]->m, v_is_k ? &seg[1]->m : &seg[2]->m};
        float *y[3] = {qkv, qkv + nq, qkv + nq + nkv};
        if ((st = launched(ctx, lt::launch_qmatvec_multi(c, 3, m, dev_x, dev_norm_w, eps, y), "qmatvec multi")) !=
            LT_OK)
            return st;
    } else {
        if ((st = launched(ctx, lt::launch_rmsnorm(c, dev_x, dev_norm_w, eps, (uint32_t)d, 1, xb), "rmsnorm")) != LT_OK)
            return st;
        if (nseg == 1) {
            if ((st = qmatvec_impl(ctx, seg[0], 0, xb, qkv, 1, dev_qkv_bias)) != LT_OK) return st;
        } else {
            const uint32_t off[3] = {0, nq, nq + nkv};
            for (uint32_t s = 0; s < 3; s++) {  // bias rows follow the rows present: V = K takes K's
                const lt_tensor *w = s == 2 && v_is_k ? seg[1] : seg[s];
                const uint32_t boff = s == 2 && v_is_k ? nq : off[s];
                if ((st = qmatvec_impl(ctx, w, 0, xb, qkv + off[s], 1, dev_qkv_bias ? dev_qkv_bias + boff : nullptr)) !=
                    LT_OK)
                    return st;
            }
        }
    }
    if ((st = ensure_counters(ctx, g.n_heads)) != LT_OK) return st;
    if ((st = launched(ctx, lt::launch_attn_prep(c, g, qkv, dev_q_norm, dev_k_norm, dev_pos, dev_k_cache, dev_v_cache),
                       "attn prep")) != LT_OK)
        return st;
    if ((st = launched(ctx, lt::launch_attn_decode(c, g, qkv, dev_k_cache, dev_v_cache, dev_pos, att,
                                                   (float *)ctx->scratch, ctx->counters),
                       "attn decode")) != LT_OK)
        return st;
    if (!dev_post_norm) return qmatvec_impl(ctx, wo, 0, att, dev_out, 1, dev_x);
    if ((st = qmatvec_impl(ctx, wo, 0, att, yb, 1, nullptr)) != LT_OK) return st;
    if (dev_out != dev_x &&
        (st = launched(ctx, cudaMemcpyAsync(dev_out, dev_x, d * 4, cudaMemcpyDeviceToDevice, ctx->stream), "copy")) !=
            LT_OK)
        return st;
    return launched(ctx, lt::launch_add_rmsnorm(c, yb, dev_post_norm, eps, (uint32_t)d, 1, dev_out), "add_rmsnorm");
}

lt_status lt_attn_block(lt_ctx *ctx, const lt_attn_cfg *cfg, const float *dev_x, const float *dev_norm_w, float eps,
                        const lt_tensor *wqkv, const float *dev_qkv_bias, const float *dev_q_norm,
                        const float *dev_k_norm, const uint32_t *dev_pos, void *dev_k_cache, void *dev_v_cache,
                        const lt_tensor *wo, float *dev_out) {
    const lt_tensor *seg[1] = {wqkv};
    return attn_block_impl(ctx, "lt_attn_block", cfg, dev_x, dev_norm_w, eps, seg, 1, dev_qkv_bias, dev_q_norm,
                           dev_k_norm, dev_pos, dev_k_cache, dev_v_cache, wo, nullptr, nullptr, dev_out);
}

lt_status lt_attn_block_split(lt_ctx *ctx, const lt_attn_cfg *cfg, const float *dev_x, const float *dev_norm_w,
                              float eps, const lt_tensor *wq, const lt_tensor *wk, const lt_tensor *wv,
                              const float *dev_qkv_bias, const float *dev_q_norm, const float *dev_k_norm,
                              const uint32_t *dev_pos, void *dev_k_cache, void *dev_v_cache, const lt_tensor *wo,
                              const float *dev_post_norm, const lt_ffn_tail_in *tail, float *dev_out) {
    const lt_tensor *seg[3] = {wq, wk, wv};
    return attn_block_impl(ctx, "lt_attn_block_split", cfg, dev_x, dev_norm_w, eps, seg, wv ? 3 : 2, dev_qkv_bias,
                           dev_q_norm, dev_k_norm, dev_pos, dev_k_cache, dev_v_cache, wo, dev_post_norm, tail,
                           dev_out);
}

// ── whole-stack decode ──────────────────────────────────────────────────────

lt_status lt_stack_create(lt_ctx *ctx, const lt_attn_cfg *cfg, uint32_t d_model, const lt_stack_layer *layers,
                          uint32_t n_layers, uint32_t k, int act, int norm_topk, float eps, lt_stack **out) {
    lt_status st = enter_uncaptured(ctx, "lt_stack_create");
    if (st != LT_OK) return st;
    if (!out || !layers || n_layers == 0) return fail(ctx, LT_EINVAL, "lt_stack_create: bad argument");
    *out = nullptr;
    lt::AttnGeom g;
    if ((st = attn_geom(ctx, cfg, g, "lt_stack_create")) != LT_OK) return st;
    if (act != LT_ACT_SILU && act != LT_ACT_GELU_TANH) return fail(ctx, LT_EINVAL, "lt_stack_create: act %d", act);
    const uint32_t nq = g.n_heads * g.hd, nkv = g.n_kv * g.hd;
    const lt_stack_layer &f = layers[0];
    const bool dense = f.router == nullptr;
    if (!f.wqkv || !f.wo || !f.gate || !f.up || !f.down)
        return fail(ctx, LT_EINVAL, "lt_stack_create: layer 0 lacks a tensor");
    lt::StackParams p{};
    p.g = g;
    p.d = d_model;
    p.dense = dense ? 1 : 0;
    p.E = dense ? 1 : (uint32_t)f.gate->m.n_experts;
    p.k = dense ? 1 : k;
    p.F = (uint32_t)f.gate->m.rows;
    p.norm_topk = norm_topk ? 1 : 0;
    p.act = act;
    p.eps = eps;
    p.n_layers = n_layers;
    p.qtype = f.wqkv->m.type;
    p.otype = f.wo->m.type;
    p.gtype = f.gate->m.type;
    p.dtype = f.down->m.type;
    p.qpitch = f.wqkv->m.pitch;
    p.opitch = f.wo->m.pitch;
    p.gpitch = f.gate->m.pitch;
    p.dpitch = f.down->m.pitch;
    std::vector<lt::StackLayerDev> dl(n_layers);
    for (uint32_t l = 0; l < n_layers; l++) {
        const lt_stack_layer &L = layers[l];
        auto same = [](const lt_tensor *t, uint32_t type, uint64_t rows, uint64_t cols, uint32_t E, uint64_t pitch) {
            return t && t->m.type == type && t->m.rows == rows && t->m.cols == cols && t->m.n_experts == E &&
                   t->m.pitch == pitch;
        };
        bool ok = same(L.wqkv, p.qtype, nq + 2 * nkv, d_model, 0, p.qpitch) &&
                  same(L.wo, p.otype, d_model, nq, 0, p.opitch) && L.attn_norm && L.ffn_norm && L.k_cache && L.v_cache &&
                  (L.router == nullptr) == dense &&
                  same(L.gate, p.gtype, p.F, d_model, dense ? 0 : p.E, p.gpitch) &&
                  same(L.up, p.gtype, p.F, d_model, dense ? 0 : p.E, p.gpitch) &&
                  same(L.down, p.dtype, d_model, p.F, dense ? 0 : p.E, p.dpitch);
        if (ok && !dense) ok = L.router->m.type == LT_TYPE_F32 && L.router->m.rows == p.E &&
                               L.router->m.cols == d_model && L.router->m.pitch == (uint64_t)d_model * 4;
        if (!ok) return fail(ctx, LT_EINVAL, "lt_stack_create: layer %u differs from layer 0 or lacks a tensor", l);
        // the norm weights are copied into shared memory by TMA: 16-byte aligned
        auto a16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
        if (!a16(L.attn_norm) || !a16(L.ffn_norm) || !a16(L.q_norm) || !a16(L.k_norm))
            return fail(ctx, LT_EUNSUPPORTED_TYPE, "lt_stack_create: layer %u norm weights not 16-byte aligned", l);
        lt::StackLayerDev &o = dl[l];
        o.wqkv = L.wqkv->m.data;
        o.wo = L.wo->m.data;
        o.attn_norm = L.attn_norm;
        o.ffn_norm = L.ffn_norm;
        o.q_norm = L.q_norm;
        o.k_norm = L.k_norm;
        o.bias = L.qkv_bias;
        o.kc = L.k_cache;
        o.vc = L.v_cache;
        o.router = dense ? nullptr : reinterpret_cast<const float *>(L.router->m.data);
        o.gate = L.gate->m.data;
        o.up = L.up->m.data;
        o.down = L.down->m.data;
        o.reserved = 0;
    }
    size_t smem = 0, scratch = 0, sync_off = 0;
    if (!lt::stack_plan(p, ctx->num_sms, &smem, &scratch, &sync_off))
        return fail(ctx, LT_EUNSUPPORTED_TYPE, "lt_stack_create: shape or types outside the stack kernel");
    lt_stack *s = new (std::nothrow) lt_stack;
    if (!s) return fail(ctx, LT_ENOMEM, "lt_stack_create: host allocation");
    s->p = p;
    s->scratch_bytes = scratch;
    cudaError_t e = cudaMalloc(&s->dev_layers, sizeof(lt::StackLayerDev) * n_layers);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&s->scratch), scratch);
    if (e == cudaSuccess) e = cudaMemsetAsync(s->scratch, 0, scratch, ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(s->dev_layers, dl.data(), sizeof(lt::StackLayerDev) * n_layers, cudaMemcpyHostToDevice,
                            ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        if (s->dev_layers) cudaFree(s->dev_layers);
        if (s->scratch) cudaFree(s->scratch);
        delete s;
        return cuda_fail(ctx, e, "lt_stack_create");
    }
    *out = s;
    return LT_OK;
}

lt_status lt_stack_run(lt_ctx *ctx, const lt_stack *s, float *dev_x, const uint32_t *dev_pos) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!s || !dev_x || !dev_pos) return fail(ctx, LT_EINVAL, "lt_stack_run: bad argument");
    return launched(ctx, lt::launch_stack(cfg_of(ctx), s->p, s->dev_layers, dev_x, dev_pos, s->scratch), "stack");
}

lt_status lt_stack_free(lt_ctx *ctx, lt_stack *s) {
    if (!s) return LT_OK;
    if (ctx) cudaSetDevice(ctx->device);
    if (ctx) cudaStreamSynchronize(ctx->stream);
    cudaFree(s->dev_layers);
    cudaFree(s->scratch);
    delete s;
    return LT_OK;
}

void lt_rng_seed(uint64_t seed, uint64_t state_out[4]) {
    uint64_t st = seed;  // SplitMix64
    for (int i = 0; i < 4; i++) {
        st += 0x9e3779b97f4a7c15ull;
        uint64_t z = st;
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        state_out[i] = z ^ (z >> 31);
    }
}

lt_status lt_sample_step(lt_ctx *ctx, const float *dev_logits, uint32_t n, const lt_sample_params *params,
                         uint64_t *dev_rng_state, uint32_t *dev_tokens, uint32_t *dev_pos,
                         const uint32_t *dev_n_prompt) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_logits || !params || !dev_rng_state || !dev_tokens || !dev_pos || !dev_n_prompt || n == 0)
        return fail(ctx, LT_EINVAL, "lt_sample_step: bad argument");
    if (!(params->temperature >= 0.0f) || !(params->top_p >= 0.0f))
        return fail(ctx, LT_EINVAL, "lt_sample_step: temperature %g, top_p %g", params->temperature, params->top_p);
    if ((st = ensure_scratch(ctx, (size_t)n * 4)) != LT_OK) return st;
    return launched(ctx,
                    lt::launch_sample(cfg_of(ctx), dev_logits, n, params->temperature, params->top_k, params->top_p,
                                      reinterpret_cast<unsigned long long *>(dev_rng_state), dev_tokens, dev_pos,
                                      dev_n_prompt, (float *)ctx->scratch),
                    "sample");
}

lt_status lt_greedy_step(lt_ctx *ctx, const float *dev_logits, uint32_t n, uint32_t *dev_tokens, uint32_t *dev_pos,
                         const uint32_t *dev_n_prompt) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_logits || !dev_tokens || !dev_pos || !dev_n_prompt || n == 0)
        return fail(ctx, LT_EINVAL, "lt_greedy_step: bad argument");
    if ((st = ensure_scratch(ctx, al256(64 * 4) * 2)) != LT_OK) return st;
    if ((st = ensure_counters(ctx, 1)) != LT_OK) return st;
    float *pv = (float *)ctx->scratch;
    uint32_t *pi = (uint32_t *)(ctx->scratch + al256(64 * 4));
    return launched(ctx,
                    lt::launch_argmax(cfg_of(ctx), dev_logits, n, 1, nullptr, pv, pi, ctx->counters, dev_tokens,
                                      dev_pos, dev_n_prompt),
                    "greedy step");
}

static lt_status check_router(lt_ctx *ctx, const lt_tensor *router, uint32_t k) {
    if (!router) return fail(ctx, LT_EINVAL, "router: null tensor");
    if (router->m.type != lt::T_F32 || router->m.n_experts != 0)
        return fail(ctx, LT_EUNSUPPORTED_TYPE, "router: weights must be a 2-D F32 matrix");
    if (router->m.rows == 0 || router->m.rows > (uint64_t)lt::kRouterMaxE)
        return fail(ctx, LT_EINVAL, "router: %llu experts (max %d)", (unsigned long long)router->m.rows,
                    lt::kRouterMaxE);
    if (k == 0 || k > 16 || k > router->m.rows) return fail(ctx, LT_EINVAL, "router: k=%u", k);
    if (router->m.cols > 8192) return fail(ctx, LT_EINVAL, "router: width %llu > 8192", (unsigned long long)router->m.cols);
    return LT_OK;
}

static lt_status route_impl(lt_ctx *ctx, const lt_tensor *router, const float *x, const float *norm_w, float eps,
                            uint32_t ntok, uint32_t k, int norm_topk, const float *escale, uint32_t *ids, float *w,
                            float *logits, uint8_t *xq, uint64_t xq_pitch, float *xn = nullptr) {
    const uint32_t groups = lt::router_token_groups(ntok);
    lt_status st = ensure_counters(ctx, groups);
    if (st != LT_OK) return st;
    return launched(ctx,
                    lt::launch_router(cfg_of(ctx), (const float *)router->m.data, (uint32_t)router->m.rows,
                                      (uint32_t)router->m.cols, (uint32_t)(router->m.pitch / 4), x, norm_w, eps, ntok,
                                      k, norm_topk, escale, ids, w, logits, ctx->counters, xq, xq_pitch, xn),
                    "router");
}

lt_status lt_moe_route(lt_ctx *ctx, const lt_tensor *router, const float *dev_x, uint32_t ntok, uint32_t k,
                       int norm_topk, const float *dev_expert_scale, uint32_t *dev_ids, float *dev_w) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if ((st = check_router(ctx, router, k)) != LT_OK) return st;
    if (!dev_x || !dev_ids || !dev_w) return fail(ctx, LT_EINVAL, "lt_moe_route: null pointer");
    if (ntok == 0) return LT_OK;
    if ((st = ensure_scratch(ctx, al256((size_t)ntok * router->m.rows * 4))) != LT_OK) return st;
    return route_impl(ctx, router, dev_x, nullptr, 0.0f, ntok, k, norm_topk, dev_expert_scale, dev_ids, dev_w,
                      (float *)ctx->scratch, nullptr, 0);
}

static lt_status check_experts(lt_ctx *ctx, const lt_tensor *gate, const lt_tensor *up, const lt_tensor *down,
                               uint32_t k, uint64_t *F_out) {
    if (!gate || !down) return fail(ctx, LT_EINVAL, "moe: null expert tensor");
    const uint32_t E = gate->m.n_experts;
    if (E == 0 || down->m.n_experts != E || (up && up->m.n_experts != E))
        return fail(ctx, LT_EINVAL, "moe: gate/up/down must be 3-D expert tensors with the same expert count");
    if (!quantized(gate->m.type) || !quantized(down->m.type) || (up && up->m.type != gate->m.type))
        return fail(ctx, LT_EUNSUPPORTED_TYPE, "moe: expert weights must be block-quantised (gate and up alike)");
    const uint64_t F = up ? gate->m.rows : gate->m.rows / 2;
    if ((!up && gate->m.rows % 2) || (up && (up->m.rows != F || up->m.cols != gate->m.cols)))
        return fail(ctx, LT_EINVAL, "moe: gate/up shapes disagree");
    if (down->m.rows != gate->m.cols || down->m.cols != F)
        return fail(ctx, LT_EINVAL, "moe: down is %llux%llu, expected %llux%llu", (unsigned long long)down->m.rows,
                    (unsigned long long)down->m.cols, (unsigned long long)gate->m.cols, (unsigned long long)F);
    lt_status st;
    if ((st = check_kernel_shape(ctx, gate->m, "moe gate")) != LT_OK) return st;
    if ((st = check_kernel_shape(ctx, down->m, "moe down")) != LT_OK) return st;
    if (F % 32 != 0) return fail(ctx, LT_EINVAL, "moe: expert width %llu not a multiple of 32", (unsigned long long)F);
    if (k == 0 || k > 16 || k > E) return fail(ctx, LT_EINVAL, "moe: k=%u", k);
    *F_out = F;
    return LT_OK;
}

// Scratch bytes of the tensor-core expert GEMM when a batch of ntok tokens
// takes that path, else 0.
static size_t gemm_bytes_of(const lt_ctx *ctx, const lt_tensor *gate, const lt_tensor *down, uint32_t ntok, uint32_t k) {
    const uint64_t F = down->m.cols;
    if (ntok < 2 || ctx->tc_min_tokens == 0 || ntok < ctx->tc_min_tokens) return 0;
    if (!lt::moe_gemm_supported(gate->m, down->m, F)) return 0;
    return lt::moe_gemm_scratch(ntok, k, gate->m.n_experts, gate->m.cols, F);
}

// xf: f32 expert input rows (used by the tensor-core path; the CUDA-core
// path reads the quantised rows s.xq).
static lt_status ffn_impl(lt_ctx *ctx, const lt_tensor *gate, const lt_tensor *up, const lt_tensor *down, int act,
                          uint32_t ntok, const uint32_t *ids, const float *w, uint32_t k, const float *resid,
                          float *out, const float *xf, const MoeScratch &s) {
    const lt::LaunchCfg c = cfg_of(ctx);
    const bool direct = ntok == 1;
    lt::DevMat upm = up ? up->m : lt::DevMat{};
    if (!up) upm.data = nullptr;
    const uint32_t E = gate->m.n_experts ? gate->m.n_experts : 1;  // a dense FFN is expert 0 of one
    lt_status st;
    if (!direct && s.gemm) {
        st = launched(ctx, lt::launch_moe_plan(c, ids, ntok, k, E, s.plan), "moe plan");
        if (st != LT_OK) return st;
        return launched(ctx,
                        lt::launch_moe_gemm_ffn(c, gate->m, upm.data, down->m, act, xf, ntok, k, w, s.plan, resid,
                                                out, s.gemm),
                        "moe gemm");
    }
    if (ntok > 65535u)  // the CUDA-core down kernel puts tokens in grid.y
        return fail(ctx, LT_EINVAL, "moe: %u tokens exceed 65535 outside the tensor-core path", ntok);
    st = ensure_counters(ctx, lt::kMoeCounterBase + s.counters);
    if (st != LT_OK) return st;
    if (!direct) {
        st = launched(ctx, lt::launch_moe_plan(c, ids, ntok, k, E, s.plan), "moe plan");
        if (st != LT_OK) return st;
    }
    st = launched(ctx,
                  lt::launch_moe_gate_up(c, gate->m, upm, act, s.xq, s.xq_pitch, ntok, k, ids, direct, s.plan, s.hf,
                                         ctx->counters + lt::kMoeCounterBase, s.hq, s.hq_pitch),
                  "moe gate_up");
    if (st != LT_OK) return st;
    return launched(ctx,
                    lt::launch_moe_down(c, down->m, s.hq, s.hq_pitch, ntok, k, ids, w, direct, s.plan, resid, out),
                    "moe down");
}

lt_status lt_moe_ffn(lt_ctx *ctx, const lt_tensor *gate, const lt_tensor *up, const lt_tensor *down, int act,
                     const float *dev_x, uint32_t ntok, const uint32_t *dev_ids, const float *dev_w, uint32_t k,
                     float *dev_out) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    uint64_t F = 0;
    if ((st = check_experts(ctx, gate, up, down, k, &F)) != LT_OK) return st;
    if (act != LT_ACT_SILU && act != LT_ACT_GELU_TANH) return fail(ctx, LT_EINVAL, "moe: act %d", act);
    if (!dev_x || !dev_ids || !dev_w || !dev_out) return fail(ctx, LT_EINVAL, "lt_moe_ffn: null pointer");
    if (ntok == 0) return LT_OK;
    const uint64_t d = gate->m.cols;
    const size_t gb = gemm_bytes_of(ctx, gate, down, ntok, k);
    const MoeScratch probe = moe_layout(nullptr, ntok, k, gate->m.n_experts, d, F, gb);
    if ((st = ensure_scratch(ctx, probe.bytes)) != LT_OK) return st;
    const MoeScratch s = moe_layout(ctx->scratch, ntok, k, gate->m.n_experts, d, F, gb);
    if (!s.gemm) {
        st = launched(ctx, lt::launch_quantize(cfg_of(ctx), dev_x, (uint32_t)d, ntok, s.xq, s.xq_pitch), "quantize");
        if (st != LT_OK) return st;
    }
    return ffn_impl(ctx, gate, up, down, act, ntok, dev_ids, dev_w, k, nullptr, dev_out, dev_x, s);
}

static lt_status forward_impl(lt_ctx *ctx, const lt_tensor *router, const lt_tensor *gate, const lt_tensor *up,
                              const lt_tensor *down, int act, int norm_topk, const float *dev_expert_scale,
                              const float *dev_norm_w, float eps, int residual, const float *dev_x, uint32_t ntok,
                              uint32_t k, float *dev_out, uint32_t *dev_ids, float *dev_w,
                              const float *dev_router_scale = nullptr, float router_gs = 1.0f) {
    struct Clear {
        lt_ctx *c;
        ~Clear() { clear_prefetch(c); }
    } clear{ctx};  // the hint applies to this call only
    lt_status st;
    uint64_t F = 0;
    if ((st = check_router(ctx, router, k)) != LT_OK) return st;
    if ((st = check_experts(ctx, gate, up, down, k, &F)) != LT_OK) return st;
    if (router->m.rows != gate->m.n_experts || router->m.cols != gate->m.cols)
        return fail(ctx, LT_EINVAL, "moe: router is %llux%llu for %u experts of width %llu",
                    (unsigned long long)router->m.rows, (unsigned long long)router->m.cols, gate->m.n_experts,
                    (unsigned long long)gate->m.cols);
    if (act != LT_ACT_SILU && act != LT_ACT_GELU_TANH) return fail(ctx, LT_EINVAL, "moe: act %d", act);
    if (!dev_x || !dev_out) return fail(ctx, LT_EINVAL, "moe: null pointer");
    if (ntok == 0) return LT_OK;
    const uint32_t E = gate->m.n_experts;
    const uint64_t d = gate->m.cols;
    const size_t gb = gemm_bytes_of(ctx, gate, down, ntok, k);
    const MoeScratch probe = moe_layout(nullptr, ntok, k, E, d, F, gb);
    const size_t pair_b = dev_router_scale ? 2 * al256((size_t)ntok * d * 4) : 0;  // expert and router inputs
    if ((st = ensure_scratch(ctx, probe.bytes + pair_b)) != LT_OK) return st;
    const MoeScratch s = moe_layout(ctx->scratch, ntok, k, E, d, F, gb);
    uint32_t *ids = dev_ids ? dev_ids : s.ids;
    float *w = dev_w ? dev_w : s.w;
    if (ntok == 1 && ctx->decode_kernel) {
        lt::DecodeParams p;
        p.router = (const float *)router->m.data;
        p.E = E;
        p.d = (uint32_t)d;
        p.router_ld = (uint32_t)(router->m.pitch / 4);
        p.x = dev_x;
        p.norm_w = dev_norm_w;
        p.router_scale = dev_router_scale;
        p.router_gs = router_gs;
        p.eps = eps;
        p.k = k;
        p.norm_topk = norm_topk;
        p.escale = dev_expert_scale;
        p.ids = ids;
        p.w = w;
        p.gate = gate->m;
        p.up_data = up ? up->m.data : nullptr;
        p.down = down->m;
        p.F = (uint32_t)F;
        p.act = act;
        p.himg = s.himg;
        p.residual = residual;
        p.out = dev_out;
        p.sync = ctx->dec_sync;
        for (int i = 0; i < 2; i++) {
            p.pf[i] = ctx->pf[i];
            p.pf_bytes[i] = ctx->pf_bytes[i];
        }
        if (lt::moe_decode_fits(p, ctx->num_sms)) return launched(ctx, lt::launch_moe_decode(cfg_of(ctx), p), "moe decode");
    }
    if (dev_router_scale) {  // separate inputs: norm_pair, then route and experts on them
        const lt::LaunchCfg c = cfg_of(ctx);
        float *xe = (float *)(ctx->scratch + probe.bytes), *xr = xe + pair_b / 8;
        st = launched(ctx, lt::launch_norm_pair(c, dev_x, dev_norm_w, dev_router_scale, router_gs, eps, (uint32_t)d,
                                                ntok, xe, xr),
                      "norm pair");
        if (st != LT_OK) return st;
        st = route_impl(ctx, router, xr, nullptr, 0.0f, ntok, k, norm_topk, dev_expert_scale, ids, w, s.logits,
                        nullptr, 0, nullptr);
        if (st != LT_OK) return st;
        if (!s.gemm) {
            st = launched(ctx, lt::launch_quantize(c, xe, (uint32_t)d, ntok, s.xq, s.xq_pitch), "quantize");
            if (st != LT_OK) return st;
        }
        return ffn_impl(ctx, gate, up, down, act, ntok, ids, w, k, residual ? dev_x : nullptr, dev_out, xe, s);
    }
    float *xn = s.gemm && dev_norm_w ? s.xn : nullptr;  // the tensor-core path reads f32 rows
    st = route_impl(ctx, router, dev_x, dev_norm_w, eps, ntok, k, norm_topk, dev_expert_scale, ids, w, s.logits,
                    s.gemm ? nullptr : s.xq, s.xq_pitch, xn);
    if (st != LT_OK) return st;
    return ffn_impl(ctx, gate, up, down, act, ntok, ids, w, k, residual ? dev_x : nullptr, dev_out, xn ? xn : dev_x,
                    s);
}

lt_status lt_moe_block_scaled(lt_ctx *ctx, const lt_tensor *router, const lt_tensor *gate, const lt_tensor *up,
                              const lt_tensor *down, int act, int norm_topk, const float *dev_expert_scale,
                              const float *dev_norm_w, const float *dev_router_scale, float router_gs, float eps,
                              const float *dev_x, uint32_t ntok, uint32_t k, int residual, float *dev_out,
                              uint32_t *dev_ids, float *dev_w) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_norm_w || !dev_router_scale) return fail(ctx, LT_EINVAL, "lt_moe_block_scaled: null norm weights");
    return forward_impl(ctx, router, gate, up, down, act, norm_topk, dev_expert_scale, dev_norm_w, eps, residual ? 1 : 0,
                        dev_x, ntok, k, dev_out, dev_ids, dev_w, dev_router_scale, router_gs);
}

lt_status lt_moe_forward(lt_ctx *ctx, const lt_tensor *router, const lt_tensor *gate, const lt_tensor *up,
                         const lt_tensor *down, int act, int norm_topk, const float *dev_expert_scale,
                         const float *dev_x, uint32_t ntok, uint32_t k, float *dev_out, uint32_t *dev_ids,
                         float *dev_w) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    return forward_impl(ctx, router, gate, up, down, act, norm_topk, dev_expert_scale, nullptr, 0.0f, 0, dev_x, ntok,
                        k, dev_out, dev_ids, dev_w);
}

lt_status lt_moe_block(lt_ctx *ctx, const lt_tensor *router, const lt_tensor *gate, const lt_tensor *up,
                       const lt_tensor *down, int act, int norm_topk, const float *dev_expert_scale,
                       const float *dev_norm_w, float eps, const float *dev_x, uint32_t ntok, uint32_t k,
                       float *dev_out, uint32_t *dev_ids, float *dev_w) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_norm_w) return fail(ctx, LT_EINVAL, "lt_moe_block: null norm weights");
    return forward_impl(ctx, router, gate, up, down, act, norm_topk, dev_expert_scale, dev_norm_w, eps, 1, dev_x,
                        ntok, k, dev_out, dev_ids, dev_w);
}

lt_status lt_scale(lt_ctx *ctx, float *dev_x, uint32_t n, uint32_t ntok, float s) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_x || n == 0) return fail(ctx, LT_EINVAL, "lt_scale: bad argument");
    if (ntok == 0) return LT_OK;
    return launched(ctx, lt::launch_scale(cfg_of(ctx), dev_x, n, ntok, s), "scale");
}

lt_status lt_add_rmsnorm(lt_ctx *ctx, const float *dev_y, const float *dev_w, float eps, uint32_t n, uint32_t ntok,
                         float *dev_x) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_y || !dev_w || !dev_x || n == 0) return fail(ctx, LT_EINVAL, "lt_add_rmsnorm: bad argument");
    if (ntok == 0) return LT_OK;
    return launched(ctx, lt::launch_add_rmsnorm(cfg_of(ctx), dev_y, dev_w, eps, n, ntok, dev_x), "add_rmsnorm");
}

lt_status lt_norm_pair(lt_ctx *ctx, const float *dev_x, const float *dev_w, const float *dev_g, float gs, float eps,
                       uint32_t n, uint32_t ntok, float *dev_a, float *dev_b) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_x || !dev_w || !dev_g || !dev_a || !dev_b || n == 0) return fail(ctx, LT_EINVAL, "lt_norm_pair: bad argument");
    if (ntok == 0) return LT_OK;
    return launched(ctx, lt::launch_norm_pair(cfg_of(ctx), dev_x, dev_w, dev_g, gs, eps, n, ntok, dev_a, dev_b),
                    "norm_pair");
}

lt_status lt_ffn_tail(lt_ctx *ctx, const float *dev_f, const float *dev_w1, float *dev_m, const float *dev_w2,
                      const float *dev_w, float los, float eps, uint32_t n, uint32_t ntok, float *dev_x) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_f || !dev_m || !dev_w2 || !dev_w || !dev_x || n == 0) return fail(ctx, LT_EINVAL, "lt_ffn_tail: bad argument");
    if (ntok == 0) return LT_OK;
    return launched(ctx, lt::launch_ffn_tail(cfg_of(ctx), dev_f, dev_w1, dev_m, dev_w2, dev_w, los, eps, n, ntok, dev_x),
                    "ffn_tail");
}

lt_status lt_softcap(lt_ctx *ctx, float *dev_x, uint64_t n, float cap) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_x || cap == 0.0f) return fail(ctx, LT_EINVAL, "lt_softcap: bad argument");
    if (n == 0) return LT_OK;
    return launched(ctx, lt::launch_softcap(cfg_of(ctx), dev_x, n, cap), "softcap");
}

lt_status lt_ffn_block(lt_ctx *ctx, const lt_tensor *gate, const lt_tensor *up, const lt_tensor *down, int act,
                       const float *dev_norm_w, float eps, const float *dev_x, uint32_t ntok, int residual,
                       float *dev_out) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!gate || !up || !down || !dev_norm_w || !dev_x || !dev_out) return fail(ctx, LT_EINVAL, "lt_ffn_block: null argument");
    if (gate->m.n_experts || up->m.n_experts || down->m.n_experts)
        return fail(ctx, LT_EINVAL, "lt_ffn_block: dense (2-D) tensors expected");
    if (!quantized(gate->m.type) || !quantized(down->m.type) || up->m.type != gate->m.type)
        return fail(ctx, LT_EUNSUPPORTED_TYPE, "lt_ffn_block: weights must be block-quantised (gate and up alike)");
    const uint64_t d = gate->m.cols, F = gate->m.rows;
    if (up->m.rows != F || up->m.cols != d || down->m.rows != d || down->m.cols != F)
        return fail(ctx, LT_EINVAL, "lt_ffn_block: gate/up/down shapes disagree");
    if ((st = check_kernel_shape(ctx, gate->m, "lt_ffn_block gate")) != LT_OK) return st;
    if ((st = check_kernel_shape(ctx, down->m, "lt_ffn_block down")) != LT_OK) return st;
    if (F % 32 != 0) return fail(ctx, LT_EINVAL, "lt_ffn_block: width %llu not a multiple of 32", (unsigned long long)F);
    if (act != LT_ACT_SILU && act != LT_ACT_GELU_TANH) return fail(ctx, LT_EINVAL, "lt_ffn_block: act %d", act);
    if (ntok == 0) return LT_OK;
    if ((st = ensure_consts(ctx, ntok)) != LT_OK) return st;
    // the expert kernels with one expert (id 0) of weight 1 per token
    const MoeScratch probe = moe_layout(nullptr, ntok, 1, 1, d, F, 0);
    const size_t xn_bytes = al256((size_t)ntok * d * 4);
    if ((st = ensure_scratch(ctx, probe.bytes + xn_bytes)) != LT_OK) return st;
    const MoeScratch s = moe_layout(ctx->scratch, ntok, 1, 1, d, F, 0);
    float *xn = (float *)(ctx->scratch + probe.bytes);
    const lt::LaunchCfg c = cfg_of(ctx);
    if (ntok == 1 && ctx->decode_kernel) {  // the single-token persistent kernel, dense mode
        lt::DecodeParams p;
        p.router = nullptr;
        p.E = 1;
        p.d = (uint32_t)d;
        p.router_ld = 0;
        p.x = dev_x;
        p.norm_w = dev_norm_w;
        p.eps = eps;
        p.k = 1;
        p.norm_topk = 0;
        p.escale = nullptr;
        p.ids = nullptr;
        p.w = nullptr;
        p.gate = gate->m;
        p.up_data = up->m.data;
        p.down = down->m;
        p.F = (uint32_t)F;
        p.act = act;
        p.himg = s.himg;
        p.residual = residual;
        p.out = dev_out;
        p.sync = ctx->dec_sync;
        for (int i = 0; i < 2; i++) {
            p.pf[i] = ctx->pf[i];
            p.pf_bytes[i] = ctx->pf_bytes[i];
        }
        if (lt::moe_decode_fits(p, ctx->num_sms)) {
            clear_prefetch(ctx);
            return launched(ctx, lt::launch_moe_decode(c, p), "ffn decode");
        }
    }
    st = launched(ctx, lt::launch_rmsnorm(c, dev_x, dev_norm_w, eps, (uint32_t)d, ntok, xn), "rmsnorm");
    if (st != LT_OK) return st;
    st = launched(ctx, lt::launch_quantize(c, xn, (uint32_t)d, ntok, s.xq, s.xq_pitch), "quantize");
    if (st != LT_OK) return st;
    return ffn_impl(ctx, gate, up, down, act, ntok, ctx->zeros, ctx->ones, 1, residual ? dev_x : nullptr, dev_out, xn,
                    s);
}

lt_status lt_ep_dispatch(lt_ctx *ctx, const uint32_t *dev_ids, uint32_t ntok, uint32_t k, uint32_t n_experts,
                         uint32_t nranks, uint32_t *dev_send_counts, uint32_t *dev_send_token,
                         uint32_t *dev_send_local, uint32_t *dev_pair_pos) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_ids || !dev_send_counts || !dev_send_token || !dev_send_local || !dev_pair_pos)
        return fail(ctx, LT_EINVAL, "lt_ep_dispatch: null pointer");
    if (nranks == 0 || nranks > 8 || n_experts == 0 || n_experts % nranks != 0 || k == 0)
        return fail(ctx, LT_EINVAL, "lt_ep_dispatch: %u experts over %u ranks", n_experts, nranks);
    if (ntok == 0)  // nothing to send: every count is zero
        return launched(ctx, cudaMemsetAsync(dev_send_counts, 0, nranks * sizeof(uint32_t), ctx->stream),
                        "ep dispatch counts");
    return launched(ctx,
                    lt::launch_ep_dispatch(cfg_of(ctx), dev_ids, ntok, k, n_experts, nranks, dev_send_counts,
                                           dev_send_token, dev_send_local, dev_pair_pos),
                    "ep dispatch");
}

lt_status lt_gather_rows(lt_ctx *ctx, const float *dev_src, uint64_t cols, const uint32_t *dev_idx, uint32_t n,
                         float *dev_dst) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_src || !dev_idx || !dev_dst) return fail(ctx, LT_EINVAL, "lt_gather_rows: null pointer");
    if (cols == 0 || cols % 4 != 0) return fail(ctx, LT_EINVAL, "lt_gather_rows: cols %llu", (unsigned long long)cols);
    if (n == 0) return LT_OK;
    return launched(ctx, lt::launch_gather_rows(cfg_of(ctx), dev_src, cols, dev_idx, n, dev_dst), "gather rows");
}

lt_status lt_moe_combine(lt_ctx *ctx, const float *dev_y, uint64_t cols, const uint32_t *dev_pair_pos,
                         const float *dev_w, uint32_t ntok, uint32_t k, const float *dev_resid, float *dev_out) {
    lt_status st = enter(ctx);
    if (st != LT_OK) return st;
    if (!dev_y || !dev_pair_pos || !dev_w || !dev_out) return fail(ctx, LT_EINVAL, "lt_moe_combine: null pointer");
    if (cols == 0 || k == 0) return fail(ctx, LT_EINVAL, "lt_moe_combine: cols %llu, k %u", (unsigned long long)cols, k);
    if (ntok == 0) return LT_OK;
    return launched(ctx, lt::launch_combine(cfg_of(ctx), dev_y, cols, dev_pair_pos, dev_w, ntok, k, dev_resid, dev_out),
                    "combine");
}

lt_status lt_quant_matvec_host(lt_ctx *ctx, float *out, const lt_tensor *mat, uint32_t expert, const float *vec,
                               uint64_t rows, uint64_t cols) {
    lt_status st = enter_uncaptured(ctx, "lt_quant_matvec_host");
    if (st != LT_OK) return st;
    if (!out || !mat || !vec) return fail(ctx, LT_EINVAL, "lt_quant_matvec_host: null pointer");
    if (rows != mat->m.rows || cols != mat->m.cols)
        return fail(ctx, LT_EINVAL, "lt_quant_matvec_host: %llux%llu given, tensor is %llux%llu",
                    (unsigned long long)rows, (unsigned long long)cols, (unsigned long long)mat->m.rows,
                    (unsigned long long)mat->m.cols);
    // device vectors live past the region lt_qmatvec uses for its quantised input
    const size_t qb = al256(lt::qact_row_pitch(cols)), xb = al256(cols * 4), yb = al256(rows * 4);
    if ((st = ensure_scratch(ctx, qb + xb + yb)) != LT_OK) return st;
    if ((st = ensure_pinned(ctx, xb + yb)) != LT_OK) return st;
    float *dx = (float *)(ctx->scratch + qb), *dy = (float *)(ctx->scratch + qb + xb);
    float *px = (float *)ctx->pinned, *py = (float *)(ctx->pinned + xb);
    memcpy(px, vec, cols * 4);
    LT_CUDA(ctx, cudaMemcpyAsync(dx, px, cols * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D");
    if ((st = lt_qmatvec(ctx, mat, expert, dx, dy, 1)) != LT_OK) return st;
    LT_CUDA(ctx, cudaMemcpyAsync(py, dy, rows * 4, cudaMemcpyDeviceToHost, ctx->stream), "D2H");
    if ((st = lt_sync(ctx)) != LT_OK) return st;
    memcpy(out, py, rows * 4);
    return LT_OK;
}

lt_status lt_moe_forward_host(lt_ctx *ctx, const lt_tensor *router, const lt_tensor *gate, const lt_tensor *up,
                              const lt_tensor *down, int act, int norm_topk, const float *expert_scale_host,
                              const float *x, uint32_t ntok, uint32_t k, float *out, uint32_t *ids, float *w) {
    lt_status st = enter_uncaptured(ctx, "lt_moe_forward_host");
    if (st != LT_OK) return st;
    if (!gate || !x || !out) return fail(ctx, LT_EINVAL, "lt_moe_forward_host: null pointer");
    if (ntok == 0) return LT_OK;
    const uint64_t d = gate->m.cols;
    const uint32_t E = gate->m.n_experts;
    const MoeScratch probe = moe_layout(nullptr, ntok, k, E ? E : 1, d, gate->m.rows,
                                        down ? gemm_bytes_of(ctx, gate, down, ntok, k) : 0);
    const size_t xb = al256((size_t)ntok * d * 4), ib = al256((size_t)ntok * k * 4), eb = al256((size_t)E * 4);
    const size_t io = 2 * xb + 2 * ib + eb;
    if ((st = ensure_scratch(ctx, probe.bytes + io)) != LT_OK) return st;
    if ((st = ensure_pinned(ctx, io)) != LT_OK) return st;
    uint8_t *dbase = ctx->scratch + probe.bytes;
    float *dx = (float *)dbase, *dout = (float *)(dbase + xb);
    uint32_t *dids = (uint32_t *)(dbase + 2 * xb);
    float *dw = (float *)(dbase + 2 * xb + ib);
    float *dscale = (float *)(dbase + 2 * xb + 2 * ib);
    uint8_t *hb = ctx->pinned;
    memcpy(hb, x, (size_t)ntok * d * 4);
    LT_CUDA(ctx, cudaMemcpyAsync(dx, hb, (size_t)ntok * d * 4, cudaMemcpyHostToDevice, ctx->stream), "H2D x");
    if (expert_scale_host) {
        memcpy(hb + 2 * xb + 2 * ib, expert_scale_host, (size_t)E * 4);
        LT_CUDA(ctx, cudaMemcpyAsync(dscale, hb + 2 * xb + 2 * ib, (size_t)E * 4, cudaMemcpyHostToDevice, ctx->stream),
                "H2D scale");
    }
    // lt_moe_forward places its scratch at the start of the arena (at most
    // probe.bytes, computed with F <= gate rows); ours lives after it.
    st = lt_moe_forward(ctx, router, gate, up, down, act, norm_topk, expert_scale_host ? dscale : nullptr, dx, ntok,
                        k, dout, dids, dw);
    if (st != LT_OK) return st;
    LT_CUDA(ctx, cudaMemcpyAsync(hb + xb, dout, (size_t)ntok * d * 4, cudaMemcpyDeviceToHost, ctx->stream), "D2H out");
    if (ids)
        LT_CUDA(ctx, cudaMemcpyAsync(hb + 2 * xb, dids, (size_t)ntok * k * 4, cudaMemcpyDeviceToHost, ctx->stream),
                "D2H ids");
    if (w)
        LT_CUDA(ctx, cudaMemcpyAsync(hb + 2 * xb + ib, dw, (size_t)ntok * k * 4, cudaMemcpyDeviceToHost, ctx->stream),
                "D2H w");
    if ((st = lt_sync(ctx)) != LT_OK) return st;
    memcpy(out, hb + xb, (size_t)ntok * d * 4);
    if (ids) memcpy(ids, hb + 2 * xb, (size_t)ntok * k * 4);
    if (w) memcpy(w, hb + 2 * xb + ib, (size_t)ntok * k * 4);
    return LT_OK;
}

}  // extern "C"
