// llmtoy_ops.hpp — C++ host mirror of llmtoy-zig's operator API, backed by the
// sm_100a C ABI (include/llmtoy_cuda.h).
//
// The names, argument order and meaning follow the reference's Zig functions
// so a host port of src/model (forward loop, KV cache, sampler) can call these
// where it called src/ops and src/quant.  Zig error unions become lt_status
// return values ([[nodiscard]]); where the reference panics (unsupported
// GGUF type, src/ops/math.zig:206,223) these return LT_EUNSUPPORTED_TYPE.
// There is no CPU fallback.
#pragma once

#include <cstddef>
#include <cstdint>
#include <utility>

#include "llmtoy_cuda.h"

namespace llmtoy {

// GgmlType, src/gguf/types.zig:23-52: the ten matrix types rowBytes /
// dequantRow handle (src/ops/math.zig:194-225), all of which the backend decodes.
enum class GgmlType : uint32_t {
    f32 = 0, f16 = 1, q5_0 = 6, q5_1 = 7, q8_0 = 8, q3_k = 11, q4_k = 12, q5_k = 13, q6_k = 14, iq4_nl = 20
};

// GpuContext (src/gpu/context.zig) -> one CUDA context + stream per GPU.
class Backend {
public:
    explicit Backend(int device = 0) { status_ = lt_init(device, &ctx_); }
    ~Backend() { lt_free(ctx_); }
    Backend(const Backend &) = delete;
    Backend &operator=(const Backend &) = delete;
    Backend(Backend &&o) noexcept : ctx_(std::exchange(o.ctx_, nullptr)), status_(o.status_) {}

    lt_status status() const { return status_; }   // LT_ENODEV without an sm_100 GPU
    lt_ctx *ctx() const { return ctx_; }
    const char *lastError() const { return lt_last_error(ctx_); }
    [[nodiscard]] lt_status sync() const { return lt_sync(ctx_); }

private:
    lt_ctx *ctx_ = nullptr;
    lt_status status_ = LT_ENODEV;
};

// RawMatrix{data,type_,rows,cols} (src/model/model_weights.zig:17-22) once
// its GGUF bytes are on the device.  For expert tensors rows is per expert
// (src/model/gemma4/loader.zig:277-292).
struct RawMatrix {
    lt_tensor *data = nullptr;
    GgmlType type_ = GgmlType::f32;
    uint64_t rows = 0;
    uint64_t cols = 0;
    uint32_t n_experts = 0;
};

// GpuWeights.init-style upload of one mmap'd tensor (gpu_weights.zig:373).
[[nodiscard]] inline lt_status upload(Backend &b, const void *gguf_bytes, size_t nbytes, GgmlType t, uint64_t rows,
                                      uint64_t cols, uint32_t n_experts, RawMatrix *out) {
    out->type_ = t;
    out->rows = rows;
    out->cols = cols;
    out->n_experts = n_experts;
    return lt_upload(b.ctx(), gguf_bytes, nbytes, static_cast<uint32_t>(t), rows, cols, n_experts, &out->data);
}

inline void release(Backend &b, RawMatrix &m) {
    lt_tensor_free(b.ctx(), m.data);
    m.data = nullptr;
}

namespace ops {

// rowBytes, src/ops/math.zig:194-208 (0 for unsupported types).
inline uint64_t rowBytes(GgmlType t, uint64_t cols) { return lt_row_bytes(static_cast<uint32_t>(t), cols); }

// quantMatvec(out, mat_data, mat_type, vec, rows, cols, row_buf),
// src/ops/math.zig:133-171.  Host vec/out; no row_buf (decode happens on the
// device).  quantMatvecPar (:277) is the same call: parallelism is the GPU's.
[[nodiscard]] inline lt_status quantMatvec(Backend &b, float *out, const RawMatrix &mat, const float *vec,
                                           uint64_t rows, uint64_t cols, uint32_t expert = 0) {
    return lt_quant_matvec_host(b.ctx(), out, mat.data, expert, vec, rows, cols);
}

// Device-resident variant for ntok activation rows.
[[nodiscard]] inline lt_status quantMatvecDev(Backend &b, float *dev_out, const RawMatrix &mat, const float *dev_vec,
                                              uint32_t ntok = 1, uint32_t expert = 0) {
    return lt_qmatvec(b.ctx(), mat.data, expert, dev_vec, dev_out, ntok);
}

// dequantRow(data, out, type), src/ops/math.zig:211-225: `row` of `mat`.
[[nodiscard]] inline lt_status dequantRow(Backend &b, const RawMatrix &mat, uint64_t row, float *dev_out) {
    return lt_dequant(b.ctx(), mat.data, row, 1, dev_out);
}

// rmsnorm(out, x, weight, eps), src/ops/math.zig:20-26 (device vectors).
[[nodiscard]] inline lt_status rmsnorm(Backend &b, float *dev_out, const float *dev_x, const float *dev_weight,
                                       uint32_t n, float eps) {
    return lt_rmsnorm(b.ctx(), dev_x, dev_weight, eps, n, 1, dev_out);
}

// softmax(x) in place, src/ops/math.zig:29-35.
[[nodiscard]] inline lt_status softmax(Backend &b, float *dev_x, uint32_t n) { return lt_softmax(b.ctx(), dev_x, n, 1); }

// routerTopKSoftmax(scores, out, router_w, router_in, scratch, pool),
// src/model/gemma4/forward.zig:648-668: ids (descending, lowest index on ties)
// and the selected softmax probabilities, times expert_scale[e] if given.
[[nodiscard]] inline lt_status routerTopKSoftmax(Backend &b, float *dev_selected_w, uint32_t *dev_out_idx, uint32_t k,
                                                 const RawMatrix &router_w, const float *dev_router_in,
                                                 bool norm_topk = false, const float *dev_expert_scale = nullptr) {
    return lt_moe_route(b.ctx(), router_w.data, dev_router_in, 1, k, norm_topk ? 1 : 0, dev_expert_scale, dev_out_idx,
                        dev_selected_w);
}

enum class Act : int { silu = LT_ACT_SILU, gelu = LT_ACT_GELU_TANH };

// moeForward(out, router_w, gate_up, down, x, n_experts_used, d_expert, pool,
// allocator), src/ops/moe.zig:18-77, on device vectors.  up == nullptr means
// `gate` is the fused gate_up tensor.  out is overwritten (the reference
// accumulates into a zeroed buffer).
[[nodiscard]] inline lt_status moeForward(Backend &b, float *dev_out, const RawMatrix &router_w, const RawMatrix &gate,
                                          const RawMatrix *up, const RawMatrix &down, const float *dev_x,
                                          uint32_t n_experts_used, Act act = Act::silu, bool norm_topk = false,
                                          const float *dev_expert_scale = nullptr, uint32_t ntok = 1) {
    return lt_moe_forward(b.ctx(), router_w.data, gate.data, up ? up->data : nullptr, down.data,
                          static_cast<int>(act), norm_topk ? 1 : 0, dev_expert_scale, dev_x, ntok, n_experts_used,
                          dev_out, nullptr, nullptr);
}

// greedy(logits), src/model/sample.zig:11-17: first index of the maximum.
[[nodiscard]] inline lt_status greedy(Backend &b, const float *dev_logits, uint32_t n, uint32_t *dev_idx) {
    return lt_argmax(b.ctx(), dev_logits, n, 1, dev_idx);
}

}  // namespace ops
}  // namespace llmtoy
