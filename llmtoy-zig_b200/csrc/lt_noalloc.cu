// lt_noalloc.cu — lt_moe_ffn_noalloc: the MoE FFN (dispatch + grouped gate/up
// + down + weighted combine) for callers that cannot allocate device memory.
//
// Some hosts cannot call cudaMalloc at all: a Zig or C program that receives
// its device buffers from an embedding runtime or a memory pool it does not
// own, code running while another owner holds the allocator (for example
// during CUDA-graph capture driven by someone else), or a plugin whose memory
// budget is fixed up front.  For them this entry point takes only caller-owned
// pointers and keeps its intermediate activations in a statically sized
// device array that lives in this library's module.
//
// The array (kNoallocScratchBytes) is part of the module, so every GPU that
// loads the library holds it until the process exits.  Every call shares it
// and it keeps the previous call's contents: the dispatch plan and the
// activations are fully rewritten each call, and the device error word and
// the gate/up block counters, which must start at zero, are cleared at the
// start of every call.  Kernels record a device-detected fault (an expert id
// past n_experts, a TMA copy that never landed) in the error word instead of
// faulting; lt_noalloc_status reads and clears it.  The array's device address
// is looked up once per device and kept: the library does not survive a
// cudaDeviceReset of a device it has already run on.  Calls
// whose work overlaps on the GPU (different streams, or graphs replayed
// concurrently) race on it; serialise them.
#include <mutex>

#include "llmtoy_cuda.h"
#include "lt_launch.cuh"

namespace lt {

constexpr size_t kNoallocScratchBytes = 8u << 20;  // 8 MiB per device

// [0, 256): device error word; then the MoE scratch carved per call.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint8_t *g_scratch_addr[kMaxDevices];  // device address of g_noalloc_scratch, per device

// Once per device, with that device current: look up the array's device
// address (host code only knows a host-side stand-in for the symbol).
lt_status scratch_address(int device, uint8_t **out) {
    if (device < 0 || device >= kMaxDevices) return LT_ENODEV;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[device]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) {
            cudaGetLastError();
            return LT_ECUDA;
        }
        g_scratch_addr[device] = static_cast<uint8_t *>(p);
    }
    *out = g_scratch_addr[device];
    return LT_OK;
}

size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

bool quantized_type(uint32_t t) { return is_quant_type(t); }

}  // namespace
}  // namespace lt

extern "C" lt_status lt_moe_ffn_noalloc(void *cuda_stream, const void *gate, const void *up, const void *down,
                                        uint32_t gate_type, uint32_t down_type, uint32_t n_experts,
                                        uint64_t d_model, uint64_t d_expert, int act, const float *dev_x,
                                        uint32_t ntok, const uint32_t *dev_ids, const float *dev_w, uint32_t k,
                                        float *dev_out) {
    using namespace lt;
    if (!gate || !down || !dev_x || !dev_ids || !dev_w || !dev_out) return LT_EINVAL;
    if (!quantized_type(gate_type) || !quantized_type(down_type)) return LT_EUNSUPPORTED_TYPE;
    if (n_experts == 0 || n_experts > 1024 || k == 0 || k > 16 || k > n_experts) return LT_EINVAL;
    if (act != LT_ACT_SILU && act != LT_ACT_GELU_TANH) return LT_EINVAL;
    if (d_expert % 32 != 0 || d_model % 32 != 0 || d_model > 65536 || d_expert > 65536) return LT_EINVAL;
    if ((is_k_type(gate_type) && d_model % 256 != 0) || (is_k_type(down_type) && d_expert % 256 != 0))
        return LT_EINVAL;
    // The caller's weights are used in place, so each GGUF row must already
    // sit at a 16-byte multiple (TMA bulk copies need 16-byte aligned rows).
    const uint64_t grb = row_bytes_of(gate_type, d_model), drb = row_bytes_of(down_type, d_expert);
    if (grb % 16 != 0 || drb % 16 != 0) return LT_EINVAL;
    if ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(down) | reinterpret_cast<uintptr_t>(up)) &
        15)
        return LT_EINVAL;
    if (ntok == 0) return LT_OK;

    // Scratch: quantised x rows, quantised h rows, dispatch plan.
    const size_t P = (size_t)ntok * k;
    const uint64_t xq_pitch = qact_row_pitch(d_model), hq_pitch = qact_row_pitch(d_expert);
    size_t off = 256;  // device error word
    auto take = [&](size_t b) {
        const size_t o = off;
        off += al256(b);
        return o;
    };
    const size_t o_xq = take((size_t)ntok * xq_pitch), o_hq = take(P * hq_pitch);
    const size_t o_na = take(4), o_ae = take((size_t)n_experts * 4), o_ao = take((size_t)n_experts * 4),
                 o_ac = take((size_t)n_experts * 4), o_pp = take(P * 4), o_ppos = take(P * 4);
    const size_t o_hf = take(P * d_expert * 4), n_cnt = P * (d_expert / 32), o_cnt = take(n_cnt * 4);
    if (off > kNoallocScratchBytes) return LT_EINVAL;  // beyond the static maximum

    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        cudaGetLastError();
        return LT_ECUDA;
    }
    uint8_t *base = nullptr;
    lt_status st = scratch_address(device, &base);
    if (st != LT_OK) return st;

    LaunchCfg c;
    c.stream = static_cast<cudaStream_t>(cuda_stream);
    c.pdl = true;
    c.dev_err = reinterpret_cast<int *>(base);
    c.num_sms = 0;
    c.prof = nullptr;

    MoePlan plan;
    plan.n_active = reinterpret_cast<uint32_t *>(base + o_na);
    plan.act_e = reinterpret_cast<uint32_t *>(base + o_ae);
    plan.act_off = reinterpret_cast<uint32_t *>(base + o_ao);
    plan.act_cnt = reinterpret_cast<uint32_t *>(base + o_ac);
    plan.pos_pair = reinterpret_cast<uint32_t *>(base + o_pp);
    plan.pair_pos = reinterpret_cast<uint32_t *>(base + o_ppos);

    const uint64_t F = d_expert;
    DevMat g{static_cast<const uint8_t *>(gate), gate_type, up ? F : 2 * F, d_model, grb, grb, n_experts};
    DevMat u{static_cast<const uint8_t *>(up), gate_type, F, d_model, grb, grb, n_experts};
    DevMat dn{static_cast<const uint8_t *>(down), down_type, d_model, F, drb, drb, n_experts};
    const bool direct = ntok == 1;

    // The error word and the gate/up block counters must start at zero: clear
    // them (memsets, not allocations).
    cudaError_t e = cudaMemsetAsync(base, 0, 4, c.stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(base + o_cnt, 0, n_cnt * 4, c.stream);
    if (e == cudaSuccess) e = launch_quantize(c, dev_x, (uint32_t)d_model, ntok, base + o_xq, xq_pitch);
    if (e == cudaSuccess && !direct) e = launch_moe_plan(c, dev_ids, ntok, k, n_experts, plan);
    if (e == cudaSuccess)
        e = launch_moe_gate_up(c, g, u, act, base + o_xq, xq_pitch, ntok, k, dev_ids, direct, plan,
                               reinterpret_cast<float *>(base + o_hf), reinterpret_cast<uint32_t *>(base + o_cnt),
                               base + o_hq, hq_pitch);
    if (e == cudaSuccess)
        e = launch_moe_down(c, dn, base + o_hq, hq_pitch, ntok, k, dev_ids, dev_w, direct, plan, nullptr, dev_out);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        cudaGetLastError();
        return e == cudaErrorMemoryAllocation ? LT_ENOMEM : LT_ECUDA;
    }
    return LT_OK;
}

extern "C" lt_status lt_noalloc_status(void *cuda_stream) {
    using namespace lt;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        cudaGetLastError();
        return LT_ECUDA;
    }
    uint8_t *base = nullptr;
    lt_status st = scratch_address(device, &base);
    if (st != LT_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
    int h = 0;
    // Ordered after the caller's lt_moe_ffn_noalloc calls on the same stream;
    // the copy to this pageable host word returns once it has landed.
    cudaError_t e = cudaMemcpyAsync(&h, base, 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && h != 0) e = cudaMemsetAsync(base, 0, 4, s);
    if (e == cudaSuccess && h != 0) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return LT_ECUDA;
    }
    if (h == DEV_ERR_BAD_INDEX) return LT_EINVAL;
    return h ? LT_ETIMEOUT : LT_OK;
}
