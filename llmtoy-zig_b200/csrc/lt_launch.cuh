// lt_launch.cuh — kernel launch helper (PDL attribute, profiler events) and
// shared-memory staging helpers used by every kernel file.
#pragma once

#include "lt_common.cuh"
#include "lt_internal.h"

namespace lt {

template <typename Kern, typename... Args>
inline cudaError_t launch_k(const LaunchCfg &c, const char *label, Kern kern, dim3 grid, dim3 block, size_t smem,
                            Args... args) {
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    cfg.numAttrs = 0;
    const bool timed = c.prof && c.prof->on;
    if (c.pdl && !timed) {  // events between kernels would serialise them anyway
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    Profiler::Rec rec;
    if (timed) c.prof->begin(label, c.stream, rec);
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
    if (timed) c.prof->end(rec, c.stream);
    return e;
}

// Static per-type profiler labels for "qmv", "moe_gate_up" and "moe_down".
template <uint32_t TYPE>
inline const char *type_label(const char *kind) {
    static const char *const names[4][8] = {
        {"qmv_q4k", "qmv_q6k", "qmv_q8_0", "qmv_q5_0", "qmv_q5_1", "qmv_q3k", "qmv_q5k", "qmv_iq4nl"},
        {"moe_gate_up_q4k", "moe_gate_up_q6k", "moe_gate_up_q8_0", "moe_gate_up_q5_0", "moe_gate_up_q5_1",
         "moe_gate_up_q3k", "moe_gate_up_q5k", "moe_gate_up_iq4nl"},
        {"moe_down_q4k", "moe_down_q6k", "moe_down_q8_0", "moe_down_q5_0", "moe_down_q5_1", "moe_down_q3k",
         "moe_down_q5k", "moe_down_iq4nl"},
        {"qmv_stream_q4k", "qmv_stream_q6k", "qmv_stream_q8_0", "qmv_stream_q5_0", "qmv_stream_q5_1",
         "qmv_stream_q3k", "qmv_stream_q5k", "qmv_stream_iq4nl"}};
    const int t = TYPE == T_Q4_K ? 0 : TYPE == T_Q6_K ? 1 : TYPE == T_Q8_0 ? 2 : TYPE == T_Q5_0 ? 3
                : TYPE == T_Q5_1 ? 4 : TYPE == T_Q3_K ? 5 : TYPE == T_Q5_K ? 6 : 7;
    const int k = kind[0] == 'q' ? (kind[3] == '_' ? 3 : 0) : kind[4] == 'g' ? 1 : 2;
    return names[k][t];
}

__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~(size_t)15; }

// Items (units one thread decodes) per weight row.
__host__ __device__ inline uint32_t items_per_row(uint32_t type, uint64_t cols) {
    if (!is_k_type(type)) return (uint32_t)((cols / 32 + 7) / 8);  // eight 32-element blocks
    return (uint32_t)(cols / 256);
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Wait for a TMA tile.  On timeout: record the error, wait once more for the
// copies still in flight (they target this CTA's shared memory), give up.
LT_DEVINL bool tile_wait(uint64_t *bar, int *dev_err) {
    if (mbar_wait_bounded(bar, 0, kWaitLimitNs)) return true;
    if (dev_err) atomicExch(dev_err, DEV_ERR_TMA_TIMEOUT);
    mbar_wait_bounded(bar, 0, kWaitLimitNs);
    return false;
}

LT_DEVINL float act_apply(int act, float g) {
    if (act == 1) {  // src/ops/math.zig:85-88
        const float c = 0.7978845608028654f;
        return 0.5f * g * (1.0f + tanhf(c * (g + 0.044715f * g * g * g)));
    }
    return g / (1.0f + expf(-g));  // src/ops/math.zig:38-40
}

}  // namespace lt
