// lt_ep.cu — building blocks of expert-parallel MoE (experts sharded across
// ranks, tokens exchanged with an all-to-all): the dispatch plan, the row
// gather that packs the send buffer, and the weighted combine of the rows
// that come back.  The reference has no expert parallelism (its MoE runs on
// one device, src/model/gemma4/forward.zig:463-479); the combine keeps its
// order: moe_buf is zeroed, then += scale * down, slot by slot.
#include "lt_launch.cuh"

namespace lt {

constexpr int kEpThreads = 1024;
constexpr int kEpMaxRanks = 8;

// Stable counting sort of the ntok*k (token, slot) pairs by destination rank
// (expert / (E / nranks)): send position of pair i = offset of its rank +
// number of earlier pairs bound to the same rank.  One block; pass 1 counts,
// pass 2 places chunk by chunk with warp ballots and a running cursor.
__global__ void __launch_bounds__(kEpThreads) k_ep_dispatch(const uint32_t *ids, uint32_t npairs, uint32_t k,
                                                            uint32_t epr, uint32_t nranks, uint32_t *send_counts,
                                                            uint32_t *send_token, uint32_t *send_local,
                                                            uint32_t *pair_pos) {
    __shared__ uint32_t s_cnt[kEpMaxRanks], s_base[kEpMaxRanks];
    __shared__ uint32_t s_warp[kEpThreads / 32][kEpMaxRanks];
    pdl_wait();
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < kEpMaxRanks) s_cnt[tid] = 0;
    __syncthreads();
    for (uint32_t i = tid; i < npairs; i += kEpThreads) atomicAdd(&s_cnt[min(ids[i] / epr, nranks - 1)], 1u);
    __syncthreads();
    if (tid == 0) {
        uint32_t off = 0;
        for (uint32_t r = 0; r < nranks; r++) {
            s_base[r] = off;
            send_counts[r] = s_cnt[r];
            off += s_cnt[r];
        }
    }
    __syncthreads();
    for (uint32_t c0 = 0; c0 < npairs; c0 += kEpThreads) {
        const uint32_t i = c0 + tid;
        const bool valid = i < npairs;
        const uint32_t e = valid ? ids[i] : 0;
        const uint32_t r = valid ? min(e / epr, nranks - 1) : 0xffffffffu;
        uint32_t before = 0;  // earlier pairs of rank r within this warp
        for (uint32_t rr = 0; rr < nranks; rr++) {
            const uint32_t m = __ballot_sync(0xffffffffu, r == rr);
            if (r == rr) before = __popc(m & ((1u << lane) - 1));
            if (lane == 0) s_warp[warp][rr] = __popc(m);
        }
        __syncthreads();
        if (valid) {
            uint32_t pos = s_base[r] + before;
            for (uint32_t w = 0; w < warp; w++) pos += s_warp[w][r];
            send_token[pos] = i / k;
            send_local[pos] = e - r * epr;
            pair_pos[i] = pos;
        }
        __syncthreads();
        if (tid < nranks) {  // advance the cursor of each rank by this chunk's pairs
            uint32_t add = 0;
            for (uint32_t w = 0; w < kEpThreads / 32; w++) add += s_warp[w][tid];
            s_base[tid] += add;
        }
        __syncthreads();
    }
}

// dst[i][:] = src[idx[i]][:], float4 columns; one row per blockIdx.x.
__global__ void k_gather_rows(const float *src, uint32_t cols4, const uint32_t *idx, uint32_t n, float *dst) {
    pdl_wait();
    const uint32_t i = blockIdx.x, c = blockIdx.y * blockDim.x + threadIdx.x;
    if (i >= n || c >= cols4) return;
    reinterpret_cast<float4 *>(dst)[(size_t)i * cols4 + c] =
        reinterpret_cast<const float4 *>(src)[(size_t)idx[i] * cols4 + c];
}

cudaError_t launch_ep_dispatch(const LaunchCfg &c, const uint32_t *ids, uint32_t ntok, uint32_t k, uint32_t E,
                               uint32_t nranks, uint32_t *send_counts, uint32_t *send_token, uint32_t *send_local,
                               uint32_t *pair_pos) {
    if (nranks == 0 || nranks > (uint32_t)kEpMaxRanks || E % nranks != 0) return cudaErrorInvalidValue;
    return launch_k(c, "ep_dispatch", k_ep_dispatch, dim3(1), dim3(kEpThreads), 0, ids, ntok * k, k, E / nranks,
                    nranks, send_counts, send_token, send_local, pair_pos);
}

cudaError_t launch_gather_rows(const LaunchCfg &c, const float *src, uint64_t cols, const uint32_t *idx, uint32_t n,
                               float *dst) {
    if (cols % 4 != 0) return cudaErrorInvalidValue;
    const uint32_t cols4 = (uint32_t)(cols / 4);
    return launch_k(c, "gather_rows", k_gather_rows, dim3(n, (cols4 + 255) / 256), dim3(256), 0, src, cols4, idx, n,
                    dst);
}

}  // namespace lt
