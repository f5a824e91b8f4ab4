// lt_ep_nccl.cu — the expert-parallel MoE layer behind the C ABI: lt_ep_init,
// lt_moe_ffn_ep.  Rank r of N holds experts [r*E/N, (r+1)*E/N); one call runs
// the layer over this rank's tokens:
//
//   route    ids, weights                          (lt_moe_route)
//   dispatch pairs ordered by destination rank     (lt_ep_dispatch)
//   counts   all-gather of every rank's N send counts; the host reads them
//            (bounded wait) to size the exchange
//   exchange token rows and local expert ids        (NCCL send/recv, grouped)
//   experts  the received rows through this rank's experts, k = 1, weight 1
//   return   results back to their token's rank     (NCCL send/recv)
//   combine  slot-order weighted sum (+ residual)   (lt_moe_combine)
//
// The reference runs its MoE on one device (src/model/gemma4/forward.zig:
// 463-479; the GPU seam is GpuWeights.runExpertBatch, gpu_weights.zig:2748);
// sharding keeps its arithmetic: each (token, slot) pair is computed by the
// rank that holds its expert and combined on the token's own rank in slot
// order, so the result equals the single-device layer's.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, the copy a host process
// has loaded already when there is one), so the library needs it only when a
// host uses these entry points.  Every host-side wait of a call is bounded by
// the ep's timeout: one that runs out aborts the communicator (NCCL's kernels
// then return) and the call reports LT_ETIMEOUT; a communicator error reported
// by NCCL on the way becomes LT_ECUDA.  An aborted ep refuses further calls.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "llmtoy_cuda.h"
#include "lt_internal.h"

namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) getUniqueId;
    decltype(&ncclCommInitRank) commInitRank;
    decltype(&ncclCommDestroy) commDestroy;
    decltype(&ncclCommAbort) commAbort;
    decltype(&ncclCommGetAsyncError) commGetAsyncError;
    decltype(&ncclGroupStart) groupStart;
    decltype(&ncclGroupEnd) groupEnd;
    decltype(&ncclSend) send;
    decltype(&ncclRecv) recv;
    decltype(&ncclAllGather) allGather;
    decltype(&ncclGetErrorString) errorString;
};

const NcclApi *nccl_api() {
    static std::once_flag once;
    static NcclApi api;
    static bool ok = false;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // a copy the process loaded already
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) return;
        auto sym = [h](const char *n) { return dlsym(h, n); };
        api.getUniqueId = reinterpret_cast<decltype(api.getUniqueId)>(sym("ncclGetUniqueId"));
        api.commInitRank = reinterpret_cast<decltype(api.commInitRank)>(sym("ncclCommInitRank"));
        api.commDestroy = reinterpret_cast<decltype(api.commDestroy)>(sym("ncclCommDestroy"));
        api.commAbort = reinterpret_cast<decltype(api.commAbort)>(sym("ncclCommAbort"));
        api.commGetAsyncError = reinterpret_cast<decltype(api.commGetAsyncError)>(sym("ncclCommGetAsyncError"));
        api.groupStart = reinterpret_cast<decltype(api.groupStart)>(sym("ncclGroupStart"));
        api.groupEnd = reinterpret_cast<decltype(api.groupEnd)>(sym("ncclGroupEnd"));
        api.send = reinterpret_cast<decltype(api.send)>(sym("ncclSend"));
        api.recv = reinterpret_cast<decltype(api.recv)>(sym("ncclRecv"));
        api.allGather = reinterpret_cast<decltype(api.allGather)>(sym("ncclAllGather"));
        api.errorString = reinterpret_cast<decltype(api.errorString)>(sym("ncclGetErrorString"));
        ok = api.getUniqueId && api.commInitRank && api.commDestroy && api.commAbort && api.commGetAsyncError &&
             api.groupStart && api.groupEnd && api.send && api.recv && api.allGather && api.errorString;
    });
    return ok ? &api : nullptr;
}

size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace

struct lt_ep {
    lt_ctx *ctx = nullptr;
    ncclComm_t comm = nullptr;
    uint32_t nranks = 0, rank = 0, timeout_ms = 0;
    int device = 0;
    cudaStream_t stream = nullptr;  // the context's stream when the ep was made
    bool aborted = false;
    cudaEvent_t ev = nullptr;
    uint32_t *host_counts = nullptr;  // pinned [nranks * nranks]
    uint8_t *buf = nullptr;           // device scratch, grown on demand
    size_t buf_bytes = 0;
};

namespace {

lt_status ep_grow(lt_ep *ep, size_t bytes) {
    if (bytes <= ep->buf_bytes) return LT_OK;
    if (ep->buf) cudaFree(ep->buf);
    ep->buf = nullptr;
    ep->buf_bytes = 0;
    if (cudaMalloc(&ep->buf, bytes) != cudaSuccess) {
        cudaGetLastError();
        return LT_ENOMEM;
    }
    ep->buf_bytes = bytes;
    return LT_OK;
}

// Wait for the work queued on the stream so far, within the ep's timeout.
lt_status ep_wait(lt_ep *ep) {
    const NcclApi *api = nccl_api();
    if (cudaEventRecord(ep->ev, ep->stream) != cudaSuccess) return LT_ECUDA;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(ep->timeout_ms);
    for (;;) {
        const cudaError_t e = cudaEventQuery(ep->ev);
        if (e == cudaSuccess) return LT_OK;
        if (e != cudaErrorNotReady) return LT_ECUDA;
        ncclResult_t ae = ncclSuccess;
        api->commGetAsyncError(ep->comm, &ae);
        if (ae != ncclSuccess && ae != ncclInProgress) {
            api->commAbort(ep->comm);
            ep->aborted = true;
            return LT_ECUDA;
        }
        if (std::chrono::steady_clock::now() > deadline) {
            api->commAbort(ep->comm);  // the communicator's kernels give up and the stream drains
            ep->aborted = true;
            return LT_ETIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

lt_status nccl_ok(lt_ep *ep, ncclResult_t r) {
    if (r == ncclSuccess) return LT_OK;
    nccl_api()->commAbort(ep->comm);
    ep->aborted = true;
    return LT_ECUDA;
}

}  // namespace

extern "C" {

lt_status lt_ep_unique_id(uint8_t id_out[128]) {
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
    if (!id_out) return LT_EINVAL;
    const NcclApi *api = nccl_api();
    if (!api) return LT_ENODEV;
    ncclUniqueId id;
    if (api->getUniqueId(&id) != ncclSuccess) return LT_ECUDA;
    std::memcpy(id_out, &id, 128);
    return LT_OK;
}

lt_status lt_ep_init(lt_ctx *ctx, uint32_t nranks, uint32_t rank, const uint8_t id[128], uint32_t timeout_ms,
                     lt_ep **out) {
    if (!ctx || !id || !out || nranks == 0 || nranks > 8 || rank >= nranks || timeout_ms == 0) return LT_EINVAL;
    *out = nullptr;
    const NcclApi *api = nccl_api();
    if (!api) return LT_ENODEV;
    lt_ep *ep = new lt_ep;
    ep->ctx = ctx;
    ep->nranks = nranks;
    ep->rank = rank;
    ep->timeout_ms = timeout_ms;
    if (lt_sync(ctx) != LT_OK) {
        delete ep;
        return LT_ECUDA;
    }
    ep->device = lt::ctx_device(ctx);
    ep->stream = lt::ctx_stream(ctx);
    ncclUniqueId uid;
    std::memcpy(&uid, id, 128);
    if (cudaEventCreateWithFlags(&ep->ev, cudaEventDisableTiming) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void **>(&ep->host_counts), (size_t)nranks * nranks * 4) != cudaSuccess) {
        cudaGetLastError();
        if (ep->ev) cudaEventDestroy(ep->ev);
        delete ep;
        return LT_ENOMEM;
    }
    if (api->commInitRank(&ep->comm, (int)nranks, uid, (int)rank) != ncclSuccess) {
        cudaEventDestroy(ep->ev);
        cudaFreeHost(ep->host_counts);
        delete ep;
        return LT_ECUDA;
    }
    *out = ep;
    return LT_OK;
}

lt_status lt_ep_free(lt_ep *ep) {
    if (!ep) return LT_OK;
    cudaSetDevice(ep->device);
    const NcclApi *api = nccl_api();
    if (ep->comm && api && !ep->aborted) api->commDestroy(ep->comm);  // an aborted one is released already
    if (ep->buf) cudaFree(ep->buf);
    if (ep->host_counts) cudaFreeHost(ep->host_counts);
    if (ep->ev) cudaEventDestroy(ep->ev);
    delete ep;
    return LT_OK;
}

lt_status lt_moe_ffn_ep(lt_ctx *ctx, lt_ep *ep, const lt_tensor *router, const lt_tensor *gate, const lt_tensor *up,
                        const lt_tensor *down, int act, int norm_topk, const float *dev_expert_scale,
                        const float *dev_norm_w, float eps, const float *dev_x, uint32_t ntok, uint32_t k,
                        float *dev_out) {
    if (!ctx || !ep || !router || !gate || !down || !dev_x || !dev_out || ep->ctx != ctx) return LT_EINVAL;
    if (ep->aborted) return LT_ETIMEOUT;
    if (cudaSetDevice(ep->device) != cudaSuccess) return LT_ECUDA;
    if (lt::ctx_stream(ctx) != ep->stream) return LT_EINVAL;  // one stream for the ep's life
    lt_tensor_desc rd{}, gd{};
    lt_status st;
    if ((st = lt_tensor_describe(router, &rd)) != LT_OK || (st = lt_tensor_describe(gate, &gd)) != LT_OK) return st;
    const uint32_t N = ep->nranks, E = (uint32_t)rd.rows;
    const uint64_t d = rd.cols;
    if (E == 0 || E % N != 0 || gd.n_experts != E / N || gd.cols != d || k == 0 || k > E) return LT_EINVAL;
    const ncclDataType_t f32 = ncclFloat32, u32 = ncclUint32;
    const NcclApi *api = nccl_api();
    const size_t P = (size_t)ntok * k;
    // scratch before the exchange: xn, ids, w, counts, send_token, send_local, pair_pos, all counts, send rows
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off += al256(b ? b : 1);
        return o;
    };
    const size_t o_xn = take((size_t)ntok * d * 4), o_ids = take(P * 4), o_w = take(P * 4), o_cnt = take(N * 4),
                 o_st = take(P * 4), o_sl = take(P * 4), o_pp = take(P * 4), o_all = take((size_t)N * N * 4),
                 o_sr = take(P * d * 4), o_ys = take(P * d * 4);
    const size_t pre = off;
    if ((st = ep_grow(ep, pre)) != LT_OK) return st;
    uint8_t *b = ep->buf;
    float *xn = reinterpret_cast<float *>(b + o_xn);
    uint32_t *ids = reinterpret_cast<uint32_t *>(b + o_ids), *cnt = reinterpret_cast<uint32_t *>(b + o_cnt);
    float *w = reinterpret_cast<float *>(b + o_w);
    uint32_t *send_token = reinterpret_cast<uint32_t *>(b + o_st), *send_local = reinterpret_cast<uint32_t *>(b + o_sl);
    uint32_t *pair_pos = reinterpret_cast<uint32_t *>(b + o_pp), *all = reinterpret_cast<uint32_t *>(b + o_all);
    float *send_rows = reinterpret_cast<float *>(b + o_sr), *y_send = reinterpret_cast<float *>(b + o_ys);

    const float *xin = dev_x;
    if (ntok) {
        if (dev_norm_w) {
            if ((st = lt_rmsnorm(ctx, dev_x, dev_norm_w, eps, (uint32_t)d, ntok, xn)) != LT_OK) return st;
            xin = xn;
        }
        if ((st = lt_moe_route(ctx, router, xin, ntok, k, norm_topk, dev_expert_scale, ids, w)) != LT_OK) return st;
    }
    if ((st = lt_ep_dispatch(ctx, ids, ntok, k, E, N, cnt, send_token, send_local, pair_pos)) != LT_OK) return st;
    if ((st = nccl_ok(ep, api->allGather(cnt, all, N, u32, ep->comm, ep->stream))) != LT_OK) return st;
    if (cudaMemcpyAsync(ep->host_counts, all, (size_t)N * N * 4, cudaMemcpyDeviceToHost, ep->stream) != cudaSuccess)
        return LT_ECUDA;
    if ((st = ep_wait(ep)) != LT_OK) return st;  // the split sizes: the call's one host sync
    std::vector<size_t> sc(N), rc(N), so(N + 1, 0), ro(N + 1, 0);
    for (uint32_t r = 0; r < N; r++) {
        sc[r] = ep->host_counts[ep->rank * N + r];
        rc[r] = ep->host_counts[r * N + ep->rank];
        so[r + 1] = so[r] + sc[r];
        ro[r + 1] = ro[r] + rc[r];
    }
    if (so[N] != P) return LT_ECUDA;
    const size_t R = ro[N];
    // scratch after the exchange sizes are known (nothing is in flight: the stream just drained)
    const size_t o_rr = take(R * d * 4), o_rl = take(R * 4), o_one = take(R * 4), o_yr = take(R * d * 4);
    if (off > ep->buf_bytes) {
        std::vector<uint8_t> keep(pre);  // the dispatch plan survives the regrowth
        if (cudaMemcpy(keep.data(), ep->buf, pre, cudaMemcpyDeviceToHost) != cudaSuccess) return LT_ECUDA;
        if ((st = ep_grow(ep, off)) != LT_OK) return st;
        if (cudaMemcpy(ep->buf, keep.data(), pre, cudaMemcpyHostToDevice) != cudaSuccess) return LT_ECUDA;
        b = ep->buf;
        xn = reinterpret_cast<float *>(b + o_xn);
        w = reinterpret_cast<float *>(b + o_w);
        send_token = reinterpret_cast<uint32_t *>(b + o_st);
        send_local = reinterpret_cast<uint32_t *>(b + o_sl);
        pair_pos = reinterpret_cast<uint32_t *>(b + o_pp);
        send_rows = reinterpret_cast<float *>(b + o_sr);
        y_send = reinterpret_cast<float *>(b + o_ys);
        xin = dev_norm_w ? xn : dev_x;
    }
    float *recv_rows = reinterpret_cast<float *>(b + o_rr), *ones = reinterpret_cast<float *>(b + o_one);
    uint32_t *recv_local = reinterpret_cast<uint32_t *>(b + o_rl);
    float *y_recv = reinterpret_cast<float *>(b + o_yr);

    if (P && (st = lt_gather_rows(ctx, xin, d, send_token, (uint32_t)P, send_rows)) != LT_OK) return st;
    if ((st = nccl_ok(ep, api->groupStart())) != LT_OK) return st;
    for (uint32_t r = 0; r < N; r++) {
        api->send(send_rows + so[r] * d, sc[r] * d, f32, (int)r, ep->comm, ep->stream);
        api->recv(recv_rows + ro[r] * d, rc[r] * d, f32, (int)r, ep->comm, ep->stream);
        api->send(send_local + so[r], sc[r], u32, (int)r, ep->comm, ep->stream);
        api->recv(recv_local + ro[r], rc[r], u32, (int)r, ep->comm, ep->stream);
    }
    if ((st = nccl_ok(ep, api->groupEnd())) != LT_OK) return st;
    if (R) {
        if (lt::launch_fill_f32(ep->stream, ones, R, 1.0f) != cudaSuccess) return LT_ECUDA;
        if ((st = lt_moe_ffn(ctx, gate, up, down, act, recv_rows, (uint32_t)R, recv_local, ones, 1, y_recv)) != LT_OK)
            return st;
    }
    if ((st = nccl_ok(ep, api->groupStart())) != LT_OK) return st;
    for (uint32_t r = 0; r < N; r++) {
        api->send(y_recv + ro[r] * d, rc[r] * d, f32, (int)r, ep->comm, ep->stream);
        api->recv(y_send + so[r] * d, sc[r] * d, f32, (int)r, ep->comm, ep->stream);
    }
    if ((st = nccl_ok(ep, api->groupEnd())) != LT_OK) return st;
    if (ntok &&
        (st = lt_moe_combine(ctx, y_send, d, pair_pos, w, ntok, k, dev_norm_w ? dev_x : nullptr, dev_out)) != LT_OK)
        return st;
    return ep_wait(ep);  // bounded: the exchanges of this call have completed when it returns LT_OK
}

}  // extern "C"
