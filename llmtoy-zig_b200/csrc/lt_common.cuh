// lt_common.cuh — device helpers shared by the sm_100a kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define LT_DEVINL __device__ __forceinline__

namespace lt {

// GGUF type codes (src/gguf/types.zig:23-52).
enum : uint32_t {
    T_F32 = 0, T_F16 = 1, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14,
    T_IQ4_NL = 20
};

// Block-quantised weight types the matvec kernels decode.
__host__ __device__ constexpr bool is_quant_type(uint32_t t) {
    return t == T_Q5_0 || t == T_Q5_1 || t == T_Q8_0 || t == T_Q3_K || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K ||
           t == T_IQ4_NL;
}
// 256-element superblock types (the rest use 32-element blocks).
__host__ __device__ constexpr bool is_k_type(uint32_t t) {
    return t == T_Q3_K || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K;
}

constexpr int kQK = 256;          // K-quant superblock elements
// IQ4_NL's non-linear table (src/quant/dequant.zig:618-621) as int8 bytes,
// entries 0-3, 4-7, 8-11, 12-15 little-endian: byte-permute lookups.
constexpr uint32_t kIq4T0 = 0xBFAD9881u, kIq4T1 = 0xF6EADDCFu, kIq4T2 = 0x26190D01u, kIq4T3 = 0x71594535u;

LT_DEVINL int iq4nl_value(uint32_t nib) {
    const uint32_t v = nib < 8 ? __byte_perm(kIq4T0, kIq4T1, nib) : __byte_perm(kIq4T2, kIq4T3, nib & 7u);
    return (int)(int8_t)(v & 0xffu);
}

// Four nibbles (one per byte of n, values 0..15) to their four int8 table values.
LT_DEVINL uint32_t iq4nl_lookup4(uint32_t n) {
    const uint32_t x = n & 0x07070707u, y = x | (x >> 4);
    const uint32_t sel = (y & 0xffu) | ((y >> 8) & 0xff00u);
    const uint32_t lo = __byte_perm(kIq4T0, kIq4T1, sel), hi = __byte_perm(kIq4T2, kIq4T3, sel);
    const uint32_t m = ((n >> 3) & 0x01010101u) * 0xffu;
    return (hi & m) | (lo & ~m);
}

constexpr int kQ4KBytes = 144;    // src/quant/dequant.zig:155
constexpr int kQ6KBytes = 210;    // src/quant/dequant.zig:235
constexpr int kQ8Bytes = 34;      // src/quant/dequant.zig:40
constexpr int kQ8Elems = 32;

// Elements covered by one "item": the unit of work a lane decodes at once.
// K-quants: one superblock; Q8_0: eight 34-byte blocks (272 B, 16-B aligned).
constexpr int kItemElems = 256;
// x vectors live in shared memory with this per-item stride (floats): the
// 4-float pad puts consecutive items 4 banks apart, so 8 lanes reading 8
// different items with 128-bit loads hit 32 distinct banks.
constexpr int kItemStride = kItemElems + 4;

LT_DEVINL float f16_bits_to_f32(uint32_t h) {
    return __half2float(__ushort_as_half((unsigned short)(h & 0xffffu)));
}

// IEEE f32 -> f16 bits, round to nearest even (what Zig's @floatCast does),
// in integer arithmetic: normals by mantissa rounding, subnormals as the
// nearest integer multiple of 2^-24, overflow to infinity.
LT_DEVINL uint32_t f32_to_f16_bits(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u);
    if (ax >= 0x477ff000u) return sign | 0x7c00u;
    if (ax < 0x38800000u) return sign | (uint32_t)__float2int_rn(__uint_as_float(ax) * 16777216.0f);
    uint32_t r = (((ax >> 23) - 112u) << 10) | ((ax >> 13) & 0x3ffu);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return sign | r;
}

// KV-cache elements: f32, or IEEE f16 stored rounded to nearest even.
LT_DEVINL float kv_ld(const void *base, size_t i, uint32_t f16) {
    return f16 ? f16_bits_to_f32(reinterpret_cast<const unsigned short *>(base)[i])
               : reinterpret_cast<const float *>(base)[i];
}
LT_DEVINL void kv_st(void *base, size_t i, float v, uint32_t f16) {
    if (f16)
        reinterpret_cast<unsigned short *>(base)[i] = (unsigned short)f32_to_f16_bits(v);
    else
        reinterpret_cast<float *>(base)[i] = v;
}
// The value a cache store then load returns.
LT_DEVINL float kv_round(float v, uint32_t f16) { return f16 ? f16_bits_to_f32(f32_to_f16_bits(v)) : v; }

// Read-only 128-bit global load (weights are never written while a kernel
// runs), allocated in L1 only if it streams: weights are touched once.
LT_DEVINL uint4 ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Packed fp32x2 arithmetic (sm_100+): two IEEE round-to-nearest results per
// instruction, identical to the scalar ops lane by lane.
union f2u {
    float2 f;
    unsigned long long u;
};

LT_DEVINL float2 ffma2(float2 a, float2 b, float2 c) {
    f2u A, B, C, D;
    A.f = a; B.f = b; C.f = c;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(D.u) : "l"(A.u), "l"(B.u), "l"(C.u));
    return D.f;
}

LT_DEVINL float2 fadd2(float2 a, float2 b) {
    f2u A, B, D;
    A.f = a; B.f = b;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(D.u) : "l"(A.u), "l"(B.u));
    return D.f;
}

// Exact integer-to-float for a byte in [0,255]: PRMT the byte into the low
// mantissa of 2^23 (bits 0x4B0000XX == 8388608 + XX); the caller subtracts
// the bias with one (packed) add.  sel picks byte 0..3 of w.
LT_DEVINL float byte_biased(uint32_t w, int sel) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | (uint32_t)sel));
}

constexpr float kMagic = 8388608.0f;  // 2^23

LT_DEVINL float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum of one value per thread over the block (warp sums, then the warps in order).
LT_DEVINL float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
    for (int i = 0; i < nw; i++) s += red[i];
    return s;
}

// 1 / sqrt(sum(x^2) / n + eps) over the block (math.zig:20-26): per-thread sums
// over 16-element strided batches, then block_sum.  One order for every kernel
// that normalises a row this way, so they agree bit for bit.
LT_DEVINL float rms_inv_block(const float *x, uint32_t n, float eps, float *red) {
    constexpr int kBatch = 16;
    float ss = 0.0f;
    for (uint32_t base = threadIdx.x; base < n; base += kBatch * blockDim.x) {
        float v[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; j++) {
            const uint32_t i = base + j * blockDim.x;
            v[j] = i < n ? x[i] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kBatch; j++) ss += v[j] * v[j];
    }
    ss = block_sum(ss, red);
    return 1.0f / sqrtf(ss / (float)n + eps);
}


// Programmatic dependent launch.  Data written by the previous kernel on the
// stream may only be read after pdl_wait(); kernels that are not launched
// with the PDL attribute see these as no-ops.
LT_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LT_DEVINL void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// ── error reporting ────────────────────────────────────────────────────────
// Kernels never trap.  A bounded wait that gives up records a code in the
// context's device error word; the host turns it into LT_ETIMEOUT.
enum : int { DEV_ERR_NONE = 0, DEV_ERR_TMA_TIMEOUT = 1, DEV_ERR_GRID_TIMEOUT = 2, DEV_ERR_BAD_INDEX = 3 };

// ── mbarrier + TMA bulk copy (global -> shared) ────────────────────────────
LT_DEVINL uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

LT_DEVINL void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

LT_DEVINL void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

LT_DEVINL void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// 1-D bulk copy; dst/src 16-byte aligned, bytes a multiple of 16.
LT_DEVINL void tma_load_1d(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

LT_DEVINL bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}

// Wait for `phase` of `bar` with an upper bound of about `limit_ns` of
// wall time (globaltimer).  Returns false if it gave up.
LT_DEVINL bool mbar_wait_bounded(uint64_t *bar, uint32_t phase, uint64_t limit_ns) {
    if (mbar_try_wait(bar, phase)) return true;
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
        if (mbar_try_wait(bar, phase)) return true;
        uint64_t t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > limit_ns) return false;
    }
}

LT_DEVINL uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ── grid-wide synchronisation for kernels whose CTAs are all resident ────────
// Counters that only grow.  Each CTA adds exactly 1 per launch to each, so
// with G CTAs a counter is a multiple of G between launches (the next launch
// starts after the previous one completed), and launch n's arrivals complete
// it at (n + 1) * G: the "epoch" of the launch, the same number in every CTA.
// Arrival is unconditional (also after a timed-out wait), which keeps that
// invariant.
LT_DEVINL uint64_t ld_acquire_u64(const unsigned long long *p) {
    uint64_t v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
LT_DEVINL uint64_t ld_relaxed_u64(const unsigned long long *p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
LT_DEVINL void st_relaxed_u64(unsigned long long *p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
LT_DEVINL void red_release_add_u64(unsigned long long *p, uint64_t v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Orders this thread's generic-proxy global accesses with its later (or, on
// the producer side, other threads' later) TMA accesses of global memory.
LT_DEVINL void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Thread 0: arrive on the epoch counter and return this launch's epoch.
LT_DEVINL uint64_t grid_epoch(unsigned long long *ctr, uint32_t G) {
    const uint64_t old = atomicAdd(ctr, 1ull);
    return old - old % G + G;
}

// Whole block: publish this CTA's global writes and arrive (no return value).
// The block barrier orders the CTA's writes before thread 0's release add,
// which publishes them at GPU scope (no separate fence: a fence.sc there
// measured ~1 us slower per hand-off on B200).
LT_DEVINL void grid_arrive(unsigned long long *ctr) {
    __syncthreads();
    if (threadIdx.x == 0) red_release_add_u64(ctr, 1ull);
}

// Whole block: bounded wait (limit_ns of wall time) until the counter
// reaches target; on timeout records DEV_ERR_GRID_TIMEOUT and continues.
LT_DEVINL void grid_wait(const unsigned long long *ctr, uint64_t target, int *dev_err, uint64_t limit_ns) {
    if (threadIdx.x == 0) {
        if (ld_acquire_u64(ctr) < target) {
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_u64(ctr) < target) {
                if (globaltimer_ns() - t0 > limit_ns) {
                    if (dev_err) atomicExch(dev_err, DEV_ERR_GRID_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncthreads();  // passes thread 0's acquire on to the block
}

// The same hand-off over kGridSplit counters, one 128-byte line each: CTA c
// arrives on counter c % kGridSplit (fewer atomics queued at one L2 slice),
// lanes 0..kGridSplit-1 of warp 0 poll one counter each and the hand-off
// completes when their sum reaches the target.  Every counter only grows and
// receives the same arrivals each launch, so a sum at the target means every
// counter is at its own.
constexpr uint32_t kGridSplit = 8;
constexpr size_t kGridSplitStride = 16;  // u64 units
constexpr size_t kGridSplitBytes = 8 * kGridSplitStride * kGridSplit;

LT_DEVINL void grid_arrive_split(unsigned long long *ctr) {
    __syncthreads();
    if (threadIdx.x == 0) red_release_add_u64(ctr + kGridSplitStride * (blockIdx.x % kGridSplit), 1ull);
}

// Arrivals of every CTA of a G-CTA grid at once (by one thread), so that a
// hand-off this launch skips keeps its counters in step.
LT_DEVINL void grid_arrive_split_all(unsigned long long *ctr, uint32_t G) {
    for (uint32_t j = 0; j < kGridSplit; j++)
        atomicAdd(ctr + kGridSplitStride * j, (unsigned long long)((G + kGridSplit - 1 - j) / kGridSplit));
}

LT_DEVINL void grid_wait_split(const unsigned long long *ctr, uint64_t target, int *dev_err, uint64_t limit_ns) {
    if (threadIdx.x < 32) {
        const uint32_t lane = threadIdx.x;
        const unsigned long long *p = ctr + kGridSplitStride * (lane % kGridSplit);
        auto total = [&]() {
            uint64_t v = lane < kGridSplit ? ld_acquire_u64(p) : 0ull;
#pragma unroll
            for (int o = kGridSplit / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            return __shfl_sync(0xffffffffu, v, 0);
        };
        if (total() < target) {
            const uint64_t t0 = __shfl_sync(0xffffffffu, globaltimer_ns(), 0);
            for (;;) {
                if (total() >= target) break;
                // lane 0's clock decides, so the warp leaves the loop together
                if (__shfl_sync(0xffffffffu, globaltimer_ns() - t0 > limit_ns ? 1 : 0, 0)) {
                    if (lane == 0 && dev_err) atomicExch(dev_err, DEV_ERR_GRID_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncthreads();  // passes the pollers' acquire on to the block
}

// Fire-and-forget prefetch of [p, p + bytes) into L2 (16-byte aligned, bytes a multiple of 16).
LT_DEVINL void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// CTA c of G prefetches its 16-byte aligned share of [p, p + bytes) into L2.
LT_DEVINL void prefetch_l2_share(const uint8_t *p, uint64_t bytes, uint32_t c, uint32_t G) {
    const uint64_t n = bytes / 16;
    const uint64_t b0 = 16 * (c * n / G), b1 = 16 * ((c + 1) * n / G);
    for (uint64_t b = b0; b < b1; b += 65536) prefetch_l2(p + b, (uint32_t)(b1 - b < 65536 ? b1 - b : 65536));
}

LT_DEVINL uint4 lds128(const void *p) {
    return *reinterpret_cast<const uint4 *>(p);
}
LT_DEVINL uint32_t lds32(const void *p) {
    return *reinterpret_cast<const uint32_t *>(p);
}

// ── integer dot products ───────────────────────────────────────────────────
// d = c + a.s16[0]*b.byte[0|2] + a.s16[1]*b.byte[1|3]  (b bytes unsigned)
LT_DEVINL int dp2a_lo_su(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
LT_DEVINL int dp2a_hi_su(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// Same with signed bytes (Q8_0 quants).
LT_DEVINL int dp2a_lo_ss(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
LT_DEVINL int dp2a_hi_ss(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// d = c + sum_i a.s8[i] * b.byte[i]  (b bytes unsigned / signed)
LT_DEVINL int dp4a_su(int a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
LT_DEVINL int dp4a_ss(int a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Small non-negative integer held in byte `sel` of w, as an exact float.
LT_DEVINL float byte_to_f32(uint32_t w, int sel) {
    return byte_biased(w, sel) - kMagic;
}

}  // namespace lt
