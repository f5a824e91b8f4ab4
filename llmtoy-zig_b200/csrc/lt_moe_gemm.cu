// lt_moe_gemm.cu — grouped expert GEMM on the 5th-generation tensor cores
// (tcgen05) for multi-token MoE batches with Q4_K experts (prefill; the
// reference's expert loop src/model/gemma4/forward.zig:463-479 and
// src/ops/moe.zig:61-76 run over many tokens).
//
// Pipeline: dispatch plan (lt_moe.cu) -> tile list -> activation prep (f32
// rows -> f16 hi/lo planes) -> gate/up GEMM with SwiGLU/GeGLU epilogue ->
// prep of h -> down GEMM -> weighted combine in slot order (+ residual).
//
// Exactness.  A Q4_K weight is d*sc*q - dmin*m (dequant.zig:157-187).  The
// tensor core multiplies f16 operands exactly and accumulates in f32, so:
//   * A = sc*q, an integer <= 945, exact in f16 (dequantised from the nibbles
//     in shared memory: (1024+q) * sc - 1024*sc in one HFMA2);
//   * the activation is split into two f16 planes, x*2^-e = hi + lo
//     (2^-e puts max|x| of the row in [0.5, 1)), ~22 significant bits;
//   * d differs per superblock, so each superblock accumulates into its own
//     TMEM accumulator and the epilogue applies sum_sb d_sb * acc_sb;
//   * the min term sum_sb sum_j (dmin_sb*m_j) * (sum of the 32 x of sub-block
//     j) is one more MMA: dmin*m is exact in f32 and split into two f16
//     planes, the sub-block sums likewise (hi*hi + hi*lo + lo*hi).
//
// CTA tile: 128 weight rows x 32 positions.  For gate/up the rows are 64
// gate rows and the same 64 up rows, so the epilogue forms h = act(g)*u.
// Per stage (half a superblock, K = 128) the CTA's 128 threads dequantise
// one weight row each (raw Q4_K rows arrive by TMA bulk copies, a superblock
// ahead) and cp.async gathers the activation rows of the tile's positions,
// two stages ahead; one thread issues the MMAs, which run while the next
// stage is prepared.
#include <cuda_fp16.h>

#include "lt_launch.cuh"
#include "lt_umma.cuh"

namespace lt {

constexpr int kGThreads = 128;
constexpr int kGN = 32;     // positions per tile (MMA N)
constexpr int kGM = 128;    // weight rows per tile (MMA M)
constexpr int kGMaxSb = 8;  // superblocks per row (K <= 2048)

// Dynamic shared memory, offsets from a 1024-byte aligned base.
constexpr uint32_t kOffA = 0;                          // 2 stages x 2 atoms x 16 KB
constexpr uint32_t kOffB = 64 * 1024;                  // 4 stages x 2 planes x 2 atoms x 4 KB
constexpr uint32_t kOffAm = kOffB + 64 * 1024;         // min-term A: 2 planes x 16 KB
constexpr uint32_t kOffBm = kOffAm + 32 * 1024;        // min-term B: 2 planes x 4 KB
constexpr uint32_t kRawStage = kGM * 144;              // one superblock of 128 rows
constexpr uint32_t kOffRaw = kOffBm + 8 * 1024;        // 2 x raw superblock
constexpr uint32_t kOffHdr = kOffRaw + 2 * kRawStage;  // d per superblock and row, f32 [8][128]
constexpr uint32_t kOffMisc = kOffHdr + kGMaxSb * kGM * 4;
constexpr uint32_t kGSmem = kOffMisc + 512 + 1024;     // + misc + alignment slack

struct GemmArgs {
    const uint8_t *w;     // gate (mode 0) or down (mode 1) weights
    const uint8_t *w_up;  // mode 0: up weights; nullptr when w holds [gate; up] per expert
    uint64_t pitch;
    uint32_t K;       // columns (multiple of 256, <= 2048)
    uint32_t rows_e;  // rows per expert in w
    uint32_t F;       // mode 0: expert width
    int act;
    MoePlan p;
    const uint2 *tiles;  // (active expert slot, first position within it)
    const uint32_t *n_tiles;
    uint32_t k;  // slots per token
    const __half *xh, *xl;  // activation rows [R][K], K permuted in groups of 4
    const float *xsum;      // [R][K/32] sub-block sums of the scaled rows
    const float *xinv;      // [R] 2^e
    float *out;             // mode 0: h [P][F]; mode 1: y [P][out_ld]
    uint32_t out_ld;
    int *dev_err;
};

LT_DEVINL void cp_async16(void *dst_smem, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst_smem)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
LT_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
LT_DEVINL void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

LT_DEVINL uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
    __half2 r = __hfma2(*reinterpret_cast<__half2 *>(&a), *reinterpret_cast<__half2 *>(&b),
                        *reinterpret_cast<__half2 *>(&c));
    return *reinterpret_cast<uint32_t *>(&r);
}
LT_DEVINL uint32_t half2_splat(float v) {
    __half2 h = __float2half2_rn(v);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Two f16 planes of v: hi = f16(v), lo = f16(v - hi).
LT_DEVINL void split_f16(float v, __half &h, __half &l) {
    h = __float2half_rn(v);
    l = __float2half_rn(v - __half2float(h));
}

LT_DEVINL void gemm_wait(uint64_t *bar, uint32_t parity, int *dev_err) {
    if (!mbar_wait_bounded(bar, parity, kWaitLimitNs) && dev_err) atomicExch(dev_err, DEV_ERR_TMA_TIMEOUT);
}

template <int MODE>
__global__ void __launch_bounds__(kGThreads, 1) k_moe_gemm(GemmArgs a) {
    extern __shared__ uint8_t g_smem_raw[];
    uint8_t *sm = g_smem_raw + ((1024u - (smem_u32(g_smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_wait();
    if (blockIdx.y >= *a.n_tiles) return;
    const uint2 tile = a.tiles[blockIdx.y];
    const uint32_t slot = tile.x, n0 = tile.y;
    const uint32_t e = a.p.act_e[slot];
    const uint32_t pos0 = a.p.act_off[slot] + n0;
    const uint32_t nvalid = min((uint32_t)kGN, a.p.act_cnt[slot] - n0);
    const uint32_t m0 = blockIdx.x;
    const uint32_t nsb = a.K / 256, nks = 2 * nsb;
    const uint32_t ncols = nsb + 1 <= 4 ? 128u : nsb + 1 <= 8 ? 256u : 512u;

    uint64_t *bar_raw = reinterpret_cast<uint64_t *>(sm + kOffMisc);  // [2]
    uint64_t *bar_mma = bar_raw + 2;                                    // [2]
    uint64_t *bar_fin = bar_raw + 4;
    uint32_t *s_taddr = reinterpret_cast<uint32_t *>(bar_raw + 5);
    uint32_t *s_row = s_taddr + 1;  // [32] activation row of each tile position
    float *s_inv = reinterpret_cast<float *>(s_row + kGN);  // [32]
    float *hdr_d = reinterpret_cast<float *>(sm + kOffHdr);

    // the weight row this thread dequantises (tile row = tid)
    auto wrow_of = [&](uint32_t r) -> const uint8_t * {
        if (MODE == 0) {
            const uint32_t f = 64 * m0 + (r & 63);
            if (r < 64) return a.w + ((uint64_t)e * a.rows_e + f) * a.pitch;
            return a.w_up ? a.w_up + ((uint64_t)e * a.F + f) * a.pitch
                          : a.w + ((uint64_t)e * a.rows_e + a.F + f) * a.pitch;  // fused: up rows [F, 2F)
        }
        return a.w + ((uint64_t)e * a.rows_e + kGM * m0 + r) * a.pitch;
    };

    if (tid < kGN) {
        uint32_t row = 0xffffffffu;
        float inv = 0.0f;
        if ((uint32_t)tid < nvalid) {
            const uint32_t pos = pos0 + tid;
            row = MODE == 0 ? a.p.pos_pair[pos] / a.k : pos;
            inv = a.xinv[row];
        }
        s_row[tid] = row;
        s_inv[tid] = inv;
    }
    if (tid == 0) {
        for (int i = 0; i < 5; i++) mbar_init(&bar_raw[i], 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(s_taddr, ncols);
        tmem_relinquish();
    }
    // min-term operands: zero (K beyond 8*nsb stays zero), then B from the sums
    for (uint32_t i = tid; i < (40u * 1024) / 16; i += kGThreads)
        reinterpret_cast<uint4 *>(sm + kOffAm)[i] = make_uint4(0, 0, 0, 0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *s_taddr;

    // raw Q4_K superblocks 0 and 1 (one 144-byte bulk copy per row)
    auto issue_raw = [&](uint32_t sb) {
        if (warp != 0) return;
        uint64_t *bar = &bar_raw[sb & 1];
        if (lane == 0) mbar_arrive_expect_tx(bar, kRawStage);
        __syncwarp();
        uint8_t *dst = sm + kOffRaw + (sb & 1) * kRawStage;
        for (uint32_t r = lane; r < (uint32_t)kGM; r += 32) tma_load_1d(dst + r * 144, wrow_of(r) + 144 * sb, 144, bar);
    };
    issue_raw(0);
    if (nsb > 1) issue_raw(1);

    // activation stage ks: 32 positions x 128 columns x 2 planes, gathered by cp.async
    auto fill_b = [&](uint32_t ks) {
        uint8_t *bs = sm + kOffB + (ks & 3) * 16384;
        const uint32_t k0 = ks * 128;
        for (uint32_t i = tid; i < 2u * kGN * 16; i += kGThreads) {
            const uint32_t plane = i >> 9, rem = i & 511, n = rem >> 4, cc = rem & 15;
            const uint32_t row = s_row[n];
            const __half *src = (plane ? a.xl : a.xh) + (size_t)(row == 0xffffffffu ? 0 : row) * a.K + k0 + cc * 8;
            uint8_t *dst = bs + plane * 8192 + (cc >> 3) * 4096 + n * 128 + (((cc & 7) ^ (n & 7)) << 4);
            cp_async16(dst, src, row == 0xffffffffu ? 0u : 16u);
        }
        cp_async_commit();
    };
    fill_b(0);
    if (nks > 1) fill_b(1); else cp_async_commit();

    // min-term B: sub-block sums of each position, two planes
    for (uint32_t i = tid; i < kGN * 8 * nsb; i += kGThreads) {
        const uint32_t n = i / (8 * nsb), j = i - n * (8 * nsb);
        const uint32_t row = s_row[n];
        const float v = row == 0xffffffffu ? 0.0f : a.xsum[(size_t)row * (a.K / 32) + j];
        __half h, l;
        split_f16(v, h, l);
        *reinterpret_cast<__half *>(sm + kOffBm + sw128_offset(n, j)) = h;
        *reinterpret_cast<__half *>(sm + kOffBm + 4096 + sw128_offset(n, j)) = l;
    }

    const uint32_t idesc = umma_idesc_f16_f32(kGM, kGN);
    for (uint32_t ks = 0; ks < nks; ks++) {
        const uint32_t sb = ks >> 1, hf = ks & 1;
        if (ks >= 2) gemm_wait(&bar_mma[ks & 1], ((ks >> 1) - 1) & 1, a.dev_err);  // MMAs of stage ks-2 done
        if (ks + 2 < nks) fill_b(ks + 2); else cp_async_commit();
        if (hf == 0) gemm_wait(&bar_raw[sb & 1], (sb >> 1) & 1, a.dev_err);

        // dequantise this thread's row: pairs c = 2hf, 2hf+1 -> atoms 0, 1
        {
            const uint8_t *raw = sm + kOffRaw + (sb & 1) * kRawStage + tid * 144;
            const uint4 hdr = lds128(raw);
            // scale_min (dequant.zig:291-300) of sub-blocks 4hf .. 4hf+3
            const uint32_t scw = hf == 0 ? (hdr.y & 0x3F3F3F3Fu)
                                         : ((hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u));
            const uint32_t mnw = hf == 0 ? (hdr.z & 0x3F3F3F3Fu)
                                         : (((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u));
            if (hf == 0) hdr_d[sb * kGM + tid] = f16_bits_to_f32(hdr.x);
            const float dmin = f16_bits_to_f32(hdr.x >> 16);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float v = dmin * (float)((mnw >> (8 * j)) & 0xffu);  // exact in f32
                __half h, l;
                split_f16(v, h, l);
                const uint32_t kk = 8 * sb + 4 * hf + j;
                *reinterpret_cast<__half *>(sm + kOffAm + sw128_offset(tid, kk)) = h;
                *reinterpret_cast<__half *>(sm + kOffAm + 16384 + sw128_offset(tid, kk)) = l;
            }
            uint8_t *as = sm + kOffA + (ks & 1) * 32768 + tid * 128;
#pragma unroll
            for (int cl = 0; cl < 2; cl++) {
                const float sc0 = (float)((scw >> (16 * cl)) & 0xffu), sc1 = (float)((scw >> (16 * cl + 8)) & 0xffu);
                const uint32_t s0 = half2_splat(sc0), b0 = half2_splat(-1024.0f * sc0);
                const uint32_t s1 = half2_splat(sc1), b1 = half2_splat(-1024.0f * sc1);
                const uint4 qa = lds128(raw + 16 + 32 * (2 * hf + cl)), qb = lds128(raw + 32 + 32 * (2 * hf + cl));
                const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                uint8_t *arow = as + cl * 16384;
                const uint32_t sw = tid & 7;
#pragma unroll
                for (int m = 0; m < 4; m++) {
                    // positions 8m..8m+7 hold elements 8m + (0,2,1,3,4,6,5,7) of sub-block 2c
                    uint4 lo, hi;
                    lo.x = hfma2_u32((w[2 * m] & 0x000F000Fu) | 0x64006400u, s0, b0);
                    lo.y = hfma2_u32(((w[2 * m] >> 8) & 0x000F000Fu) | 0x64006400u, s0, b0);
                    lo.z = hfma2_u32((w[2 * m + 1] & 0x000F000Fu) | 0x64006400u, s0, b0);
                    lo.w = hfma2_u32(((w[2 * m + 1] >> 8) & 0x000F000Fu) | 0x64006400u, s0, b0);
                    hi.x = hfma2_u32(((w[2 * m] >> 4) & 0x000F000Fu) | 0x64006400u, s1, b1);
                    hi.y = hfma2_u32(((w[2 * m] >> 12) & 0x000F000Fu) | 0x64006400u, s1, b1);
                    hi.z = hfma2_u32(((w[2 * m + 1] >> 4) & 0x000F000Fu) | 0x64006400u, s1, b1);
                    hi.w = hfma2_u32(((w[2 * m + 1] >> 12) & 0x000F000Fu) | 0x64006400u, s1, b1);
                    *reinterpret_cast<uint4 *>(arow + ((m ^ sw) << 4)) = lo;
                    *reinterpret_cast<uint4 *>(arow + (((4 + m) ^ sw) << 4)) = hi;
                }
            }
        }
        if (hf == 1 && sb + 2 < nsb) {  // raw slot sb&1 is consumed: fetch superblock sb+2 into it
            __syncthreads();
            issue_raw(sb + 2);
        }
        cp_async_wait<2>();  // this thread's copies of stage ks have landed
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t abase = smem_u32(sm + kOffA + (ks & 1) * 32768);
            const uint32_t bbase = smem_u32(sm + kOffB + (ks & 3) * 16384);
            const uint32_t d_tmem = taddr + sb * kGN;
#pragma unroll
            for (uint32_t s = 0; s < 8; s++) {
                const uint32_t ao = abase + (s >> 2) * 16384 + (s & 3) * 32;
                const uint32_t bo = bbase + (s >> 2) * 4096 + (s & 3) * 32;
                umma_f16(d_tmem, umma_desc_sw128(ao), umma_desc_sw128(bo), idesc, (hf | s) != 0);
                umma_f16(d_tmem, umma_desc_sw128(ao), umma_desc_sw128(bo + 8192), idesc, 1);
            }
            umma_commit(&bar_mma[ks & 1]);
        }
    }
    // min term into the last accumulator: hi*hi + hi*lo + lo*hi over K = 8*nsb
    if (tid == 0) {
        const uint32_t am = smem_u32(sm + kOffAm), bm = smem_u32(sm + kOffBm);
        const uint32_t d_tmem = taddr + nsb * kGN;
        const uint32_t nkm = (8 * nsb + 15) / 16;
        for (uint32_t s = 0; s < nkm; s++) {
            umma_f16(d_tmem, umma_desc_sw128(am + s * 32), umma_desc_sw128(bm + s * 32), idesc, s != 0);
            umma_f16(d_tmem, umma_desc_sw128(am + s * 32), umma_desc_sw128(bm + 4096 + s * 32), idesc, 1);
            umma_f16(d_tmem, umma_desc_sw128(am + 16384 + s * 32), umma_desc_sw128(bm + s * 32), idesc, 1);
        }
        umma_commit(bar_fin);
    }
    gemm_wait(bar_fin, 0, a.dev_err);
    tc_fence_after();

    // epilogue: thread tid owns tile row tid (TMEM lane), all 32 positions
    const uint32_t lane_addr = taddr + ((uint32_t)(32 * warp) << 16);
    float y[kGN];
#pragma unroll
    for (int n = 0; n < kGN; n++) y[n] = 0.0f;
    for (uint32_t sb = 0; sb < nsb; sb++) {
        uint32_t v[32];
        tmem_ld32(lane_addr + sb * kGN, v);
        tmem_wait_ld();
        const float dsb = hdr_d[sb * kGM + tid];
#pragma unroll
        for (int n = 0; n < kGN; n++) y[n] = fmaf(dsb, __uint_as_float(v[n]), y[n]);
    }
    {
        uint32_t v[32];
        tmem_ld32(lane_addr + nsb * kGN, v);
        tmem_wait_ld();
#pragma unroll
        for (int n = 0; n < kGN; n++) y[n] = (y[n] - __uint_as_float(v[n])) * s_inv[n];
    }
    tc_fence_before();
    if (MODE == 1) {
        const uint32_t r = kGM * m0 + tid;
#pragma unroll
        for (uint32_t n = 0; n < (uint32_t)kGN; n++)
            if (n < nvalid) a.out[(size_t)(pos0 + n) * a.out_ld + r] = y[n];
    } else {
        float *uex = reinterpret_cast<float *>(sm + kOffA);  // [64][33]; the A stages are free now
        if (tid >= 64)
#pragma unroll
            for (int n = 0; n < kGN; n++) uex[(tid - 64) * 33 + n] = y[n];
        __syncthreads();
        if (tid < 64) {
            const uint32_t f = 64 * m0 + tid;
#pragma unroll
            for (uint32_t n = 0; n < (uint32_t)kGN; n++)
                if (n < nvalid) a.out[(size_t)(pos0 + n) * a.F + f] = act_apply(a.act, y[n]) * uex[tid * 33 + n];
        }
    }
    __syncthreads();
    if (warp == 0) tmem_dealloc(taddr, ncols);
}

// ── activation prep: f32 rows -> f16 hi/lo planes (K permuted in groups of 4
// as the dequantised weights are), sub-block sums, 2^e per row ─────────────
__global__ void __launch_bounds__(256) k_gemm_prep(const float *src, uint32_t K, __half *xh, __half *xl, float *xsum,
                                                   float *xinv) {
    __shared__ float s_red[8];
    pdl_wait();
    const uint32_t row = blockIdx.x;
    const float *s = src + (size_t)row * K;
    float amax = 0.0f;
    for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) amax = fmaxf(amax, fabsf(s[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x < 32) {
        float m = threadIdx.x < blockDim.x / 32 ? s_red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (threadIdx.x == 0) s_red[0] = m;
    }
    __syncthreads();
    int ex = 0;
    frexpf(s_red[0], &ex);  // max|x| * 2^-ex in [0.5, 1)
    const float scale = ldexpf(1.0f, -ex);
    for (uint32_t m = threadIdx.x; m < K / 8; m += blockDim.x) {
        const float4 p = *reinterpret_cast<const float4 *>(s + 8 * m);
        const float4 q = *reinterpret_cast<const float4 *>(s + 8 * m + 4);
        const float v[8] = {p.x, p.z, p.y, p.w, q.x, q.z, q.y, q.w};  // positions <- elements (0,2,1,3,...)
        __align__(16) __half h[8], l[8];
#pragma unroll
        for (int i = 0; i < 8; i++) split_f16(v[i] * scale, h[i], l[i]);
        *reinterpret_cast<uint4 *>(xh + (size_t)row * K + 8 * m) = *reinterpret_cast<uint4 *>(h);
        *reinterpret_cast<uint4 *>(xl + (size_t)row * K + 8 * m) = *reinterpret_cast<uint4 *>(l);
    }
    for (uint32_t j = threadIdx.x; j < K / 32; j += blockDim.x) {
        float t = 0.0f;
        for (int i = 0; i < 32; i++) t += s[32 * j + i] * scale;
        xsum[(size_t)row * (K / 32) + j] = t;
    }
    if (threadIdx.x == 0) xinv[row] = ldexpf(1.0f, ex);
}

// ── tile list: (active expert slot, first position) per 32 positions ───────
__global__ void k_gemm_tiles(MoePlan p, uint2 *tiles, uint32_t *n_tiles) {
    pdl_wait();
    if (threadIdx.x != 0) return;
    uint32_t n = 0;
    const uint32_t na = *p.n_active;
    for (uint32_t s = 0; s < na; s++)
        for (uint32_t n0 = 0; n0 < p.act_cnt[s]; n0 += kGN) tiles[n++] = make_uint2(s, n0);
    *n_tiles = n;
}

// ── weighted combine in slot order (+ residual) ─────────────────────────────
__global__ void k_gemm_combine(const float *y, uint32_t D, const uint32_t *pair_pos, const float *w, uint32_t k,
                               const float *resid, float *out) {
    pdl_wait();
    const uint32_t t = blockIdx.y, c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= D) return;
    float o = 0.0f;  // moe_buf is zeroed, then += scale * down, slot by slot
    for (uint32_t s = 0; s < k; s++) o += w[(size_t)t * k + s] * y[(size_t)pair_pos[(size_t)t * k + s] * D + c];
    const size_t oi = (size_t)t * D + c;
    out[oi] = resid ? resid[oi] + o : o;
}

bool moe_gemm_supported(const DevMat &gate, const DevMat &down, uint64_t F) {
    return gate.type == T_Q4_K && down.type == T_Q4_K && gate.cols % 256 == 0 && F % 256 == 0 &&
           gate.cols <= 256u * kGMaxSb && F <= 256u * kGMaxSb && down.rows % kGM == 0;
}

size_t moe_gemm_scratch(uint32_t T, uint32_t k, uint32_t E, uint64_t d, uint64_t F) {
    const size_t P = (size_t)T * k;
    auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t max_tiles = (E < P ? E : P) + P / kGN + 1;
    return al(max_tiles * 8) + al(4) + 2 * al((size_t)T * d * 2) + al((size_t)T * d / 8) + al((size_t)T * 4) +
           al(P * F * 4) + 2 * al(P * F * 2) + al(P * F / 8) + al(P * 4) + al(P * d * 4);
}

cudaError_t launch_moe_gemm_ffn(const LaunchCfg &c, const DevMat &gate, const uint8_t *up, const DevMat &down, int act,
                                const float *x, uint32_t T, uint32_t k, const float *w, const MoePlan &p,
                                const float *resid, float *out, uint8_t *scratch) {
    const uint32_t E = gate.n_experts;
    const uint64_t d = gate.cols, F = down.cols;
    const size_t P = (size_t)T * k;
    const size_t max_tiles = (E < P ? E : P) + P / kGN + 1;
    size_t off = 0;
    auto take = [&](size_t b) {
        uint8_t *q = scratch + off;
        off += (b + 255) & ~(size_t)255;
        return q;
    };
    uint2 *tiles = reinterpret_cast<uint2 *>(take(max_tiles * 8));
    uint32_t *n_tiles = reinterpret_cast<uint32_t *>(take(4));
    __half *xh = reinterpret_cast<__half *>(take((size_t)T * d * 2));
    __half *xl = reinterpret_cast<__half *>(take((size_t)T * d * 2));
    float *xsum = reinterpret_cast<float *>(take((size_t)T * d / 8));
    float *xinv = reinterpret_cast<float *>(take((size_t)T * 4));
    float *hbuf = reinterpret_cast<float *>(take(P * F * 4));
    __half *hh = reinterpret_cast<__half *>(take(P * F * 2));
    __half *hl = reinterpret_cast<__half *>(take(P * F * 2));
    float *hsum = reinterpret_cast<float *>(take(P * F / 8));
    float *hinv = reinterpret_cast<float *>(take(P * 4));
    float *ybuf = reinterpret_cast<float *>(take(P * d * 4));

    cudaError_t e = launch_k(c, "moe_gemm_tiles", k_gemm_tiles, dim3(1), dim3(32), 0, p, tiles, n_tiles);
    if (e == cudaSuccess)
        e = launch_k(c, "moe_gemm_prep", k_gemm_prep, dim3(T), dim3(256), 0, x, (uint32_t)d, xh, xl, xsum, xinv);
    GemmArgs g;
    g.w = gate.data;
    g.w_up = up;
    g.pitch = gate.pitch;
    g.K = (uint32_t)d;
    g.rows_e = (uint32_t)gate.rows;
    g.F = (uint32_t)F;
    g.act = act;
    g.p = p;
    g.tiles = tiles;
    g.n_tiles = n_tiles;
    g.k = k;
    g.xh = xh;
    g.xl = xl;
    g.xsum = xsum;
    g.xinv = xinv;
    g.out = hbuf;
    g.out_ld = (uint32_t)F;
    g.dev_err = c.dev_err;
    if (e == cudaSuccess)
        e = launch_k(c, "moe_gemm_gate_up", k_moe_gemm<0>, dim3((uint32_t)(F / 64), (uint32_t)max_tiles),
                     dim3(kGThreads), (size_t)kGSmem, g);
    if (e == cudaSuccess)
        e = launch_k(c, "moe_gemm_prep", k_gemm_prep, dim3((uint32_t)P), dim3(256), 0, (const float *)hbuf,
                     (uint32_t)F, hh, hl, hsum, hinv);
    GemmArgs gd = g;
    gd.w = down.data;
    gd.w_up = nullptr;
    gd.pitch = down.pitch;
    gd.K = (uint32_t)F;
    gd.rows_e = (uint32_t)down.rows;
    gd.xh = hh;
    gd.xl = hl;
    gd.xsum = hsum;
    gd.xinv = hinv;
    gd.out = ybuf;
    gd.out_ld = (uint32_t)d;
    if (e == cudaSuccess)
        e = launch_k(c, "moe_gemm_down", k_moe_gemm<1>, dim3((uint32_t)(d / kGM), (uint32_t)max_tiles),
                     dim3(kGThreads), (size_t)kGSmem, gd);
    if (e == cudaSuccess)
        e = launch_k(c, "moe_gemm_combine", k_gemm_combine, dim3((uint32_t)((d + 255) / 256), T), dim3(256), 0,
                     (const float *)ybuf, (uint32_t)d, (const uint32_t *)p.pair_pos, w, k, resid, out);
    return e;
}

}  // namespace lt
