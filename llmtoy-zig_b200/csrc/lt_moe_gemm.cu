// lt_moe_gemm.cu — grouped expert GEMM on the 5th-generation tensor cores
// (tcgen05) for multi-token MoE batches with Q4_K, Q6_K or Q8_0 experts
// (prefill; the reference's expert loop src/model/gemma4/forward.zig:463-479
// and src/ops/moe.zig:61-76 run over many tokens).  Q4_K up to 2048 columns
// takes the single-plane scheme described next; Q6_K, Q8_0 and wider Q4_K
// take the stacked-plane scheme (see StkFmt below).
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
// Work item: 128 weight rows x 32 positions.  For gate/up the rows are 64
// gate rows and the same 64 up rows, so the epilogue forms h = act(g)*u.
// Per stage (half a superblock, K = 128) four warps dequantise one weight row
// per thread from raw Q4_K rows that a producer warp streams in by TMA bulk
// copies; another warp gathers the activation rows of the item's positions
// with cp.async; one lane issues the MMAs.  Each superblock accumulates in
// one of two TMEM buffers, which the dequantising warps fold into registers
// (y += d * acc) while the next superblock runs.
#include <cuda.h>  // CUtensorMap (encoded through the runtime's driver entry point)
#include <cuda_fp16.h>

#include <cstring>
#include <mutex>

#include "lt_launch.cuh"
#include "lt_umma.cuh"

namespace lt {

constexpr int kGN = 32;     // positions per tile of the small-batch shape (MMA N = 64)
constexpr int kGM = 128;    // weight rows per tile (MMA M)
constexpr int kGMaxSb = 8;  // superblocks per row (K <= 2048)

// Roles (warps): 0-7 dequantise weight rows into the A stages and run the
// epilogue (two threads per tile row: one per 64-column pair of the stage;
// row = TMEM lane); 8 streams raw Q4_K superblocks (tiled TMA; stacked
// planes: every lane copies row windows by cp.async); 9 gathers
// the activation stages (cp.async, one position per lane) and the min-term
// operand; 10 issues the MMAs (one lane).  The CTA is persistent: it walks the
// (tile, 128-row block) work items of the launch with stride gridDim.x, and
// every ring keeps running across items.
//
// The activation operand stacks the two planes: rows 0-(NP-1) of B are the hi
// plane of the NP positions, rows NP-(2NP-1) the lo plane, so one N = 2 NP MMA
// per K step covers both and the accumulator's column halves are added.  NP
// is 32 for small per-expert batches and 64 for large ones: one
// tcgen05.mma takes about as long at N = 128 as at N = 64, so the wider tile
// halves the MMA issue and the dequantisation per FLOP.
constexpr int kGMath = 256;
constexpr int kGWarpRaw = 8, kGWarpB = 9, kGWarpMma = 10;
constexpr int kGThreadsV2 = 11 * 32;
constexpr int kGAStages = 2;   // dequantised A stages (K = 128 each)
constexpr uint32_t kRawStage = kGM * 144;  // one superblock of 128 rows

// Per tile width NP: MMA N, rings, TMEM columns (2 x 2NP superblock
// accumulators + 2NP min-term columns) and the shared-memory map (offsets
// from a 1024-byte aligned base).
template <int NP>
struct GemmGeo {
    static constexpr int NNP = 2 * NP;                      // MMA N: hi and lo planes
    static constexpr int kBStages = NP == 32 ? 3 : 2;       // activation stages
    static constexpr int kRawSlots = NP == 32 ? 3 : 2;      // raw superblocks in flight
    static constexpr uint32_t kBAtom = NNP * 128;           // NNP rows x 64 K (f16)
    static constexpr uint32_t kBStage = 2 * kBAtom;         // K = 128
    static constexpr uint32_t kTmemCols = NP == 32 ? 256 : 512;
    static constexpr uint32_t kOffA = 0;                                  // kGAStages x 2 atoms x 16 KB
    static constexpr uint32_t kOffB = kOffA + kGAStages * 32768;
    static constexpr uint32_t kOffAm = kOffB + kBStages * kBStage;        // min-term A: 2 planes x 16 KB
    static constexpr uint32_t kOffBm = kOffAm + 32768;                    // min-term B: one NNP-row atom
    static constexpr uint32_t kOffRaw = kOffBm + kBAtom;
    static constexpr uint32_t kOffHdr = kOffRaw + kRawSlots * kRawStage;  // d [8][128] f32
    static constexpr uint32_t kOffMisc = kOffHdr + kGMaxSb * kGM * 4;     // barriers, TMEM address, scales
    static constexpr uint32_t kSmem = kOffMisc + 1024 + 1024;             // + alignment slack
};
static_assert(GemmGeo<64>::kSmem <= 227 * 1024, "NP = 64 shared memory");
static_assert(GemmGeo<32>::kSmem <= 227 * 1024, "NP = 32 shared memory");

struct GemmArgs {
    // 2-D byte views [rows][pitch] of the weights for tiled TMA: one load
    // moves a 64-row x 144-byte box (one Q4_K superblock column)
    alignas(64) CUtensorMap map_w;
    alignas(64) CUtensorMap map_up;
    // the activation planes [P][K] (f16, 128B swizzle, box 64 x NP), rows in
    // dispatch-position order: an item's positions are consecutive rows, so
    // the B warp loads each stage with four tiled TMA copies
    alignas(64) CUtensorMap map_bh;
    alignas(64) CUtensorMap map_bl;
    const uint8_t *w;     // gate (mode 0) or down (mode 1) weights
    const uint8_t *w_up;  // mode 0: up weights; nullptr when w holds [gate; up] per expert
    const uint8_t *w_end, *up_end;  // one past the last byte of w / w_up
    uint64_t pitch;
    uint32_t K;       // columns (Q4_K single plane: multiple of 256, <= 2048; stacked planes: <= 4096)
    uint32_t rows_e;  // rows per expert in w
    uint32_t F;       // mode 0: expert width
    uint32_t mt;      // row blocks per tile (128 rows; 64 with stacked planes)
    int act;
    MoePlan p;
    const uint2 *tiles;  // (active expert slot, first position within it)
    const uint32_t *n_tiles;
    uint32_t k;  // slots per token
    const __half *xh, *xl;  // activation planes [P][K] by position, K permuted in groups of 4 (read through the maps)
    const float *xsum;      // [P][K/32] sub-block sums of the scaled rows
    const float *xinv;      // [P] 2^e
    float *out;             // mode 0: h [P][F]; mode 1: y [P][out_ld]
    uint32_t out_ld;
    int *dev_err;
};

LT_DEVINL void cp_async16(void *dst_smem, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst_smem)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
// Arrive on an mbarrier once this thread's earlier cp.async copies land
// (the arrival counts against the barrier's expected count).
LT_DEVINL void cp_async_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
LT_DEVINL void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 2-D tiled TMA load of box (x, y) of a tensor map held in kernel parameters.
LT_DEVINL void tma_load_2d(void *dst_smem, const CUtensorMap *map, uint32_t x, uint32_t y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst_smem)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 16 consecutive 32-bit TMEM columns of this thread's lane.
LT_DEVINL void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

// Barrier among the eight dequantising warps only.
LT_DEVINL void math_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

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

// Wait for completion number n (0, 1, ...) of a barrier.
LT_DEVINL void gemm_wait(uint64_t *bar, uint32_t n, int *dev_err) {
    if (!mbar_wait_bounded(bar, n & 1, kWaitLimitNs) && dev_err) atomicExch(dev_err, DEV_ERR_TMA_TIMEOUT);
}

struct GemmItem {
    uint32_t e, pos0, nvalid, m0;
};

template <int NP>
LT_DEVINL GemmItem gemm_item(const GemmArgs &a, uint32_t w) {
    const uint2 tile = a.tiles[w / a.mt];
    GemmItem it;
    it.m0 = w % a.mt;
    it.e = a.p.act_e[tile.x];
    it.pos0 = a.p.act_off[tile.x] + tile.y;
    it.nvalid = min((uint32_t)NP, a.p.act_cnt[tile.x] - tile.y);
    return it;
}

// ── stacked-plane weights (Q6_K, Q8_0, and Q4_K wider than 2048 columns) ──
// The scheme above needs sc*q to be a small integer and one scale per
// superblock; Q6_K's sc*(q-32) reaches 4096 (not exact in f16) and Q8_0 has
// a scale per 32 columns.  For these an item covers 64 weight rows and the
// tile's 128 MMA rows hold each of them twice: rows 0-63 the high f16 plane
// of the row's values, rows 64-127 the low plane.  A value is the
// reference's own f32 dequantisation (dequantRow: the same products and
// roundings), times 2^-E for a power of two chosen per row and superblock
// from the block header (|v| 2^-E < 2^15), split hi = f16(v'), lo =
// f16(v' - hi) (22 significant bits; the scaling keeps both normal).  Each
// superblock still accumulates in its own TMEM buffer and the fold applies
// 2^E; the two planes' lanes add up in the epilogue.  No minimum term.
//
// Raw rows need not be 16-byte aligned (a Q6_K superblock is 210 bytes, a
// Q8_0 row 34 bytes per 32 columns), so the producer warp copies each row's
// superblock window with 16-byte cp.async from the aligned address below it
// into a slot of kSlot bytes, and the dequantising threads read from the
// window's offset inside the slot.
template <int WS>
struct StkFmt;
template <>
struct StkFmt<T_Q4_K> {
    static constexpr uint32_t kSbBytes = 144, kSlot = 160;
};
template <>
struct StkFmt<T_Q6_K> {
    static constexpr uint32_t kSbBytes = 210, kSlot = 224;
};
template <>
struct StkFmt<T_Q8_0> {
    static constexpr uint32_t kSbBytes = 272, kSlot = 288;  // eight 34-byte blocks
};
constexpr int kStkRows = 64;
constexpr int kStkMaxSb = 16;  // K <= 4096

// Bytes of superblock sb of a row (a Q8_0 row may end inside its last 256 columns).
template <int WS>
LT_DEVINL uint32_t stk_len(uint32_t K, uint32_t sb) {
    if constexpr (WS == T_Q8_0) return 34u * min(8u, K / 32 - 8 * sb);
    return StkFmt<WS>::kSbBytes;
}

// First byte of weight row wr (0-63) of an item, and the end of its tensor.
template <int MODE>
LT_DEVINL const uint8_t *stk_row(const GemmArgs &a, const GemmItem &it, uint32_t wr, const uint8_t *&end) {
    if (MODE == 1) {
        end = a.w_end;
        return a.w + (size_t)(it.e * a.rows_e + kStkRows * it.m0 + wr) * a.pitch;
    }
    if (wr < 32) {  // gate rows, then the same 32 up rows
        end = a.w_end;
        return a.w + (size_t)(it.e * a.rows_e + 32 * it.m0 + wr) * a.pitch;
    }
    const uint32_t u = 32 * it.m0 + wr - 32;
    if (a.w_up) {
        end = a.up_end;
        return a.w_up + (size_t)(it.e * a.F + u) * a.pitch;
    }
    end = a.w_end;
    return a.w + (size_t)(it.e * a.rows_e + a.F + u) * a.pitch;
}

LT_DEVINL uint32_t lds16(const uint8_t *p) { return *reinterpret_cast<const unsigned short *>(p); }

// N little-endian words from a 2-byte aligned shared address (aligned loads,
// one PRMT each).
template <int N>
LT_DEVINL void lds_words_a2(const uint8_t *p, uint32_t (&w)[N]) {
    const uint32_t mis = smem_u32(p) & 3u;  // 0 or 2
    const uint8_t *pa = p - mis;
    const uint32_t sel = mis ? 0x5432u : 0x3210u;
    uint32_t prev = lds32(pa);
#pragma unroll
    for (int i = 0; i < N; i++) {
        const uint32_t nx = lds32(pa + 4 * (i + 1));
        w[i] = __byte_perm(prev, nx, sel);
        prev = nx;
    }
}

// 2^E for superblock sb of a row: |every value| * 2^-E < 2^15.
template <int WS>
LT_DEVINL float stk_exp2(const uint8_t *sbp, uint32_t K, uint32_t sb) {
    float bound;
    if constexpr (WS == T_Q4_K) {
        const uint32_t h = lds16(sbp) | (lds16(sbp + 2) << 16);
        bound = fabsf(f16_bits_to_f32(h & 0xffffu)) * 945.0f + fabsf(f16_bits_to_f32(h >> 16)) * 63.0f;
    } else if constexpr (WS == T_Q6_K) {
        bound = fabsf(f16_bits_to_f32(lds16(sbp + 208))) * 4096.0f;
    } else {
        const uint32_t nb = min(8u, K / 32 - 8 * sb);
        float m = 0.0f;
        for (uint32_t b = 0; b < nb; b++) m = fmaxf(m, fabsf(f16_bits_to_f32(lds16(sbp + 34 * b))));
        bound = m * 128.0f;
    }
    if (!(bound > 0.0f)) return 1.0f;
    const int e = (int)((__float_as_uint(bound) >> 23) & 0xffu) - 127 - 14;  // bound < 2^(e + 15)
    return __uint_as_float((uint32_t)(127 + e) << 23);
}

// Element order inside each 8-column chunk of an A row, (0,2,1,3,4,6,5,7):
// the activation rows are permuted the same way by k_gemm_prep.
constexpr int chunk_perm(int i) { return (i & 4) | ((i & 1) << 1) | ((i >> 1) & 1); }

// One plane (pl: 0 hi, 1 lo) of 64 columns (64-column chunk c of superblock
// sbp, 2-byte aligned in shared memory) scaled by sv = 2^-E, written as eight
// 16-byte 128B-swizzled chunks of the A row at arow.
template <int WS>
LT_DEVINL void stk_dequant(const uint8_t *sbp, uint32_t c, float sv, uint32_t pl, uint8_t *arow, uint32_t swz) {
    float v[64];
    if constexpr (WS == T_Q4_K) {
        // dequant.zig:157-187: d1 * q - m1 with d1 = d*sc, m1 = dmin*m (sub-blocks 2c, 2c+1)
        const uint32_t h = lds16(sbp) | (lds16(sbp + 2) << 16);
        const float d = f16_bits_to_f32(h & 0xffffu), dmin = f16_bits_to_f32(h >> 16);
        uint32_t s[3], q[8];
        lds_words_a2<3>(sbp + 4, s);
        lds_words_a2<8>(sbp + 16 + 32 * c, q);
        float d1[2], m1[2];
#pragma unroll
        for (int t = 0; t < 2; t++) {
            const uint32_t j = 2 * c + t;  // get_scale_min_k4 (dequant.zig:291-300)
            uint32_t sc, mn;
            if (j < 4) {
                sc = (s[0] >> (8 * j)) & 63u;
                mn = (s[1] >> (8 * j)) & 63u;
            } else {
                const uint32_t b = 8 * (j - 4);
                sc = ((s[2] >> b) & 15u) | (((s[0] >> b) >> 6 & 3u) << 4);
                mn = ((s[2] >> b) >> 4 & 15u) | (((s[1] >> b) >> 6 & 3u) << 4);
            }
            d1[t] = __fmul_rn(__fmul_rn(d, (float)sc), sv);
            m1[t] = __fmul_rn(__fmul_rn(dmin, (float)mn), sv);
        }
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const uint32_t byte = (q[i >> 2] >> (8 * (i & 3))) & 0xffu;
            v[i] = __fsub_rn(__fmul_rn(d1[0], (float)(byte & 15u)), m1[0]);
            v[32 + i] = __fsub_rn(__fmul_rn(d1[1], (float)(byte >> 4)), m1[1]);
        }
    } else if constexpr (WS == T_Q6_K) {
        // dequant.zig:237-287: (d*sc) * (q - 32); this thread's columns are
        // half n = c >> 1 of the superblock, kinds 2(c&1) and 2(c&1)+1
        const uint32_t n = c >> 1, hk = c & 1;
        const float d = f16_bits_to_f32(lds16(sbp + 208));
        uint32_t ql[16], qh[8], scw[1];
        lds_words_a2<16>(sbp + 64 * n, ql);
        lds_words_a2<8>(sbp + 128 + 32 * n, qh);
        lds_words_a2<1>(sbp + 192 + 8 * n + 4 * hk, scw);
#pragma unroll
        for (int kk = 0; kk < 2; kk++) {  // kind 2hk + kk
#pragma unroll
            for (int l = 0; l < 32; l++) {
                const uint32_t qlb = (ql[8 * kk + (l >> 2)] >> (8 * (l & 3))) & 0xffu;
                const uint32_t qhb = (qh[l >> 2] >> (8 * (l & 3))) & 0xffu;
                const uint32_t lo4 = hk ? qlb >> 4 : qlb & 15u;
                const uint32_t hi2 = (qhb >> (4 * hk + 2 * kk)) & 3u;
                const int sc = (int)(int8_t)((scw[0] >> (8 * (2 * kk + (l >> 4)))) & 0xffu);
                const float s = __fmul_rn(__fmul_rn(d, (float)sc), sv);
                v[32 * kk + l] = __fmul_rn(s, (float)((int)(lo4 | (hi2 << 4)) - 32));
            }
        }
    } else {
        // dequant.zig:42-52: d * q, blocks 2c and 2c+1 of the superblock
#pragma unroll
        for (int bb = 0; bb < 2; bb++) {
            const uint8_t *blk = sbp + 34 * (2 * c + bb);
            const float ds = __fmul_rn(f16_bits_to_f32(lds16(blk)), sv);
            uint32_t q[8];
            lds_words_a2<8>(blk + 2, q);
#pragma unroll
            for (int i = 0; i < 32; i++)
                v[32 * bb + i] = __fmul_rn(ds, (float)(int)(int8_t)((q[i >> 2] >> (8 * (i & 3))) & 0xffu));
        }
    }
#pragma unroll
    for (int m = 0; m < 8; m++) {
        uint32_t pk[4];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            float p2[2];
#pragma unroll
            for (int t = 0; t < 2; t++) {
                const float x = v[8 * m + chunk_perm(i + t)];
                const float hi = __half2float(__float2half_rn(x));
                p2[t] = pl ? x - hi : x;
            }
            const __half2 h2 = __floats2half2_rn(p2[0], p2[1]);
            pk[i >> 1] = *reinterpret_cast<const uint32_t *>(&h2);
        }
        *reinterpret_cast<uint4 *>(arow + ((m ^ swz) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
}

// WS: 0 for Q4_K in one exact plane with the minimum term; T_Q4_K, T_Q6_K or
// T_Q8_0 for stacked planes.
template <int MODE, int NP, int WS>
__global__ void __launch_bounds__(kGThreadsV2, 1) k_moe_gemm(const __grid_constant__ GemmArgs a) {
    using Geo = GemmGeo<NP>;
    constexpr bool kStk = WS != 0;
    constexpr int NNP = Geo::NNP, kGBStages = Geo::kBStages, kGRawSlots = Geo::kRawSlots;
    constexpr uint32_t kOffA = Geo::kOffA, kOffB = Geo::kOffB, kOffAm = Geo::kOffAm, kOffBm = Geo::kOffBm;
    constexpr uint32_t kOffRaw = Geo::kOffRaw, kOffHdr = Geo::kOffHdr, kOffMisc = Geo::kOffMisc;
    constexpr int PH = NP / 2;  // positions per epilogue thread
    extern __shared__ uint8_t g_smem_raw[];
    uint8_t *sm = g_smem_raw + ((1024u - (smem_u32(g_smem_raw) & 1023u)) & 1023u);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kOffMisc);
    uint64_t *raw_full = bars, *raw_empty = bars + 3;        // [3]
    uint64_t *a_full = bars + 6, *a_empty = bars + 8;        // [2]
    uint64_t *b_full = bars + 10, *b_empty = bars + 13;      // [3]
    uint64_t *acc_full = bars + 16, *acc_empty = bars + 18;  // [2]
    uint64_t *min_full = bars + 20, *min_empty = bars + 21, *bm_full = bars + 22;
    uint32_t *s_taddr = reinterpret_cast<uint32_t *>(bars + 23);
    float *s_inv = reinterpret_cast<float *>(s_taddr + 4);  // [2][NP] by item parity
    float *hdr_d = reinterpret_cast<float *>(sm + kOffHdr);

    const uint32_t nsb = (a.K + 255) / 256;  // stacked Q8_0: the last superblock may be partial
    if (tid == 0) {
        for (int i = 0; i < 3; i++) {
            mbar_init(&raw_full[i], kStk ? 32 : 1);  // stacked: one cp.async arrival per producer lane
            mbar_init(&raw_empty[i], kGMath);
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&a_full[i], kGMath);
            mbar_init(&a_empty[i], 1);
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kGMath);
        }
        mbar_init(min_full, 1);
        mbar_init(min_empty, kGMath);
        mbar_init(bm_full, 32);
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(s_taddr, Geo::kTmemCols);
        tmem_relinquish();
    }
    // min-term operands stay zero beyond K = 8*nsb
    for (uint32_t i = tid; i < (32768u + Geo::kBAtom) / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(sm + kOffAm)[i] = make_uint4(0, 0, 0, 0);
    pdl_wait();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *s_taddr;
    const uint32_t n_work = *a.n_tiles * a.mt;

    if (warp == kGWarpRaw && kStk) {
        // ── stacked planes: each row's superblock window by 16-byte cp.async,
        //    from the aligned address below it (clamped to the tensor's end) ──
        if constexpr (kStk) {
            constexpr uint32_t kSlot = StkFmt<WS>::kSlot, kCh = kSlot / 16;
            uint32_t gsb = 0;
            for (uint32_t w = blockIdx.x; w < n_work; w += gridDim.x) {
                const GemmItem it = gemm_item<NP>(a, w);
                for (uint32_t sb = 0; sb < nsb; sb++, gsb++) {
                    const uint32_t slot = gsb % kGRawSlots;
                    if (gsb >= (uint32_t)kGRawSlots) gemm_wait(&raw_empty[slot], gsb / kGRawSlots - 1, a.dev_err);
                    uint8_t *dst = sm + kOffRaw + slot * kRawStage;
                    const uint32_t len = stk_len<WS>(a.K, sb);
                    for (uint32_t idx = lane; idx < kStkRows * kCh; idx += 32) {
                        const uint32_t row = idx / kCh, ch = idx % kCh;
                        const uint8_t *end;
                        const uint8_t *src = stk_row<MODE>(a, it, row, end) + (size_t)StkFmt<WS>::kSbBytes * sb;
                        const uint32_t off = (uint32_t)(reinterpret_cast<uintptr_t>(src) & 15u);
                        if (16 * ch >= off + len) continue;
                        const uint8_t *cp = src - off + 16 * ch;
                        const uint32_t nb = (uint32_t)min((uintptr_t)16, (uintptr_t)(end - cp));
                        cp_async16(dst + row * kSlot + 16 * ch, cp, nb);
                    }
                    cp_async_arrive(&raw_full[slot]);
                }
            }
        }
    } else if (warp == kGWarpRaw) {
        // ── raw Q4_K superblocks: two 64-row x 144-byte tiled loads ──
        if (lane == 0) {
            uint32_t gsb = 0;
            for (uint32_t w = blockIdx.x; w < n_work; w += gridDim.x) {
                const GemmItem it = gemm_item<NP>(a, w);
                uint32_t y0, y1;  // first weight row of tile rows 0-63 and 64-127
                const CUtensorMap *m1 = &a.map_w;
                if (MODE == 0) {
                    y0 = it.e * a.rows_e + 64 * it.m0;
                    if (a.w_up) {
                        y1 = it.e * a.F + 64 * it.m0;
                        m1 = &a.map_up;
                    } else {
                        y1 = y0 + a.F;  // fused: up rows [F, 2F)
                    }
                } else {
                    y0 = it.e * a.rows_e + kGM * it.m0;
                    y1 = y0 + 64;
                }
                for (uint32_t sb = 0; sb < nsb; sb++, gsb++) {
                    const uint32_t slot = gsb % kGRawSlots;
                    if (gsb >= (uint32_t)kGRawSlots) gemm_wait(&raw_empty[slot], gsb / kGRawSlots - 1, a.dev_err);
                    uint8_t *dst = sm + kOffRaw + slot * kRawStage;
                    mbar_arrive_expect_tx(&raw_full[slot], kRawStage);
                    tma_load_2d(dst, &a.map_w, 144 * sb, y0, &raw_full[slot]);
                    tma_load_2d(dst + 64 * 144, m1, 144 * sb, y1, &raw_full[slot]);
                }
            }
        }
    } else if (warp == kGWarpB) {
        // ── activation stages (lane n gathers positions n, n + 32, ...; zero
        //    past the item) and, once per item, the min-term B rows and 2^e ──
        constexpr int PPL = NP / 32;  // positions per lane
        uint32_t gs = 0, gi = 0;
        for (uint32_t w = blockIdx.x; w < n_work; w += gridDim.x, gi++) {
            const GemmItem it = gemm_item<NP>(a, w);
            uint32_t row[PPL];
            bool valid[PPL];
#pragma unroll
            for (int pp = 0; pp < PPL; pp++) {
                const uint32_t n = lane + 32 * pp;
                valid[pp] = n < it.nvalid;
                row[pp] = valid[pp] ? it.pos0 + n : 0;  // the planes are in dispatch-position order
            }
            const uint32_t nks = 2 * nsb, ks_bm = nks > 2 ? 2 : nks - 1;
            for (uint32_t ks = 0; ks < nks; ks++, gs++) {
                const uint32_t s = gs % kGBStages;
                if (gs >= (uint32_t)kGBStages) gemm_wait(&b_empty[s], gs / kGBStages - 1, a.dev_err);
                {
                    // rows past the last position read as zeros, columns past K too;
                    // rows of other experts' positions are never stored
                    if (lane == 0) {
                        uint8_t *bs = sm + kOffB + s * Geo::kBStage;
                        mbar_arrive_expect_tx(&b_full[s], Geo::kBStage);
#pragma unroll
                        for (uint32_t at = 0; at < 2; at++) {
                            tma_load_2d(bs + at * Geo::kBAtom, &a.map_bh, ks * 128 + at * 64, it.pos0, &b_full[s]);
                            tma_load_2d(bs + at * Geo::kBAtom + NP * 128, &a.map_bl, ks * 128 + at * 64, it.pos0,
                                        &b_full[s]);
                        }
                    }
                }
                if (!kStk && ks == ks_bm) {
                    // the previous item's min term has consumed the old B rows
                    if (gi >= 1) gemm_wait(min_full, gi - 1, a.dev_err);
#pragma unroll
                    for (int pp = 0; pp < PPL; pp++) {
                        const uint32_t n = lane + 32 * pp;
                        const float inv = valid[pp] ? __ldg(a.xinv + row[pp]) : 0.0f;
                        // every sub-block sum of the row in flight at once (K <= 2048: 16 float4)
                        const float4 *xs4 = reinterpret_cast<const float4 *>(a.xsum + (size_t)row[pp] * (a.K / 32));
                        float4 v4[2 * kGMaxSb];
#pragma unroll
                        for (int u = 0; u < 2 * kGMaxSb; u++)
                            v4[u] = valid[pp] && (uint32_t)u < 2 * nsb ? __ldg(xs4 + u) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int u = 0; u < 2 * kGMaxSb; u++) {
                            if ((uint32_t)u >= 2 * nsb) break;
                            const float v[4] = {v4[u].x, v4[u].y, v4[u].z, v4[u].w};
#pragma unroll
                            for (int q = 0; q < 4; q++) {
                                __half h, l;
                                split_f16(v[q], h, l);
                                *reinterpret_cast<__half *>(sm + kOffBm + sw128_offset(n, 4 * u + q)) = h;
                                *reinterpret_cast<__half *>(sm + kOffBm + sw128_offset(NP + n, 4 * u + q)) = l;
                            }
                        }
                        s_inv[(gi & 1) * NP + n] = inv;
                    }
                    fence_async_smem();
                    mbar_arrive(bm_full);
                }
            }
        }
    } else if (warp == kGWarpMma) {
        // ── MMA issue ──
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16_f32(kGM, NNP);
            uint32_t gs = 0, gsb = 0, gi = 0;
            for (uint32_t w = blockIdx.x; w < n_work; w += gridDim.x, gi++) {
                for (uint32_t sb = 0; sb < nsb; sb++, gsb++) {
                    const uint32_t ab = gsb & 1;
                    if (gsb >= 2) gemm_wait(&acc_empty[ab], gsb / 2 - 1, a.dev_err);
                    const uint32_t d_tmem = taddr + ab * NNP;
                    for (uint32_t hf = 0; hf < 2; hf++, gs++) {
                        const uint32_t sa = gs % kGAStages, s3 = gs % kGBStages;
                        gemm_wait(&a_full[sa], gs / kGAStages, a.dev_err);
                        gemm_wait(&b_full[s3], gs / kGBStages, a.dev_err);
                        tc_fence_after();
                        const uint32_t abase = smem_u32(sm + kOffA + sa * 32768);
                        const uint32_t bbase = smem_u32(sm + kOffB + s3 * Geo::kBStage);
#pragma unroll
                        for (uint32_t st = 0; st < 8; st++) {
                            const uint32_t ao = abase + (st >> 2) * 16384 + (st & 3) * 32;
                            const uint32_t bo = bbase + (st >> 2) * Geo::kBAtom + (st & 3) * 32;
                            umma_f16(d_tmem, umma_desc_sw128(ao), umma_desc_sw128(bo), idesc, (hf | st) != 0);
                        }
                        umma_commit(&a_empty[sa]);
                        umma_commit(&b_empty[s3]);
                    }
                    umma_commit(&acc_full[ab]);
                }
                if constexpr (kStk) continue;
                // min term: A planes (hi, lo) x B rows (hi plane | lo plane) over K = 8*nsb
                gemm_wait(bm_full, gi, a.dev_err);
                if (gi >= 1) gemm_wait(min_empty, gi - 1, a.dev_err);
                tc_fence_after();
                const uint32_t am = smem_u32(sm + kOffAm), bm = smem_u32(sm + kOffBm);
                const uint32_t d_tmem = taddr + 2 * NNP;
                const uint32_t nkm = (8 * nsb + 15) / 16;
                for (uint32_t st = 0; st < nkm; st++) {
                    umma_f16(d_tmem, umma_desc_sw128(am + st * 32), umma_desc_sw128(bm + st * 32), idesc, st != 0);
                    umma_f16(d_tmem, umma_desc_sw128(am + 16384 + st * 32), umma_desc_sw128(bm + st * 32), idesc, 1);
                }
                umma_commit(min_full);
            }
        }
    } else {
        // ── dequantise (thread = tile row x column pair) and epilogue ──
        const uint32_t r = tid & 127, hh = tid >> 7;  // row, pair within the stage / position half
        const uint32_t lane_addr = taddr + ((uint32_t)(32 * (warp & 3)) << 16);
        uint32_t gs = 0, gsb = 0, gi = 0;
        float y[PH];  // positions [PH hh, PH hh + PH) of tile row r
        // PH consecutive accumulator columns of this thread's lane (hi plane at
        // column c0, lo plane at c0 + NP)
        auto tload = [&](uint32_t c0, uint32_t (&vh)[PH], uint32_t (&vl)[PH]) {
            if constexpr (PH == 16) {
                tmem_ld16(lane_addr + c0, vh);
                tmem_ld16(lane_addr + c0 + NP, vl);
            } else {
                tmem_ld32(lane_addr + c0, vh);
                tmem_ld32(lane_addr + c0 + NP, vl);
            }
            tmem_wait_ld();
        };
        // superblock accumulator n (global count) of superblock sb; stacked
        // planes pass their own factor fs = 2^E
        auto fold = [&](uint32_t n, uint32_t sb, float fs) {
            gemm_wait(&acc_full[n & 1], n / 2, a.dev_err);
            tc_fence_after();
            uint32_t vh[PH], vl[PH];
            tload((n & 1) * NNP + PH * hh, vh, vl);
            tc_fence_before();
            mbar_arrive(&acc_empty[n & 1]);
            const float dsb = kStk ? fs : hdr_d[sb * kGM + r];
#pragma unroll
            for (int q = 0; q < PH; q++)
                y[q] = fmaf(dsb, __uint_as_float(vh[q]) + __uint_as_float(vl[q]), y[q]);
        };
        if constexpr (kStk) {
            // A row r = plane r >> 6 of weight row r & 63 (TMEM lane r)
            constexpr uint32_t kSlot = StkFmt<WS>::kSlot;
            const uint32_t wr = r & 63, pl = r >> 6;
            for (uint32_t w = blockIdx.x; w < n_work; w += gridDim.x) {
                const GemmItem it = gemm_item<NP>(a, w);
                const uint8_t *end;
                const uint8_t *srow = stk_row<MODE>(a, it, wr, end);
#pragma unroll
                for (int q = 0; q < PH; q++) y[q] = 0.0f;
                float fs_prev = 1.0f;
                for (uint32_t sb = 0; sb < nsb; sb++, gsb++) {
                    const uint32_t slot = gsb % kGRawSlots;
                    gemm_wait(&raw_full[slot], gsb / kGRawSlots, a.dev_err);
                    const uint32_t off =
                        (uint32_t)((reinterpret_cast<uintptr_t>(srow) + (size_t)StkFmt<WS>::kSbBytes * sb) & 15u);
                    const uint8_t *sbp = sm + kOffRaw + slot * kRawStage + wr * kSlot + off;
                    const float fs = stk_exp2<WS>(sbp, a.K, sb);
                    const float sv = 1.0f / fs;  // a power of two: exact
                    for (uint32_t hf = 0; hf < 2; hf++, gs++) {
                        const uint32_t sa = gs % kGAStages;
                        if (gs >= (uint32_t)kGAStages) gemm_wait(&a_empty[sa], gs / kGAStages - 1, a.dev_err);
                        uint8_t *arow = sm + kOffA + sa * 32768 + hh * 16384 + r * 128;
                        if (256 * sb + 128 * hf + 64 * hh < a.K) {
                            stk_dequant<WS>(sbp, 2 * hf + hh, sv, pl, arow, r & 7);
                        } else {
#pragma unroll
                            for (int m = 0; m < 8; m++) *reinterpret_cast<uint4 *>(arow + 16 * m) = make_uint4(0, 0, 0, 0);
                        }
                        fence_async_smem();
                        mbar_arrive(&a_full[sa]);
                    }
                    mbar_arrive(&raw_empty[slot]);
                    if (sb >= 1) fold(gsb - 1, sb - 1, fs_prev);
                    fs_prev = fs;
                }
                fold(gsb - 1, nsb - 1, fs_prev);
                // activation scale 2^e of each position, then the two planes' lanes add up
                const uint32_t q0 = PH * hh;
#pragma unroll
                for (uint32_t q = 0; q < (uint32_t)PH; q++) {
                    const uint32_t n = q0 + q;
                    const uint32_t row = it.pos0 + min(n, it.nvalid - 1);
                    y[q] = n < it.nvalid ? y[q] * a.xinv[row] : 0.0f;
                }
                constexpr int UX = NP + 1;  // odd stride: no bank conflicts
                float *uex = reinterpret_cast<float *>(sm + kOffA);  // [64][UX]; the A stages are idle here
                if (pl == 1)
#pragma unroll
                    for (int q = 0; q < PH; q++) uex[wr * UX + q0 + q] = y[q];
                math_sync();
                if (pl == 0)
#pragma unroll
                    for (int q = 0; q < PH; q++) y[q] += uex[wr * UX + q0 + q];
                if (MODE == 1) {
                    if (pl == 0) {
                        const uint32_t orow = kStkRows * it.m0 + wr;
#pragma unroll
                        for (uint32_t q = 0; q < (uint32_t)PH; q++)
                            if (q0 + q < it.nvalid) a.out[(size_t)(it.pos0 + q0 + q) * a.out_ld + orow] = y[q];
                    }
                } else {
                    math_sync();
                    if (pl == 0 && wr >= 32)
#pragma unroll
                        for (int q = 0; q < PH; q++) uex[(wr - 32) * UX + q0 + q] = y[q];
                    math_sync();
                    if (pl == 0 && wr < 32) {
                        const uint32_t f = 32 * it.m0 + wr;
#pragma unroll
                        for (uint32_t q = 0; q < (uint32_t)PH; q++)
                            if (q0 + q < it.nvalid)
                                a.out[(size_t)(it.pos0 + q0 + q) * a.F + f] =
                                    act_apply(a.act, y[q]) * uex[wr * UX + q0 + q];
                    }
                }
                math_sync();  // uex read before the next item's A writes
            }
        } else
        for (uint32_t w = blockIdx.x; w < n_work; w += gridDim.x, gi++) {
            const GemmItem it = gemm_item<NP>(a, w);
#pragma unroll
            for (int q = 0; q < PH; q++) y[q] = 0.0f;
            for (uint32_t sb = 0; sb < nsb; sb++, gsb++) {
                const uint32_t slot = gsb % kGRawSlots;
                gemm_wait(&raw_full[slot], gsb / kGRawSlots, a.dev_err);
                const uint8_t *raw = sm + kOffRaw + slot * kRawStage + r * 144;
                const uint4 hdr = lds128(raw);
                if (hh == 0) hdr_d[sb * kGM + r] = f16_bits_to_f32(hdr.x);
                const float dmin = f16_bits_to_f32(hdr.x >> 16);
                for (uint32_t hf = 0; hf < 2; hf++, gs++) {
                    const uint32_t sa = gs % kGAStages;
                    if (gs >= (uint32_t)kGAStages) gemm_wait(&a_empty[sa], gs / kGAStages - 1, a.dev_err);
                    // scale_min (dequant.zig:291-300) of sub-blocks 4hf .. 4hf+3
                    const uint32_t scw = hf == 0 ? (hdr.y & 0x3F3F3F3Fu)
                                                 : ((hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u));
                    const uint32_t mnw = hf == 0 ? (hdr.z & 0x3F3F3F3Fu)
                                                 : (((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u));
                    // this thread: pair c = 2hf + hh (sub-blocks 2c, 2c+1) -> atom hh
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        const float v = dmin * (float)((mnw >> (16 * hh + 8 * j)) & 0xffu);  // exact in f32
                        __half h, l;
                        split_f16(v, h, l);
                        const uint32_t kk = 8 * sb + 4 * hf + 2 * hh + j;
                        *reinterpret_cast<__half *>(sm + kOffAm + sw128_offset(r, kk)) = h;
                        *reinterpret_cast<__half *>(sm + kOffAm + 16384 + sw128_offset(r, kk)) = l;
                    }
                    {
                        const float sc0 = (float)((scw >> (16 * hh)) & 0xffu);
                        const float sc1 = (float)((scw >> (16 * hh + 8)) & 0xffu);
                        const uint32_t s0 = half2_splat(sc0), b0 = half2_splat(-1024.0f * sc0);
                        const uint32_t s1 = half2_splat(sc1), b1 = half2_splat(-1024.0f * sc1);
                        const uint4 qa = lds128(raw + 16 + 32 * (2 * hf + hh));
                        const uint4 qb = lds128(raw + 32 + 32 * (2 * hf + hh));
                        const uint32_t wq[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                        uint8_t *arow = sm + kOffA + sa * 32768 + hh * 16384 + r * 128;
                        const uint32_t swz = r & 7;
#pragma unroll
                        for (int m = 0; m < 4; m++) {
                            // positions 8m..8m+7 hold elements 8m + (0,2,1,3,4,6,5,7) of sub-block 2c
                            uint4 lo, hi;
                            lo.x = hfma2_u32((wq[2 * m] & 0x000F000Fu) | 0x64006400u, s0, b0);
                            lo.y = hfma2_u32(((wq[2 * m] >> 8) & 0x000F000Fu) | 0x64006400u, s0, b0);
                            lo.z = hfma2_u32((wq[2 * m + 1] & 0x000F000Fu) | 0x64006400u, s0, b0);
                            lo.w = hfma2_u32(((wq[2 * m + 1] >> 8) & 0x000F000Fu) | 0x64006400u, s0, b0);
                            hi.x = hfma2_u32(((wq[2 * m] >> 4) & 0x000F000Fu) | 0x64006400u, s1, b1);
                            hi.y = hfma2_u32(((wq[2 * m] >> 12) & 0x000F000Fu) | 0x64006400u, s1, b1);
                            hi.z = hfma2_u32(((wq[2 * m + 1] >> 4) & 0x000F000Fu) | 0x64006400u, s1, b1);
                            hi.w = hfma2_u32(((wq[2 * m + 1] >> 12) & 0x000F000Fu) | 0x64006400u, s1, b1);
                            *reinterpret_cast<uint4 *>(arow + ((m ^ swz) << 4)) = lo;
                            *reinterpret_cast<uint4 *>(arow + (((4 + m) ^ swz) << 4)) = hi;
                        }
                    }
                    fence_async_smem();
                    mbar_arrive(&a_full[sa]);
                }
                mbar_arrive(&raw_empty[slot]);
                if (sb >= 1) fold(gsb - 1, sb - 1, 0.0f);
            }
            fold(gsb - 1, nsb - 1, 0.0f);
            gemm_wait(min_full, gi, a.dev_err);
            tc_fence_after();
            {
                uint32_t vh[PH], vl[PH];
                tload(2 * NNP + PH * hh, vh, vl);
                tc_fence_before();
                mbar_arrive(min_empty);
                const float *inv = s_inv + (gi & 1) * NP + PH * hh;  // written before bm_full, which min_full follows
#pragma unroll
                for (int q = 0; q < PH; q++)
                    y[q] = (y[q] - (__uint_as_float(vh[q]) + __uint_as_float(vl[q]))) * inv[q];
            }
            const uint32_t q0 = PH * hh;
            if (MODE == 1) {
                const uint32_t orow = kGM * it.m0 + r;
#pragma unroll
                for (uint32_t q = 0; q < (uint32_t)PH; q++)
                    if (q0 + q < it.nvalid) a.out[(size_t)(it.pos0 + q0 + q) * a.out_ld + orow] = y[q];
            } else {
                // the A stages are idle here: every MMA of this item has completed
                constexpr int UX = NP + 1;  // odd stride: no bank conflicts
                float *uex = reinterpret_cast<float *>(sm + kOffA);  // [64][UX]
                if (r >= 64)
#pragma unroll
                    for (int q = 0; q < PH; q++) uex[(r - 64) * UX + q0 + q] = y[q];
                math_sync();
                if (r < 64) {
                    const uint32_t f = 64 * it.m0 + r;
#pragma unroll
                    for (uint32_t q = 0; q < (uint32_t)PH; q++)
                        if (q0 + q < it.nvalid)
                            a.out[(size_t)(it.pos0 + q0 + q) * a.F + f] = act_apply(a.act, y[q]) * uex[r * UX + q0 + q];
                }
            }
            math_sync();  // uex read before the next item's A writes
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(taddr, Geo::kTmemCols);
}

// ── activation prep: f32 rows -> f16 hi/lo planes (K permuted in groups of 4
// as the dequantised weights are), sub-block sums, 2^e per row ─────────────
// One warp per row (eight rows per block): no block barriers, and every
// warp's loads in flight at once.  K % 256 == 0.
// With rowmap, output row r (a dispatch position) takes source row
// rowmap[r] / kdiv (its token); positions past the plan's last one hold stale
// map entries and are clamped to a valid row (no tile reads their results).
__global__ void __launch_bounds__(256) k_gemm_prep(const float *src, uint32_t K, uint32_t rows, __half *xh,
                                                   __half *xl, float *xsum, float *xinv, const uint32_t *rowmap,
                                                   uint32_t kdiv, uint32_t nsrc) {
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31, row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;
    const uint32_t srow = rowmap ? min(__ldg(rowmap + row) / kdiv, nsrc - 1) : row;
    const float *s = src + (size_t)srow * K;
    float amax = 0.0f;
#pragma unroll 4
    for (uint32_t i = 4 * lane; i < K; i += 128) {
        const float4 v = *reinterpret_cast<const float4 *>(s + i);
        amax = fmaxf(fmaxf(amax, fabsf(v.x)), fmaxf(fabsf(v.y), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int ex = 0;
    frexpf(amax, &ex);  // max|x| * 2^-ex in [0.5, 1)
    const float scale = ldexpf(1.0f, -ex);
    for (uint32_t m = lane; m < K / 8; m += 32) {
        const float4 p = *reinterpret_cast<const float4 *>(s + 8 * m);
        const float4 q = *reinterpret_cast<const float4 *>(s + 8 * m + 4);
        const float v[8] = {p.x, p.z, p.y, p.w, q.x, q.z, q.y, q.w};  // positions <- elements (0,2,1,3,...)
        __align__(16) __half h[8], l[8];
#pragma unroll
        for (int i = 0; i < 8; i++) split_f16(v[i] * scale, h[i], l[i]);
        *reinterpret_cast<uint4 *>(xh + (size_t)row * K + 8 * m) = *reinterpret_cast<uint4 *>(h);
        *reinterpret_cast<uint4 *>(xl + (size_t)row * K + 8 * m) = *reinterpret_cast<uint4 *>(l);
    }
    for (uint32_t j = lane; j < K / 32; j += 32) {  // each 32-column sum in column order
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            const float4 q = *reinterpret_cast<const float4 *>(s + 32 * j + i);
            v[i] = q.x;
            v[i + 1] = q.y;
            v[i + 2] = q.z;
            v[i + 3] = q.w;
        }
        float t = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; i++) t += v[i] * scale;
        xsum[(size_t)row * (K / 32) + j] = t;
    }
    if (lane == 0) xinv[row] = ldexpf(1.0f, ex);
}

// ── tile list: (active expert slot, first position) per NP positions ───────
// One block of kRouterMaxE threads: thread s counts the tiles of active slot
// s, a block-wide exclusive scan places them.
template <int NP>
__global__ void __launch_bounds__(kRouterMaxE) k_gemm_tiles(MoePlan p, uint2 *tiles, uint32_t *n_tiles) {
    __shared__ uint32_t s_warp[kRouterMaxE / 32];
    pdl_wait();
    const uint32_t s = threadIdx.x, lane = s & 31, warp = s >> 5;
    const uint32_t na = *p.n_active;
    const uint32_t cnt = s < na ? p.act_cnt[s] : 0;
    const uint32_t nt = (cnt + NP - 1) / NP;
    uint32_t incl = nt;  // inclusive scan within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= (uint32_t)o) incl += v;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    uint32_t base = 0;
    for (uint32_t w = 0; w < warp; w++) base += s_warp[w];
    const uint32_t first = base + incl - nt;
    for (uint32_t i = 0; i < nt; i++) tiles[first + i] = make_uint2(s, i * NP);
    if (s == blockDim.x - 1) *n_tiles = base + incl;
}

// ── weighted combine in slot order (+ residual) ─────────────────────────────
// One token row per blockIdx.x; with vec, four consecutive columns per thread
// (16-byte loads and stores; D % 4 == 0 and every pointer 16-byte aligned),
// else one.  Each element is the same sum in slot order either way.
__global__ void k_gemm_combine(const float *y, uint32_t D, const uint32_t *pair_pos, const float *w, uint32_t k,
                               const float *resid, float *out, int vec) {
    pdl_wait();
    const uint32_t t = blockIdx.x, c = blockIdx.y * blockDim.x + threadIdx.x;  // token rows in x: no 65535 cap
    if (vec) {
        if (4 * c >= D) return;
        float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);  // moe_buf is zeroed, then += scale * down, slot by slot
        for (uint32_t s = 0; s < k; s++) {
            const uint32_t pp = __ldg(pair_pos + (size_t)t * k + s);
            if (pp == 0xffffffffu) continue;  // a pair whose id the dispatch plan rejected contributes nothing
            const float ws = __ldg(w + (size_t)t * k + s);
            const float4 v = __ldg(reinterpret_cast<const float4 *>(y + (size_t)pp * D) + c);
            o.x = __fadd_rn(o.x, __fmul_rn(ws, v.x));
            o.y = __fadd_rn(o.y, __fmul_rn(ws, v.y));
            o.z = __fadd_rn(o.z, __fmul_rn(ws, v.z));
            o.w = __fadd_rn(o.w, __fmul_rn(ws, v.w));
        }
        const size_t oi = (size_t)t * D / 4 + c;
        if (resid) {
            const float4 r = reinterpret_cast<const float4 *>(resid)[oi];
            o.x = r.x + o.x;
            o.y = r.y + o.y;
            o.z = r.z + o.z;
            o.w = r.w + o.w;
        }
        reinterpret_cast<float4 *>(out)[oi] = o;
        return;
    }
    if (c >= D) return;
    float o = 0.0f;  // moe_buf is zeroed, then += scale * down, slot by slot (no fused multiply-add)
    for (uint32_t s = 0; s < k; s++) {
        const uint32_t pp = pair_pos[(size_t)t * k + s];
        if (pp == 0xffffffffu) continue;  // a pair whose id the dispatch plan rejected contributes nothing
        o = __fadd_rn(o, __fmul_rn(w[(size_t)t * k + s], y[(size_t)pp * D + c]));
    }
    const size_t oi = (size_t)t * D + c;
    out[oi] = resid ? resid[oi] + o : o;
}

// The combine's launch: the vector form when the shape and pointers allow it.
static cudaError_t launch_combine_k(const LaunchCfg &c, const char *label, const float *y, uint64_t D,
                                    const uint32_t *pair_pos, const float *w, uint32_t ntok, uint32_t k,
                                    const float *resid, float *out) {
    auto a16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    const int vec = D % 4 == 0 && a16(y) && a16(out) && (!resid || a16(resid));
    const uint64_t per = vec ? D / 4 : D;
    return launch_k(c, label, k_gemm_combine, dim3(ntok, (uint32_t)((per + 255) / 256)), dim3(256), 0, y, (uint32_t)D,
                    pair_pos, w, k, resid, out, vec);
}

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

// [total rows][pitch] byte view of a weight tensor, box = 144 bytes x 64 rows.
bool encode_rows(CUtensorMap *map, const void *base, uint64_t pitch, uint64_t total_rows) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[2] = {pitch, total_rows};
    const cuuint64_t strides[1] = {pitch};
    const cuuint32_t box[2] = {144, 64};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [rows][K] f16 activation plane as a tiled map: box 64 columns (128 bytes,
// 128B swizzle, the UMMA K-major atom) x np rows; out-of-range reads as zero.
bool encode_act(CUtensorMap *map, const void *base, uint64_t K, uint64_t rows, uint32_t np) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || (K * 2) % 16) return false;
    const cuuint64_t dims[2] = {K, rows};
    const cuuint64_t strides[1] = {K * 2};
    const cuuint32_t box[2] = {64, np};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_combine(const LaunchCfg &c, const float *y, uint64_t D, const uint32_t *pair_pos, const float *w,
                           uint32_t ntok, uint32_t k, const float *resid, float *out) {
    return launch_combine_k(c, "moe_combine", y, D, pair_pos, w, ntok, k, resid, out);
}

// The GEMM scheme of one weight tensor with K columns whose items take
// `rows` consecutive rows (gate/up: the expert width, in gate/up pairs;
// down: d_model): 0 for Q4_K in one exact plane, the type for stacked planes,
// -1 when neither takes it.
static int gemm_scheme(const DevMat &m, uint64_t K, uint64_t rows, bool gate_up) {
    if (m.type == T_Q4_K && K % 256 == 0 && K <= 256u * kGMaxSb && rows % (gate_up ? 64 : kGM) == 0) return 0;
    const bool rows_ok = rows % (gate_up ? 32 : kStkRows) == 0 && K <= 256u * kStkMaxSb;
    if ((m.type == T_Q4_K || m.type == T_Q6_K) && K % 256 == 0 && rows_ok) return (int)m.type;
    if (m.type == T_Q8_0 && K % 64 == 0 && rows_ok) return (int)m.type;
    return -1;
}

bool moe_gemm_supported(const DevMat &gate, const DevMat &down, uint64_t F) {
    return gate.n_experts <= (uint32_t)kRouterMaxE && gemm_scheme(gate, gate.cols, F, true) >= 0 &&
           gemm_scheme(down, F, down.rows, false) >= 0;
}

size_t moe_gemm_scratch(uint32_t T, uint32_t k, uint32_t E, uint64_t d, uint64_t F) {
    const size_t P = (size_t)T * k;
    auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t max_tiles = (E < P ? E : P) + P / kGN + 1;
    return al(max_tiles * 8) + al(4) + 2 * al(P * d * 2) + al(P * d / 8) + al(P * 4) + al(P * F * 4) +
           2 * al(P * F * 2) + al(P * F / 8) + al(P * 4) + al(P * d * 4);
}

// One GEMM launch of a mode with the instantiation for its weight scheme and
// tile width.
template <int MODE>
static cudaError_t launch_gemm(const LaunchCfg &c, const char *label, bool wide, int ws, const GemmArgs &g) {
    const dim3 grid((uint32_t)c.num_sms), block(kGThreadsV2);
#define LT_GEMM_CASE(WS_)                                                                                   \
    return wide ? launch_k(c, label, k_moe_gemm<MODE, 64, WS_>, grid, block, (size_t)GemmGeo<64>::kSmem, g) \
                : launch_k(c, label, k_moe_gemm<MODE, 32, WS_>, grid, block, (size_t)GemmGeo<32>::kSmem, g)
    switch (ws) {
        case 0: LT_GEMM_CASE(0);
        case T_Q4_K: LT_GEMM_CASE(T_Q4_K);
        case T_Q6_K: LT_GEMM_CASE(T_Q6_K);
        case T_Q8_0: LT_GEMM_CASE(T_Q8_0);
        default: return cudaErrorInvalidValue;
    }
#undef LT_GEMM_CASE
}

cudaError_t launch_moe_gemm_ffn(const LaunchCfg &c, const DevMat &gate, const uint8_t *up, const DevMat &down, int act,
                                const float *x, uint32_t T, uint32_t k, const float *w, const MoePlan &p,
                                const float *resid, float *out, uint8_t *scratch) {
    const uint32_t E = gate.n_experts;
    const uint64_t d = gate.cols, F = down.cols;
    const int ws_gu = gemm_scheme(gate, d, F, true), ws_dn = gemm_scheme(down, F, d, false);
    if (ws_gu < 0 || ws_dn < 0) return cudaErrorInvalidValue;
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
    // the expert input's planes in dispatch-position order (P rows: each
    // token once per selected expert), so every tile's rows are consecutive
    __half *xh = reinterpret_cast<__half *>(take(P * d * 2));
    __half *xl = reinterpret_cast<__half *>(take(P * d * 2));
    float *xsum = reinterpret_cast<float *>(take(P * d / 8));
    float *xinv = reinterpret_cast<float *>(take(P * 4));
    float *hbuf = reinterpret_cast<float *>(take(P * F * 4));
    __half *hh = reinterpret_cast<__half *>(take(P * F * 2));
    __half *hl = reinterpret_cast<__half *>(take(P * F * 2));
    float *hsum = reinterpret_cast<float *>(take(P * F / 8));
    float *hinv = reinterpret_cast<float *>(take(P * 4));
    float *ybuf = reinterpret_cast<float *>(take(P * d * 4));

    // wide tiles when the experts average at least 48 positions
    const bool wide = P >= (size_t)48 * (E ? E : 1);
    cudaError_t e = wide ? launch_k(c, "moe_gemm_tiles", k_gemm_tiles<64>, dim3(1), dim3(kRouterMaxE), 0, p, tiles,
                                    n_tiles)
                         : launch_k(c, "moe_gemm_tiles", k_gemm_tiles<32>, dim3(1), dim3(kRouterMaxE), 0, p, tiles,
                                    n_tiles);
    if (e == cudaSuccess)
        e = launch_k(c, "moe_gemm_prep", k_gemm_prep, dim3((uint32_t)((P + 7) / 8)), dim3(256), 0, x, (uint32_t)d,
                     (uint32_t)P, xh, xl, xsum, xinv, (const uint32_t *)p.pos_pair, k, T);
    GemmArgs g;
    memset(&g, 0, sizeof(g));  // the tensor maps a launch does not use stay zero
    const uint32_t E1 = E ? E : 1;
    // tensor maps only for the single-plane Q4_K scheme (its rows are 16-byte multiples)
    if (ws_gu == 0 && (!encode_rows(&g.map_w, gate.data, gate.pitch, (uint64_t)gate.rows * E1) ||
                       (up && !encode_rows(&g.map_up, up, gate.pitch, (uint64_t)F * E1))))
        return cudaErrorInvalidValue;
    if (ws_gu != 0) memset(&g.map_w, 0, sizeof(g.map_w));
    if (!up || ws_gu != 0) g.map_up = g.map_w;
    g.w = gate.data;
    g.w_up = up;
    g.w_end = gate.data + (size_t)gate.rows * E1 * gate.pitch;
    g.up_end = up ? up + (size_t)F * E1 * gate.pitch : nullptr;
    g.pitch = gate.pitch;
    g.K = (uint32_t)d;
    g.rows_e = (uint32_t)gate.rows;
    g.F = (uint32_t)F;
    g.mt = (uint32_t)(ws_gu == 0 ? F / 64 : F / 32);
    g.act = act;
    g.p = p;
    g.tiles = tiles;
    g.n_tiles = n_tiles;
    g.k = k;
    g.xh = xh;
    g.xl = xl;
    if (!encode_act(&g.map_bh, xh, d, P, wide ? 64 : 32) || !encode_act(&g.map_bl, xl, d, P, wide ? 64 : 32))
        return cudaErrorInvalidValue;
    g.xsum = xsum;
    g.xinv = xinv;
    g.out = hbuf;
    g.out_ld = (uint32_t)F;
    g.dev_err = c.dev_err;
    if (e == cudaSuccess) e = launch_gemm<0>(c, "moe_gemm_gate_up", wide, ws_gu, g);
    if (e == cudaSuccess)
        e = launch_k(c, "moe_gemm_prep", k_gemm_prep, dim3((uint32_t)((P + 7) / 8)), dim3(256), 0, (const float *)hbuf,
                     (uint32_t)F, (uint32_t)P, hh, hl, hsum, hinv, (const uint32_t *)nullptr, 1u, (uint32_t)P);
    GemmArgs gd = g;
    if (ws_dn == 0) {
        if (!encode_rows(&gd.map_w, down.data, down.pitch, (uint64_t)down.rows * E1)) return cudaErrorInvalidValue;
    } else {
        memset(&gd.map_w, 0, sizeof(gd.map_w));
    }
    gd.map_up = gd.map_w;
    gd.w = down.data;
    gd.w_up = nullptr;
    gd.w_end = down.data + (size_t)down.rows * E1 * down.pitch;
    gd.up_end = nullptr;
    gd.pitch = down.pitch;
    gd.K = (uint32_t)F;
    gd.rows_e = (uint32_t)down.rows;
    gd.mt = (uint32_t)(ws_dn == 0 ? d / kGM : d / kStkRows);
    gd.xh = hh;
    gd.xl = hl;
    if (!encode_act(&gd.map_bh, hh, F, P, wide ? 64 : 32) || !encode_act(&gd.map_bl, hl, F, P, wide ? 64 : 32))
        return cudaErrorInvalidValue;
    gd.xsum = hsum;
    gd.xinv = hinv;
    gd.out = ybuf;
    gd.out_ld = (uint32_t)d;
    if (e == cudaSuccess) e = launch_gemm<1>(c, "moe_gemm_down", wide, ws_dn, gd);
    if (e == cudaSuccess)
        e = launch_combine_k(c, "moe_gemm_combine", (const float *)ybuf, d, (const uint32_t *)p.pair_pos, w, T, k,
                             resid, out);
    return e;
}

}  // namespace lt
