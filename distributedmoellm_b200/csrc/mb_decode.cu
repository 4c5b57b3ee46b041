// Fused decode mat-vecs over packed experts: one MoE layer's gate|up, SiLU,
// down for every (expert, pick) of experts picked by few tokens.
//
// Reference: moelan/kernels.py:712-782 (_moe_q4, one call per layer) and the
// per-expert int8 kernels (kernels.py:133-168), all f32.
//
// Design (sm_100a):
//  * Weights live in the device tile layout: 16-row tiles, each a contiguous
//    run of 1 KB (int4) / 2 KB (int8) blocks of 128 columns plus the blocks'
//    group scales.  One producer warp streams MT consecutive tiles per stage
//    (~30 KB) into a shared-memory ring with 1-D bulk copies on the TMA engine
//    (mbarrier completion); the working set moves HBM -> SMEM exactly once.
//  * MMA warps split K: warp w owns quad w (128 columns) of every tile.
//    Weights are unpacked to exact f16 (values -8..7 / -128..127) with
//    lop3/prmt + one f16x2 op per pair, and multiplied on the tensor cores by
//    mma.sync m16n8k16 against the activations split into two f16 pieces
//    (x * 2^e = hi + lo, 22 significant bits) laid along N, with f32
//    accumulation: the products are exact, so results match an f32 mat-vec to
//    rounding.  mma.sync is used because its operands come from registers:
//    a decode mat-vec is bound by HBM, and this keeps the unpacked weights out
//    of shared memory entirely (tcgen05 would need them staged there).
//  * Each group of 32 columns is accumulated separately and scaled by its
//    group scale in f32; the K-split partials go through shared-memory
//    reduction buffers (mbarrier hand-off) to two epilogue warps, which sum
//    them with 128-bit loads.
//  * Phase 1 (gate|up) tiles interleave 8 gate rows with the 8 matching up
//    rows, so SiLU(gate) * up is formed in the epilogue and only the
//    activation row (P x I) goes back to HBM, with each pick's max |act|.
//  * Phase 2 (down) writes each pick's unweighted output row; the weighted
//    combine is a separate deterministic kernel.
//  * Work units are (expert, chunk of 8 picks, MT row tiles), split
//    contiguously over a persistent grid so each CTA touches one or two
//    experts.
//  * K above 2048 (16 MMA warps of one 128-column quad each) is cut into
//    windows of 16 quads: a CTA walks each segment of its units (up to 32 row
//    tiles of one chunk) once per window, loading the activation fragments of
//    the window once per segment, and the epilogue keeps the segment's partial
//    sums in shared memory until the last window.
//  * The affine int4 format (GGUF Q4_K as (u - 8) * scale + bias per group of
//    32) adds bias * (the group's sum of the activations) per group, the sums
//    formed once per chunk and window from the same scaled activations.
#include <algorithm>
#include <type_traits>

#include "mb_common.cuh"

namespace {

constexpr int kMaxKW = 16;      // MMA warps: one per quad (128 columns) of a K window of up to 2048 columns
constexpr int kEpiWarps = 2;    // epilogue warps, taking alternate items (one warp with K windows)
#ifndef MB_DECODE_MAX_MT
#define MB_DECODE_MAX_MT 6
#endif
constexpr int kMaxMT = MB_DECODE_MAX_MT;   // row tiles per stage
constexpr int kRedTile = 128;   // floats of one warp's partial of one tile: [8 input rows][16 rows]
constexpr int kMaxCachedE = 1024;  // experts whose weight address the kernel keeps in shared memory
constexpr int kMaxCachedP = 1024;  // picks whose token row and exponent the kernel keeps in shared memory
#ifndef MB_DECODE_WAIT
#define MB_DECODE_WAIT mb_mbar_wait   // the MMA and epilogue warps' waits (mb_mbar_wait_spin: no sleeps)
#endif
#ifndef MB_DECODE_STAGE_KB
#define MB_DECODE_STAGE_KB 48   // target bytes of one stage of row tiles, in KB
#endif
#ifndef MB_DECODE_STAGE_KB_SMALL
#define MB_DECODE_STAGE_KB_SMALL 32   // the same for calls of at most MB_DECODE_SMALL_P picks
#endif
#ifndef MB_DECODE_SMALL_P
#define MB_DECODE_SMALL_P 16
#endif
#ifndef MB_DECODE_NRED
#define MB_DECODE_NRED 2        // reduction slots per epilogue warp with many MMA warps
#endif
#ifndef MB_DECODE_NRED_NARROW
#define MB_DECODE_NRED_NARROW 1 // the same with at most 8 MMA warps (two CTAs per SM)
#endif
constexpr int kSegTiles = 32;   // K > 2048: row tiles of a segment whose partial sums wait in shared memory

struct Fmt {
    int data_bytes;   // per block: 1024 (int4) or 2048 (int8)
    int scale_f16;    // scale element 2 or 4 bytes
    int affine;       // int4 with an f32 bias per group after the scales (GGUF Q4_K)
    int block_bytes;
};

__host__ __device__ inline Fmt fmt_info(int fmt)
{
    Fmt f;
    f.data_bytes = (fmt == MB_FMT_Q8_F16 || fmt == MB_FMT_Q8_F32) ? 2048 : 1024;
    f.scale_f16 = (fmt == MB_FMT_Q4_F16 || fmt == MB_FMT_Q8_F16) ? 1 : 0;
    f.affine = fmt == MB_FMT_Q4K_F32;
    f.block_bytes = f.data_bytes + 16 * 4 * (f.scale_f16 ? 2 : 4) + (f.affine ? 16 * 4 * 4 : 0);
    return f;
}

struct DecodeArgs {
    const MbExpert* table;
    int E;
    int phase;        // 1: gate|up -> act, 2: down -> y
    int K;            // real input columns
    int NQ;           // quads per tile row (K padded to 128)
    int QW;           // quads per K window (= MMA warps)
    int NW;           // K windows: one MMA warp per quad of a window, windows one after another
    int SEG;          // units (stages) of a segment: the partial sums of its tiles wait for the last window
    int RT;           // row tiles
    int MT;           // row tiles per stage
    int O_real;       // phase 1: I (act columns), phase 2: H (y columns)
    int src_ld;       // floats per input row (x: H, act: I_pad)
    int act_ld;       // I_pad
    int y_ld;         // H
    int KW;           // MMA warps (= QW)
    int stages, tile_bytes, nred;
    const int32_t* counts;
    const int32_t* offsets;
    const int32_t* sorted_rows;
    const float* x;
    const int32_t* row_exp;
    float* act;
    unsigned* act_max;
    float* y;
    int max_rows;
    int P;            // picks (rows of act / entries of sorted_rows)
    int PC;           // picks 0..PC-1 have their row and exponent in shared memory
    unsigned* status;
    // single-matrix mode (mb_matmul_t): one "expert" whose phase-2 matrix is
    // single_w, picked by single_n input rows 0..single_n-1
    const void* single_w;
    int single_n;
};

__device__ __forceinline__ int64_t items_of(int n, int max_rows, int RTS)
{
    return (n > 0 && n <= max_rows) ? (int64_t)((n + 7) >> 3) * RTS : 0;
}

// Estimated cost of the work, for splitting it over the CTAs: a unit (one
// stage of row tiles over all of K) of a chunk of at most 4 picks costs
// kCostOne, of 5..8 picks (both N tiles of the MMAs live) kCostTwo, and the
// first unit of a chunk kCostSwitch more (the chunk's activation rows are
// gathered from global memory there).  Unit weights from per-unit timings on
// B200 (0.94 / 1.18 us per two-tile unit); the switch weight is the best of 0,
// 3, 6, 12 and 20 in timed decode steps (T = 32 and 64): with the rows kept in
// L2 a switch mostly overlaps the stages already in flight.
constexpr int kCostOne = 4, kCostTwo = 5, kCostSwitch = 3;

__device__ __forceinline__ int64_t cost_of(int n, int max_rows, int RTS)
{
    if (n <= 0 || n > max_rows) return 0;
    const int64_t full = (n - 1) >> 3;                // chunks of 8 picks before the last
    const int last = n - 8 * (int)full;               // picks of the last chunk, 1..8
    return full * ((int64_t)RTS * kCostTwo + kCostSwitch) + (int64_t)RTS * (last > 4 ? kCostTwo : kCostOne) +
           kCostSwitch;
}

// The first unit whose start cost is at least c (pre: unit prefix, cpre: cost prefix over experts).
__device__ int64_t item_at_cost(const int64_t* pre, const int64_t* cpre, const int32_t* cnt, int E, int RTS, int64_t c)
{
    if (c >= cpre[E]) return pre[E];
    int lo = 0, hi = E;  // the last expert with cpre[lo] <= c (a non-empty one, since cpre[lo + 1] > c)
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (cpre[mid] <= c) lo = mid;
        else hi = mid;
    }
    const int n = cnt[lo];
    const int64_t full = (n - 1) >> 3;
    const int last = n - 8 * (int)full;
    const int64_t tf = (int64_t)RTS * kCostTwo + kCostSwitch;
    int64_t rel = c - cpre[lo], j;
    int cc;
    if (rel < full * tf) {
        j = rel / tf;
        rel -= j * tf;
        cc = kCostTwo;
    } else {
        j = full;
        rel -= full * tf;
        cc = last > 4 ? kCostTwo : kCostOne;
    }
    // unit 0 of a chunk spans [0, kCostSwitch + cc), unit k >= 1 starts at kCostSwitch + k * cc
    const int64_t k = rel == 0 ? 0 : max((int64_t)1, (rel - kCostSwitch + cc - 1) / cc);
    return pre[lo] + j * RTS + k;
}

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// Unpacked f16 pairs of one 32-bit word of offset-form nibbles (u = v + 8):
// p[j] holds the values of columns 8t+j and 8t+j+4 of the group.
__device__ __forceinline__ void unpack_q4(uint32_t w, uint32_t (&p)[4])
{
    const uint32_t kMagic = 0x64006400u, kSubLo = 0x64086408u, kSixteenth = 0x2C002C00u, kMinus72 = 0xD480D480u;
    const uint32_t w8 = w >> 8;
    p[0] = mb_hsub2(mb_lop_and_or(w, 0x000F000Fu, kMagic), kSubLo);
    p[1] = mb_hfma2(mb_lop_and_or(w, 0x00F000F0u, kMagic), kSixteenth, kMinus72);
    p[2] = mb_hsub2(mb_lop_and_or(w8, 0x000F000Fu, kMagic), kSubLo);
    p[3] = mb_hfma2(mb_lop_and_or(w8, 0x00F000F0u, kMagic), kSixteenth, kMinus72);
}

// Unpacked f16 pairs of two words of offset-form int8 (u = q + 128) stored as
// [c0 c4 c1 c5][c2 c6 c3 c7]: p[j] = (q(c_j), q(c_j+4)).
__device__ __forceinline__ void unpack_q8(uint32_t w0, uint32_t w1, uint32_t (&p)[4])
{
    const uint32_t kHi = 0x64646464u, kSub = 0x64806480u;
    p[0] = mb_hsub2(mb_prmt(w0, kHi, 0x4140u), kSub);
    p[1] = mb_hsub2(mb_prmt(w0, kHi, 0x4342u), kSub);
    p[2] = mb_hsub2(mb_prmt(w1, kHi, 0x4140u), kSub);
    p[3] = mb_hsub2(mb_prmt(w1, kHi, 0x4342u), kSub);
}

template <bool F16S>
__device__ __forceinline__ void scales4(const uint8_t* p, float (&s)[4])
{
    if (F16S) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        const __half2 a = *reinterpret_cast<const __half2*>(&v.x), b = *reinterpret_cast<const __half2*>(&v.y);
        s[0] = __low2float(a);
        s[1] = __high2float(a);
        s[2] = __low2float(b);
        s[3] = __high2float(b);
    } else {
        const float4 v = *reinterpret_cast<const float4*>(p);
        s[0] = v.x;
        s[1] = v.y;
        s[2] = v.z;
        s[3] = v.w;
    }
}

// Cursor over the units (expert, chunk of 8 picks, stage of MT row tiles).
struct ItemCursor {
    int e, c, sg;
    __device__ __forceinline__ void start(const int64_t* pre, int E, int RTS, int64_t item)
    {
        int lo = 0, hi = E;  // pre[lo] <= item < pre[hi]
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (pre[mid] <= item) lo = mid;
            else hi = mid;
        }
        e = lo;
        const int rem = (int)(item - pre[lo]);
        c = rem / RTS;
        sg = rem - c * RTS;
    }
    __device__ __forceinline__ void next(const int64_t* pre, int E, int RTS)
    {
        if (++sg < RTS) return;
        sg = 0;
        if ((int64_t)(++c) * RTS < pre[e + 1] - pre[e]) return;
        c = 0;
        do {
            ++e;
        } while (e < E - 1 && pre[e + 1] == pre[e]);
    }
};

// Cursor over the work items of one CTA: its run of units is cut into
// segments (consecutive units of one chunk, at most SEG of them), and each
// segment is walked once per K window, so the activation fragments of a window
// are loaded once per segment and the partial sums of a segment's tiles wait in
// shared memory for the last window.  With one window (K <= 2048) the items are
// the units themselves, in order.
struct WinCursor {
    ItemCursor u, s0;   // the current unit, the segment's first unit
    int64_t rem;        // units of the run from the segment's first unit on
    int j, len, w;      // unit within the segment, segment length, window
    __device__ __forceinline__ void seg_init(int RTS, int SEG)
    {
        int64_t l = RTS - u.sg;                 // units left in this chunk
        if (l > SEG) l = SEG;
        if (l > rem) l = rem;
        len = (int)l;
    }
    __device__ __forceinline__ void start(const int64_t* pre, int E, int RTS, int SEG, int64_t lo, int64_t hi)
    {
        u.start(pre, E, RTS, lo);
        s0 = u;
        rem = hi - lo;
        j = w = 0;
        seg_init(RTS, SEG);
    }
    // With one window the items are the units: only the unit cursor moves.
    __device__ __forceinline__ void advance(const int64_t* pre, int E, int RTS, int SEG, int NW)
    {
        if (NW == 1) u.next(pre, E, RTS);
        else next(pre, E, RTS, SEG, NW);
    }
    __device__ __forceinline__ void next(const int64_t* pre, int E, int RTS, int SEG, int NW)
    {
        if (++j < len) {
            u.next(pre, E, RTS);
            return;
        }
        j = 0;
        if (++w < NW) {
            u = s0;
            return;
        }
        w = 0;
        rem -= len;
        u.next(pre, E, RTS);
        s0 = u;
        if (rem > 0) seg_init(RTS, SEG);
    }
};

// One row tile of one MMA warp: its block (16 rows x 128 columns) of a tile in
// shared memory against the activation fragments bf, group scales applied in
// f32 (and for the affine format the group biases times the rows' group sums
// xs), the partial sums stored to rt ([input row][16 rows]).  has: the warp's
// quad exists in this K window (else its partials are zero).  TWO: the second N
// tile (input rows 4..7) is live.  The plain int4 formats test `has` once per
// item in the caller (always true here: fewer instructions per tile, measured
// faster); the int8 and affine formats test it per tile, which keeps their
// register allocation (the hoisted form spilled more there and measured
// slower on the Mixtral GGUF layer).
template <bool Q8, bool F16S, bool AFF, bool TWO>
__device__ __forceinline__ void tile_mma(const uint8_t* __restrict__ blk, bool has, const uint32_t (&bf)[2][4][4],
                                         const float (&xs)[2][4], float* __restrict__ rt, int t, int g)
{
    constexpr int kData = Q8 ? 2048 : 1024;
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // [N tile][row g, row g+8] of input row 4nt + t
    if ((!Q8 && !AFF) || has) {
        const uint8_t* wp = blk + g * 64 + t * 16;
        const uint8_t* sp = blk + kData + g * (F16S ? 8 : 16);
        uint32_t wg[Q8 ? 8 : 4], wh[Q8 ? 8 : 4];
        {
            const uint4 a0 = *reinterpret_cast<const uint4*>(wp);
            const uint4 b0 = *reinterpret_cast<const uint4*>(wp + 8 * 64);
            wg[0] = a0.x; wg[1] = a0.y; wg[2] = a0.z; wg[3] = a0.w;
            wh[0] = b0.x; wh[1] = b0.y; wh[2] = b0.z; wh[3] = b0.w;
        }
        if (Q8) {
            const uint4 a1 = *reinterpret_cast<const uint4*>(wp + 1024);
            const uint4 b1 = *reinterpret_cast<const uint4*>(wp + 1024 + 8 * 64);
            wg[Q8 ? 4 : 0] = a1.x; wg[Q8 ? 5 : 1] = a1.y; wg[Q8 ? 6 : 2] = a1.z; wg[Q8 ? 7 : 3] = a1.w;
            wh[Q8 ? 4 : 0] = b1.x; wh[Q8 ? 5 : 1] = b1.y; wh[Q8 ? 6 : 2] = b1.z; wh[Q8 ? 7 : 3] = b1.w;
        }
        float sg[4], sh[4], bg[4], bh[4];
        scales4<F16S>(sp, sg);
        scales4<F16S>(sp + 8 * (F16S ? 8 : 16), sh);
        if (AFF) {   // biases follow the 16 x 4 f32 scales
            scales4<false>(sp + 256, bg);
            scales4<false>(sp + 256 + 8 * 16, bh);
        }
#pragma unroll
        for (int gi = 0; gi < 4; ++gi) {
            uint32_t pg[4], ph_[4];
            if (Q8) {
                unpack_q8(wg[(2 * gi) % (Q8 ? 8 : 4)], wg[(2 * gi + 1) % (Q8 ? 8 : 4)], pg);
                unpack_q8(wh[(2 * gi) % (Q8 ? 8 : 4)], wh[(2 * gi + 1) % (Q8 ? 8 : 4)], ph_);
            } else {
                unpack_q4(wg[gi], pg);
                unpack_q4(wh[gi], ph_);
            }
            float d[4];
            mb_mma_f16_zero(d, pg[0], ph_[0], pg[1], ph_[1], bf[0][gi][0], bf[0][gi][1]);
            mb_mma_f16(d, pg[2], ph_[2], pg[3], ph_[3], bf[0][gi][2], bf[0][gi][3]);
            acc[0][0] = fmaf(d[0] + d[1], sg[gi], acc[0][0]);
            acc[0][1] = fmaf(d[2] + d[3], sh[gi], acc[0][1]);
            if (AFF) {
                acc[0][0] = fmaf(xs[0][gi], bg[gi], acc[0][0]);
                acc[0][1] = fmaf(xs[0][gi], bh[gi], acc[0][1]);
            }
            if (TWO) {
                float e[4];
                mb_mma_f16_zero(e, pg[0], ph_[0], pg[1], ph_[1], bf[1][gi][0], bf[1][gi][1]);
                mb_mma_f16(e, pg[2], ph_[2], pg[3], ph_[3], bf[1][gi][2], bf[1][gi][3]);
                acc[1][0] = fmaf(e[0] + e[1], sg[gi], acc[1][0]);
                acc[1][1] = fmaf(e[2] + e[3], sh[gi], acc[1][1]);
                if (AFF) {
                    acc[1][0] = fmaf(xs[1][gi], bg[gi], acc[1][0]);
                    acc[1][1] = fmaf(xs[1][gi], bh[gi], acc[1][1]);
                }
            }
        }
    }
    rt[t * 16 + g] = acc[0][0];
    rt[t * 16 + g + 8] = acc[0][1];
    rt[(4 + t) * 16 + g] = acc[1][0];
    rt[(4 + t) * 16 + g + 8] = acc[1][1];
}

// Warp roles: [0, KW) MMA warps (warp w owns quad w of the current K window),
// KW the TMA producer, KW+1 and KW+2 the epilogue (alternate items; with K
// windows the first takes every item).  Shared memory: weight stages | reduction buffers [nred][KW][MT][8][16]
// | segment sums [SEG * MT][8][16] (K > 2048 only) | mbarriers | unit prefix |
// abort flag.
constexpr int kThreadsMax = (kMaxKW + 1 + kEpiWarps) * 32;

template <int FMT>
__global__ void __launch_bounds__(kThreadsMax, 1) moe_decode_kernel(const __grid_constant__ DecodeArgs a)
{
    constexpr bool Q8 = (FMT == MB_FMT_Q8_F16 || FMT == MB_FMT_Q8_F32);
    constexpr bool F16S = (FMT == MB_FMT_Q4_F16 || FMT == MB_FMT_Q8_F16);
    constexpr bool AFF = FMT == MB_FMT_Q4K_F32;
    constexpr int kData = Q8 ? 2048 : 1024;
    constexpr int kBlock = kData + 16 * 4 * (F16S ? 2 : 4) + (AFF ? 16 * 4 * 4 : 0);

    const int S = a.stages, KW = a.KW, E = a.E, RT = a.RT, MT = a.MT, NR = a.nred;
    const int NW = a.NW, QW = a.QW, NQ = a.NQ, SEG = a.SEG;
    const int RTS = (RT + MT - 1) / MT;
    const int tile_bytes = a.tile_bytes;      // one row tile over all of K in global memory
    const int wt_bytes = QW * kBlock;         // one row tile over one K window in a stage
    const int stage_bytes = MT * wt_bytes;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem;
    float* red = reinterpret_cast<float*>(smem + (size_t)S * stage_bytes);
    const int red_buf = KW * MT * kRedTile;  // floats per reduction buffer
    float* segsum = red + NR * red_buf;                                   // [SEG * MT][kRedTile] when NW > 1
    uint64_t* full = reinterpret_cast<uint64_t*>(segsum + (NW > 1 ? SEG * MT * kRedTile : 0));
    uint64_t* empty = full + S;
    uint64_t* rfull = empty + S;
    uint64_t* rempty = rfull + NR;
    int64_t* pre = reinterpret_cast<int64_t*>(rempty + NR);  // [E+1] units before expert e
    int64_t* cpre = pre + E + 1;                                // [E+1] their cost
    const uint8_t** wptr_s = reinterpret_cast<const uint8_t**>(cpre + E + 1);  // [E] when E <= kMaxCachedE
    int32_t* cnt_s = reinterpret_cast<int32_t*>(wptr_s + (E <= kMaxCachedE ? E : 0));  // [E] picks per expert
    int32_t* off_s = cnt_s + E;                                                          // [E] first pick
    const int PC = a.PC;  // picks cached below
    int32_t* row_s = off_s + E;                                // [PC] phase 1: token row of pick p
    int32_t* exp_s = row_s + (a.phase == 1 ? PC : 0);          // [PC] exponent of pick p's input row
    volatile int* abort_flag = reinterpret_cast<volatile int*>(exp_s + PC);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;

    // Launched programmatically after the kernel before it (mb_launch_pdl).  The gate|up phase reads the
    // routing that kernel wrote, so it waits first.  The down phase needs only the routing (complete
    // before the gate|up phase began) and its own weights until it reads the activations: its producer
    // starts streaming while the gate|up phase drains, the other warps wait below.
    if (a.phase == 1) mb_pdl_wait();
    mb_pdl_trigger();

    // the routing of every expert (and its weights' address) into shared memory,
    // all loads in flight together
    for (int e = tid; e < E; e += blockDim.x) {
        cnt_s[e] = a.single_n ? (e == 0 ? a.single_n : 0) : a.counts[e];
        off_s[e] = a.single_n ? 0 : a.offsets[e];
        if (E <= kMaxCachedE)
            wptr_s[e] = reinterpret_cast<const uint8_t*>(
                a.single_w ? a.single_w : (a.phase == 1 ? a.table[e].gu : a.table[e].down));
    }
    __syncthreads();
    if (warp == 0) {  // units and costs per expert -> prefixes
        int64_t run = 0, crun = 0;
        for (int base = 0; base < E; base += 32) {
            const int e = base + lane;
            int64_t v = 0, cv = 0;
            if (e < E) {
                v = items_of(cnt_s[e], a.max_rows, RTS);
                cv = cost_of(cnt_s[e], a.max_rows, RTS);
            }
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t u = __shfl_up_sync(0xffffffffu, v, o), cu = __shfl_up_sync(0xffffffffu, cv, o);
                if (lane >= o) {
                    v += u;
                    cv += cu;
                }
            }
            if (e < E) {
                pre[e + 1] = run + v;
                cpre[e + 1] = crun + cv;
            }
            run += __shfl_sync(0xffffffffu, v, 31);
            crun += __shfl_sync(0xffffffffu, cv, 31);
        }
        if (lane == 0) pre[0] = cpre[0] = 0;
    }
    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mb_mbar_init(&full[i], 1);
            mb_mbar_init(&empty[i], KW);
        }
        for (int i = 0; i < NR; ++i) {
            mb_mbar_init(&rfull[i], KW);
            mb_mbar_init(&rempty[i], 1);  // the epilogue warp that took the item
        }
        *abort_flag = 0;
        mb_fence_mbar_init();
    }
    __syncthreads();

    // this CTA's contiguous run of units: an equal share of the estimated cost
    const int64_t ctotal = cpre[E];
    const int64_t lo = item_at_cost(pre, cpre, cnt_s, E, RTS, ctotal * blockIdx.x / gridDim.x);
    const int64_t hi = item_at_cost(pre, cpre, cnt_s, E, RTS, ctotal * (blockIdx.x + 1) / gridDim.x);
    if (lo >= hi) {
        // nothing to do; still wait, so that this kernel completes only after the one before it
        if (a.phase == 2) mb_pdl_wait();
        return;
    }
    const int64_t n_items = (hi - lo) * NW;
    WinCursor cur;
    cur.start(pre, E, RTS, SEG, lo, hi);

    // the picks' rows and exponents, filled by the MMA and epilogue warps while the
    // producer starts the first weight copies (named barrier 1 excludes the producer)
    if (a.phase == 2 && warp != KW) mb_pdl_wait();   // the activations and their maxima are complete
    if (PC > 0 && warp != KW) {
        const int nthr = (KW + kEpiWarps) * 32, i0 = warp < KW ? tid : tid - 32;
        for (int p = i0; p < PC; p += nthr) {
            if (a.phase == 1) {
                const int row = a.sorted_rows[p];
                row_s[p] = row;
                exp_s[p] = a.row_exp[row];
            } else {
                exp_s[p] = mb_row_exponent(__uint_as_float(a.act_max[p]));
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
    }

    // ------------------------------------------------------------- producer
    if (warp == KW) {
        if (lane == 0) {
            const uint64_t wpol = mb_policy_evict_first();
            int s = 0;
            uint32_t ph = 0;
            int we = -1;
            const uint8_t* wbase = nullptr;
            for (int64_t it = 0; it < n_items; ++it, cur.advance(pre, E, RTS, SEG, NW)) {
                if (it >= S && !mb_mbar_wait(&empty[s], ph ^ 1u, a.status, abort_flag)) break;
                if (cur.u.e != we) {
                    we = cur.u.e;
                    wbase = E <= kMaxCachedE ? wptr_s[we]
                                             : reinterpret_cast<const uint8_t*>(
                                                   a.single_w ? a.single_w
                                                              : (a.phase == 1 ? a.table[we].gu : a.table[we].down));
                }
                const int nt = min(MT, RT - cur.u.sg * MT);
                uint8_t* dst = stages + (size_t)s * stage_bytes;
                const uint8_t* src = wbase + (int64_t)cur.u.sg * MT * tile_bytes;
                if (NW == 1) {   // the stage's tiles are contiguous: one copy
                    const uint32_t bytes = (uint32_t)(nt * tile_bytes);
                    mb_mbar_arrive_expect_tx(&full[s], bytes);
                    mb_bulk_g2s_hint(dst, src, bytes, &full[s], wpol);   // weights are read once: rows stay in L2
                } else {         // one copy per tile: the window's blocks of each tile
                    const int qn = min(QW, NQ - cur.w * QW);
                    const uint32_t wb = (uint32_t)(qn * kBlock);
                    mb_mbar_arrive_expect_tx(&full[s], wb * (uint32_t)nt);
                    src += (int64_t)cur.w * QW * kBlock;
                    for (int mt = 0; mt < nt; ++mt)
                        mb_bulk_g2s_hint(dst + (size_t)mt * wt_bytes, src + (int64_t)mt * tile_bytes, wb, &full[s],
                                         wpol);
                }
                if (++s == S) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
        return;
    }

    // ------------------------------------------------------------- epilogue
    if (warp > KW) {
        // Which items this warp takes.  One K window: alternate items (it % kEpiWarps), so each reduction
        // slot (NR a multiple of kEpiWarps) always goes to the same warp, which therefore never waits on a
        // slot whose earlier item another warp has yet to take.  Several windows: the windows of a unit
        // must meet in one warp's segment sums, so the first epilogue warp takes every item.
        const int which = warp - KW - 1;
        if (NW > 1 && which != 0) return;
        const int n = lane >> 2, rg = lane & 3;  // this lane: input row n, tile rows 4rg..4rg+3
        int ke = -1, kc = -1, pbase = 0, nvalid = 0;
        float fs = 1.f;     // 2^-e of input row n
        float rmax = 0.f;   // phase 1: running max |act| of input row n
        int rnext = 0;      // the ring slot of the next item and its phase
        uint32_t rphn = 0;
        auto flush = [&]() {
            float m = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 1));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
            if (rg == 0 && n < nvalid) atomicMax(&a.act_max[pbase + n], __float_as_uint(m));
            rmax = 0.f;
        };
        for (int64_t it = 0; it < n_items; ++it, cur.advance(pre, E, RTS, SEG, NW)) {
            const int r = rnext;
            const uint32_t rph = rphn;
            if (++rnext == NR) {
                rnext = 0;
                rphn ^= 1u;
            }
            if (NW == 1 && (int)(it & (kEpiWarps - 1)) != which) continue;
            if (cur.u.e != ke || cur.u.c != kc) {
                if (a.phase == 1 && ke >= 0) flush();
                ke = cur.u.e;
                kc = cur.u.c;
                pbase = off_s[ke] + 8 * kc;
                nvalid = min(8, cnt_s[ke] - 8 * kc);
                int ex = 0;
                if (n < nvalid) {
                    if (pbase + n < PC) ex = exp_s[pbase + n];
                    else if (a.phase == 1) ex = a.row_exp[a.sorted_rows[pbase + n]];
                    else ex = mb_row_exponent(__uint_as_float(a.act_max[pbase + n]));
                }
                fs = pow2f(-ex);
            }
            const bool ok = MB_DECODE_WAIT(&rfull[r], rph, a.status, abort_flag);
            const int nt = min(MT, RT - cur.u.sg * MT);
            if (ok) {
                const float* rr = red + r * red_buf;
                for (int mt = 0; mt < nt; ++mt) {
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
                    for (int w = 0; w < KW; ++w) {
                        const float4 u = *reinterpret_cast<const float4*>(rr + (w * MT + mt) * kRedTile + n * 16 + 4 * rg);
                        v.x += u.x;
                        v.y += u.y;
                        v.z += u.z;
                        v.w += u.w;
                    }
                    if (NW > 1) {   // the sums over earlier windows wait in shared memory
                        float4* sp = reinterpret_cast<float4*>(segsum + (cur.j * MT + mt) * kRedTile + n * 16 + 4 * rg);
                        if (cur.w > 0) {
                            const float4 q = *sp;
                            v.x += q.x;
                            v.y += q.y;
                            v.z += q.z;
                            v.w += q.w;
                        }
                        if (cur.w + 1 < NW) {
                            *sp = v;
                            continue;
                        }
                    }
                    const int rt = cur.u.sg * MT + mt;
                    if (a.phase == 1) {
                        // lanes rg 0,1 hold gate rows 4rg..4rg+3, lanes rg 2,3 the matching up rows
                        const float ux = __shfl_down_sync(0xffffffffu, v.x, 2), uy = __shfl_down_sync(0xffffffffu, v.y, 2);
                        const float uz = __shfl_down_sync(0xffffffffu, v.z, 2), uw = __shfl_down_sync(0xffffffffu, v.w, 2);
                        if (rg < 2 && n < nvalid) {
                            float4 o;
                            float gg;
                            gg = v.x * fs; o.x = __fdividef(gg, 1.0f + __expf(-gg)) * (ux * fs);
                            gg = v.y * fs; o.y = __fdividef(gg, 1.0f + __expf(-gg)) * (uy * fs);
                            gg = v.z * fs; o.z = __fdividef(gg, 1.0f + __expf(-gg)) * (uz * fs);
                            gg = v.w * fs; o.w = __fdividef(gg, 1.0f + __expf(-gg)) * (uw * fs);
                            *reinterpret_cast<float4*>(a.act + (int64_t)(pbase + n) * a.act_ld + 8 * rt + 4 * rg) = o;
                            rmax = fmaxf(rmax, fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w))));
                        }
                    } else if (n < nvalid) {
                        const int orow = 16 * rt + 4 * rg;
                        float* dst = a.y + (int64_t)(pbase + n) * a.y_ld + orow;
                        const float4 o = make_float4(v.x * fs, v.y * fs, v.z * fs, v.w * fs);
                        if (orow + 4 <= a.O_real) {
                            *reinterpret_cast<float4*>(dst) = o;
                        } else {
                            if (orow < a.O_real) dst[0] = o.x;
                            if (orow + 1 < a.O_real) dst[1] = o.y;
                            if (orow + 2 < a.O_real) dst[2] = o.z;
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mb_mbar_arrive(&rempty[r]);
        }
        if (a.phase == 1 && ke >= 0) flush();
        return;
    }

    // ------------------------------------------------------------- MMA warps
    // One mma.sync m16n8k16 covers 16 weight rows x 16 columns of a group x 8
    // N slots = 4 input rows x {hi, lo} piece.  N tile nt holds input rows
    // 4nt..4nt+3 of the chunk; the second N tile runs only for chunks of more
    // than 4 picks.  For group column c = 8t + j (j = 0..7), mma 0 takes
    // j in {0, 4 | 1, 5} and mma 1 takes j in {2, 6 | 3, 7} (K slots 2t, 2t+1 |
    // 2t+8, 2t+9), which is the order unpack_q4 / unpack_q8 produce.
    const int K = a.K;
    uint32_t bf[2][4][4];  // [N tile][group][mma 0 b0, b1, mma 1 b0, b1]
    float xs[2][4];        // affine format: group sums of input row 4nt + t (scaled like the pieces)
    int ke = -1, kc = -1, kw = -1;
    bool two = false, has = false;
    int s = 0, r = 0;
    uint32_t ph = 0, rph = 0;
    for (int64_t it = 0; it < n_items; ++it, cur.advance(pre, E, RTS, SEG, NW)) {
        if (cur.u.e != ke || cur.u.c != kc || cur.w != kw) {
            ke = cur.u.e;
            kc = cur.u.c;
            kw = cur.w;
            const int pbase = off_s[ke] + 8 * kc;
            const int nvalid = min(8, cnt_s[ke] - 8 * kc);
            const int qg = kw * QW + warp;   // this warp's quad of K
            two = nvalid > 4;
            has = qg < NQ;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                // this lane supplies N slot g: input row 4nt + (g >> 1), piece g & 1
                const int xr = 4 * nt + (g >> 1);
                const bool lo_piece = g & 1;
                const bool valid = xr < nvalid && has;
                const float* src = nullptr;
                float up = 1.0f;
                if (valid) {
                    int ex;
                    const int p = pbase + xr;
                    if (a.phase == 1) {
                        const int row = p < PC ? row_s[p] : a.sorted_rows[p];
                        src = a.x + (int64_t)row * a.src_ld;
                        ex = p < PC ? exp_s[p] : a.row_exp[row];
                    } else {
                        src = a.act + (int64_t)p * a.src_ld;
                        ex = p < PC ? exp_s[p] : mb_row_exponent(__uint_as_float(a.act_max[p]));
                    }
                    up = pow2f(ex);
                }
#pragma unroll
                for (int gi = 0; gi < 4; ++gi) {
                    float v[8];
                    const int col0 = (qg * 4 + gi) * 32 + 8 * t;
                    if (valid && col0 + 8 <= K) {
                        const float4 u0 = *reinterpret_cast<const float4*>(src + col0);
                        const float4 u1 = *reinterpret_cast<const float4*>(src + col0 + 4);
                        v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
                        v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
                    } else {
#pragma unroll
                        for (int j = 0; j < 8; ++j) v[j] = (valid && col0 + j < K) ? src[col0 + j] : 0.0f;
                    }
                    __half pc[8];
                    float sum = 0.0f;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float xsc = v[j] * up;
                        const __half h = __float2half_rn(xsc);
                        pc[j] = lo_piece ? __float2half_rn(xsc - __half2float(h)) : h;
                        sum += xsc;
                    }
                    bf[nt][gi][0] = mb_pack_h2(pc[0], pc[4]);
                    bf[nt][gi][1] = mb_pack_h2(pc[1], pc[5]);
                    bf[nt][gi][2] = mb_pack_h2(pc[2], pc[6]);
                    bf[nt][gi][3] = mb_pack_h2(pc[3], pc[7]);
                    if (AFF) {
                        // the 32-column group sum of input row xr (lanes t of this g hold its four 8-column
                        // parts), then lane (g, t) takes the sum of input row 4nt + t from lane 8t (g = 2t)
                        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                        xs[nt][gi] = __shfl_sync(0xffffffffu, sum, 8 * t);
                    }
                }
            }
        }

        const int ntiles = min(MT, RT - cur.u.sg * MT);
        if (it >= NR) MB_DECODE_WAIT(&rempty[r], rph ^ 1u, a.status, abort_flag);
        const bool ok = MB_DECODE_WAIT(&full[s], ph, a.status, abort_flag);
        float* rb = red + r * red_buf + warp * MT * kRedTile;
        if (ok && (Q8 || AFF || has)) {
            const uint8_t* stage = stages + (size_t)s * stage_bytes + warp * kBlock;
            if (two) {
                for (int mt = 0; mt < ntiles; ++mt)
                    tile_mma<Q8, F16S, AFF, true>(stage + mt * wt_bytes, has, bf, xs, rb + mt * kRedTile, t, g);
            } else {
                for (int mt = 0; mt < ntiles; ++mt)
                    tile_mma<Q8, F16S, AFF, false>(stage + mt * wt_bytes, has, bf, xs, rb + mt * kRedTile, t, g);
            }
        } else {   // a failed wait, or (plain int4) no quad of this warp in this K window: zero partials
            for (int mt = 0; mt < ntiles; ++mt) {
                float* rt = rb + mt * kRedTile;
                rt[t * 16 + g] = rt[t * 16 + g + 8] = rt[(4 + t) * 16 + g] = rt[(4 + t) * 16 + g + 8] = 0.f;
            }
        }
        __syncwarp();
        if (lane == 0) {
            mb_mbar_arrive(&empty[s]);
            mb_mbar_arrive(&rfull[r]);
        }
        if (++s == S) {
            s = 0;
            ph ^= 1u;
        }
        if (++r == NR) {
            r = 0;
            rph ^= 1u;
        }
    }
}

struct Cfg {
    int KW, NQ, QW, NW, SEG, MT, stages, tile_bytes, nred, pc;
    size_t smem;
};

// Stage = MT row tiles (of one K window) of ~32 KB; as many stages as fit in
// the shared memory of one CTA per SM (many MMA warps) or of two (few MMA
// warps: short K).  K above 2048 is cut into windows of 16 quads.
Cfg plan(int fmt, int K, int E, int RT, int P, int phase)
{
    Cfg c;
    const Fmt f = fmt_info(fmt);
    c.NQ = (K + 127) / 128;
    c.KW = c.NQ < kMaxKW ? c.NQ : kMaxKW;
    c.QW = c.KW;
    c.NW = (c.NQ + c.QW - 1) / c.QW;
    c.tile_bytes = c.NQ * f.block_bytes;
    const int wt = c.QW * f.block_bytes;
    // stages of ~48 KB (fewer hand-offs per byte), ~32 KB for a handful of picks, where more and
    // smaller units spread the little work there is over more SMs
    const int stage_kb = P <= MB_DECODE_SMALL_P ? MB_DECODE_STAGE_KB_SMALL : MB_DECODE_STAGE_KB;
    int mt0 = (stage_kb * 1024 + wt / 2) / wt;
    mt0 = mt0 < 1 ? 1 : (mt0 > kMaxMT ? kMaxMT : mt0);
    if (mt0 > RT) mt0 = RT < 1 ? 1 : RT;
    // reduction buffers: with many MMA warps each epilogue warp keeps two items in
    // hand (the MMA warps run further ahead); with few, shared memory goes to stages
    c.nred = (c.KW > 8 ? MB_DECODE_NRED : MB_DECODE_NRED_NARROW) * kEpiWarps;
    // one CTA per SM with many MMA warps, two with few (113 KB each leaves the per-CTA reserve)
    const size_t budget = c.KW <= 8 ? 113 * 1024 : 220 * 1024;
    const size_t cache = 2 * (size_t)(E + 1) * sizeof(int64_t) + (E <= kMaxCachedE ? (size_t)E * sizeof(void*) : 0) +
                         2 * (size_t)E * sizeof(int32_t);
    // the largest stage that leaves room for at least two of them
    for (c.MT = mt0;; --c.MT) {
        c.SEG = c.NW > 1 ? (kSegTiles / c.MT > 0 ? kSegTiles / c.MT : 1) : (1 << 30);
        const size_t red = (size_t)c.nred * c.KW * c.MT * kRedTile * sizeof(float);
        const size_t seg = c.NW > 1 ? (size_t)c.SEG * c.MT * kRedTile * sizeof(float) : 0;
        const size_t stage = (size_t)c.MT * wt;
        auto stages_for = [&](size_t fixed) {
            const int st = budget > fixed ? (int)((budget - fixed) / stage) : 2;
            return st < 2 ? 2 : (st > 8 ? 8 : st);
        };
        const size_t fixed = red + seg + cache + 64 + 16 * sizeof(uint64_t);
        // the picks' rows and exponents go to shared memory only where that costs no weight stage
        const size_t pcache = P <= kMaxCachedP ? (phase == 1 ? 2 : 1) * (size_t)P * sizeof(int32_t) : 0;
        c.stages = stages_for(fixed);
        c.pc = (pcache && stages_for(fixed + pcache) == c.stages) ? P : 0;
        c.smem = (size_t)c.stages * stage + red + seg + (size_t)(2 * c.stages + 2 * c.nred) * sizeof(uint64_t) +
                 cache + (c.pc ? pcache : 0) + 16;
        if (c.smem <= budget + 7 * 1024 || c.MT == 1) break;
    }
    return c;
}

template <int FMT>
int launch_phase(const DecodeArgs& base, int K, int RT, cudaStream_t st)
{
    DecodeArgs a = base;
    const Cfg c = plan(FMT, K, a.E, RT, a.P, a.phase);
    if (c.smem > 227 * 1024)
        return mb_fail(MB_EUNSUPPORTED, "mb_moe_decode: %d experts leave no room for two weight stages", a.E);
    a.K = K;
    a.NQ = c.NQ;
    a.QW = c.QW;
    a.NW = c.NW;
    a.SEG = c.SEG;
    a.RT = RT;
    a.MT = c.MT;
    a.KW = c.KW;
    a.stages = c.stages;
    a.tile_bytes = c.tile_bytes;
    a.nred = c.nred;
    a.PC = c.pc;
    auto kern = moe_decode_kernel<FMT>;
    const int threads = (c.KW + 1 + kEpiWarps) * 32;
    // one-time per (device, kernel, configuration): raise the shared-memory
    // limit and look up the occupancy, so later calls (and graph captures) only
    // enqueue work
    struct Occ {
        int dev, threads;
        size_t smem;
        int per_sm;
    };
    static thread_local Occ cache[16];
    static thread_local int ncache = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    int per_sm = -1;
    for (int i = 0; i < ncache; ++i)
        if (cache[i].dev == dev && cache[i].threads == threads && cache[i].smem == c.smem) per_sm = cache[i].per_sm;
    // the shared-memory limit is an attribute of the kernel, shared by every
    // configuration that launches it: only ever raise it
    static thread_local size_t smem_attr[64] = {0};
    const int di = dev & 63;
    if (smem_attr[di] < c.smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c.smem);
        if (e != cudaSuccess) {
            (void)cudaGetLastError();
            return mb_fail(MB_ECUDA, "mb_moe_decode: smem attribute: %s", cudaGetErrorString(e));
        }
        smem_attr[di] = c.smem;
    }
    if (per_sm < 0) {
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, c.smem);
        if (e != cudaSuccess) (void)cudaGetLastError();
        if (e != cudaSuccess || per_sm < 1) per_sm = 1;
        if (ncache < 16) cache[ncache++] = Occ{dev, threads, c.smem, per_sm};
    }
    const int grid = mb_num_sms() * per_sm;
    const cudaError_t le = mb_launch_pdl(kern, dim3(grid), dim3(threads), c.smem, st, a);
    if (le != cudaSuccess) return mb_fail(MB_ECUDA, "mb_moe_decode launch: %s", cudaGetErrorString(le));
    return MB_OK;
}

template <typename F>
int dispatch_fmt(int fmt, F&& f)
{
    switch (fmt) {
    case MB_FMT_Q4_F32: return f(std::integral_constant<int, MB_FMT_Q4_F32>());
    case MB_FMT_Q4_F16: return f(std::integral_constant<int, MB_FMT_Q4_F16>());
    case MB_FMT_Q8_F32: return f(std::integral_constant<int, MB_FMT_Q8_F32>());
    case MB_FMT_Q8_F16: return f(std::integral_constant<int, MB_FMT_Q8_F16>());
    case MB_FMT_Q4K_F32: return f(std::integral_constant<int, MB_FMT_Q4K_F32>());
    default: return mb_fail(MB_EUNSUPPORTED, "mb_moe_decode: weight format %d", fmt);
    }
}

// Clears each pick's max |act| word before the gate|up phase, as one more kernel in the programmatic launch
// chain (a memset node would break it): it is placed while the kernel before it drains, waits on it (the
// last reader of these words, a previous call's down phase, is complete by then), clears, and lets the
// gate|up phase launch.
__global__ void clear_words_kernel(unsigned* __restrict__ words, int64_t n)
{
    mb_pdl_wait();
    mb_pdl_trigger();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        words[i] = 0u;
}

__global__ void row_absmax_bits_kernel(const float* __restrict__ x, int64_t n, int K, unsigned* __restrict__ out)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    if (r >= n) return;
    float m = 0.0f;
    for (int h = lane; h < K; h += 32) m = fmaxf(m, fabsf(x[r * K + h]));
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) out[r] = __float_as_uint(m);
}

}  // namespace

// Workspace of mb_matmul_t: the rows' max |x| (n u32) | a status word.
extern "C" int64_t mb_matmul_t_workspace_bytes(int64_t n) { return ((n * 4 + 255) / 256) * 256 + 256; }

// x @ W.T for one packed matrix W (O x K) in the tile layout:
// moelan/kernels.py:1018 q4_matmul_t and :1030 q8_matmul_t (also GGUF Q8_0 via
// its int8 tiles, kernels.py:981).  x (n, K) f32, y (n, O) f32.
extern "C" int mb_matmul_t(const void* w_tiles, int fmt, int O, int K, const float* x, int64_t n, float* y,
                           void* workspace, int64_t workspace_bytes, unsigned* status, void* stream)
{
    MB_REQUIRE(w_tiles && x && y && workspace, "mb_matmul_t: null pointer");
    MB_REQUIRE(O > 0 && K > 0 && n >= 0 && n < (1 << 30), "mb_matmul_t: bad sizes");
    MB_REQUIRE(K % 4 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)w_tiles & 15) == 0 &&
                   ((uintptr_t)workspace & 255) == 0,
               "mb_matmul_t: K must be a multiple of 4, x/W 16-byte and workspace 256-byte aligned");
    MB_REQUIRE(workspace_bytes >= mb_matmul_t_workspace_bytes(n), "mb_matmul_t: workspace too small");
    if (n == 0) return MB_OK;
    cudaStream_t st = mb_stream(stream);
    unsigned* amax = reinterpret_cast<unsigned*>(workspace);
    unsigned* ws_status = reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(workspace) + ((n * 4 + 255) / 256) * 256);
    row_absmax_bits_kernel<<<(unsigned)((n + 7) / 8), 256, 0, st>>>(x, n, K, amax);
    int rc = mb_check_launch("mb_matmul_t");
    if (rc) return rc;
    DecodeArgs a{};
    a.E = 1;
    a.phase = 2;
    a.O_real = O;
    a.src_ld = K;
    a.y_ld = O;
    a.act = const_cast<float*>(x);
    a.act_max = amax;
    a.y = y;
    a.max_rows = 1 << 30;
    a.status = status ? status : ws_status;
    a.single_w = w_tiles;
    a.single_n = (int)n;
    a.P = (int)n;
    return dispatch_fmt(fmt, [&](auto f) { return launch_phase<decltype(f)::value>(a, K, (O + 15) / 16, st); });
}

// Workspace: act (P x I_pad f32) | act_max (P u32) | a status word.
extern "C" int64_t mb_moe_decode_workspace_bytes(int64_t P, int I)
{
    const int64_t I_pad = (I + 127) / 128 * 128;
    return ((P * I_pad * 4 + 255) / 256) * 256 + ((P * 4 + 255) / 256) * 256 + 256;
}

extern "C" int mb_moe_decode(const MbExpert* table, int E, int H, int I, int gs, int fmt_gu, int fmt_down,
                             const float* x, const int32_t* row_exp, int64_t T, const int32_t* counts,
                             const int32_t* offsets, const int32_t* sorted_rows, int64_t P, int max_rows, float* y,
                             void* workspace, int64_t workspace_bytes, unsigned* status, void* stream)
{
    MB_REQUIRE(table && x && row_exp && counts && offsets && sorted_rows && y, "mb_moe_decode: null pointer");
    MB_REQUIRE(E > 0 && E <= 4096 && H > 0 && I > 0 && T >= 0 && P >= 0, "mb_moe_decode: bad sizes");
    MB_REQUIRE(gs % 32 == 0 && H % gs == 0 && I % gs == 0, "mb_moe_decode: group size %d must be a multiple of 32 "
               "dividing H=%d and I=%d", gs, H, I);
    MB_REQUIRE(H % 4 == 0, "mb_moe_decode: H must be a multiple of 4");
    MB_REQUIRE(((uintptr_t)x & 15) == 0 && ((uintptr_t)workspace & 255) == 0,
               "mb_moe_decode: x must be 16-byte and workspace 256-byte aligned");
    MB_REQUIRE(workspace_bytes >= mb_moe_decode_workspace_bytes(P, I), "mb_moe_decode: workspace too small");
    if (P == 0) return MB_OK;
    if (max_rows <= 0) max_rows = 1 << 30;
    const int I_pad = (I + 127) / 128 * 128;
    const int I8 = (I + 7) / 8 * 8;
    cudaStream_t st = mb_stream(stream);
    float* act = reinterpret_cast<float*>(workspace);
    unsigned* act_max = reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(workspace) +
                                                    ((P * I_pad * 4 + 255) / 256) * 256);
    unsigned* ws_status = reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(act_max) + ((P * 4 + 255) / 256) * 256);
    const unsigned nclr = (unsigned)std::min<int64_t>((P + 255) / 256, 148);
    cudaError_t e = mb_launch_pdl(clear_words_kernel, dim3(nclr), dim3(256), 0, st, act_max, P);
    if (e != cudaSuccess) return mb_fail(MB_ECUDA, "mb_moe_decode: %s", cudaGetErrorString(e));

    DecodeArgs a{};
    a.table = table;
    a.E = E;
    a.counts = counts;
    a.offsets = offsets;
    a.sorted_rows = sorted_rows;
    a.x = x;
    a.row_exp = row_exp;
    a.act = act;
    a.act_max = act_max;
    a.y = y;
    a.max_rows = max_rows;
    a.P = (int)P;
    a.status = status;
    a.act_ld = I_pad;
    a.y_ld = H;
    if (!a.status) a.status = ws_status;  // caller did not ask to see it

    int rc;
    a.phase = 1;
    a.O_real = I;
    a.src_ld = H;
    rc = dispatch_fmt(fmt_gu, [&](auto f) { return launch_phase<decltype(f)::value>(a, H, I8 / 8, st); });
    if (rc) return rc;
    a.phase = 2;
    a.O_real = H;
    a.src_ld = I_pad;
    rc = dispatch_fmt(fmt_down, [&](auto f) { return launch_phase<decltype(f)::value>(a, I, (H + 15) / 16, st); });
    return rc;
}

// ---- the decode without a caller workspace -----------------------------------
// Some callers cannot hand the library a workspace: bindings that only forward
// pointers they were given and have no device allocator of their own, or code
// running where allocating device memory is not allowed or would fragment a
// pool it does not own.  For them the decode's scratch (activations, each
// pick's max |act|, a status word) lives in this array, built into the
// library: every GPU that loads the library holds MB_NOALLOC_SCRATCH_BYTES of
// it until the process exits.  All calls share it and it keeps the last
// call's contents; what must start at zero (the max |act| words) is cleared by
// every call on the stream before use.
static __device__ __align__(256) uint8_t g_moe_decode_scratch[MB_NOALLOC_SCRATCH_BYTES];

#include <mutex>

// The array's device address for the current device, looked up once per device
// (host code may not use the symbol itself as a device address).
static int noalloc_scratch(void** out)
{
    static std::mutex mu;
    static void* addr[64] = {nullptr};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return mb_fail(MB_ECUDA, "mb_moe_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return mb_fail(MB_EUNSUPPORTED, "mb_moe_decode_noalloc: device %d", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_moe_decode_scratch);
        if (e != cudaSuccess || !p)
            return mb_fail(MB_ECUDA, "mb_moe_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        addr[dev] = p;
    }
    *out = addr[dev];
    return MB_OK;
}

extern "C" int mb_moe_decode_noalloc(const MbExpert* table, int E, int H, int I, int gs, int fmt_gu, int fmt_down,
                                     const float* x, const int32_t* row_exp, int64_t T, const int32_t* counts,
                                     const int32_t* offsets, const int32_t* sorted_rows, int64_t P, int max_rows,
                                     float* y, unsigned* status, void* stream)
{
    MB_REQUIRE(P >= 0 && I > 0, "mb_moe_decode_noalloc: bad sizes");
    const int64_t need = mb_moe_decode_workspace_bytes(P, I);
    if (need > (int64_t)MB_NOALLOC_SCRATCH_BYTES)
        return mb_fail(MB_EINVAL,
                       "mb_moe_decode_noalloc: %lld picks with I=%d need %lld bytes of scratch, more than the %lld "
                       "built into the library; use mb_moe_decode with a workspace",
                       (long long)P, I, (long long)need, (long long)MB_NOALLOC_SCRATCH_BYTES);
    void* ws = nullptr;
    const int rc = noalloc_scratch(&ws);
    if (rc) return rc;
    return mb_moe_decode(table, E, H, I, gs, fmt_gu, fmt_down, x, row_exp, T, counts, offsets, sorted_rows, P,
                         max_rows, y, ws, (int64_t)MB_NOALLOC_SCRATCH_BYTES, status, stream);
}
