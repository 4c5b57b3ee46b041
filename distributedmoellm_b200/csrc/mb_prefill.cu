// Prefill: the routed experts as grouped GEMMs on the 5th-generation tensor
// cores (tcgen05), for experts picked by many tokens.
//
// Reference: moelan/experts.py:148-151, 216-219 (GroupQuant / Packed4
// matmul_t with 8 or more rows: widen the matrix to f32, then BLAS x @ W.T),
// run per expert by ExpertStore.compute (experts.py:707-727).
//
// Two launches per layer (gate|up -> activations, down -> y) of one
// persistent, warp-specialised kernel: one CTA per SM walks work items
// (expert, pass of at most 160 of its picks, block of 128 weight rows), dealt
// round-robin over the CTAs, with
//  * a weight producer warp: the packed tiles (the same HBM tile layout the
//    decode kernels read) in 1-D bulk copies into a shared-memory ring;
//  * a token producer warp: the expert's tokens, gathered once per layer
//    into an f16 matrix in pick order, as 2-D TMA boxes (128-byte swizzle,
//    K-major) into a second ring;
//  * eight dequant warps: (q - offset) * group scale * 2^w in packed f16x2
//    arithmetic (exact until the one rounding of the product), written with
//    tcgen05.st straight into tensor memory, where tcgen05.mma reads its A
//    operand (the converted weights never pass through shared memory);
//  * one MMA thread: tcgen05.mma M=128, N <= 160 tokens, K=16, f32
//    accumulators in TMEM, two accumulator buffers;
//  * four epilogue warps: tcgen05.ld, undo the power-of-two scalings, form
//    SiLU(gate) * up (written as f16 for the down GEMM) or the f32 output
//    rows, overlapped with the next item's main loop.
// Every wait is bounded (status word + abort flag); TMEM is freed on exit.
//
// Range scaling (all by powers of two, so exact): a token row is multiplied
// by 2^row_exp (its largest value in [2^13, 2^14)); a weight matrix by
// 2^w_exp (its largest possible value in [2^13, 2^14)); a pick's activation
// row by 2^(a_exp + 2 row_exp), where a_exp comes from the bound
// |SiLU(g) u| <= max|x|^2 * max_j |Wg_j|_1 * max_j |Wu_j|_1, keeping it
// below 2^15.  f16 rather than bf16 operands: the same tensor-core rate and
// 3 more mantissa bits; results agree with the f32 reference within 2e-3 of
// each row's max (bf16 operands would give ~7e-3).
//
// K order: within every 8 columns the f16 operands hold the columns in the
// order 0 4 1 5 2 6 3 7 (both A and B, so the products are unchanged); it is
// the order in which the packed nibbles / bytes unpack into f16 pairs.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "mb_common.cuh"

namespace {

constexpr int kBM = 128;       // weight rows per item = TMEM lanes
// The K loop runs in quads of 128 columns (two 64-column halves, each one
// 128-byte swizzle atom of f16), the unit of every hand-off.
constexpr int kMaxN = 160;     // tokens per pass
constexpr int kBStages = 3;    // token (B) quad stages: [2 halves][kMaxN rows][128 B] = 40 KB each
// Packed-weight stages, one quad of 8 row tiles each.  Even, so that every stage is always consumed by the
// same dequant set (sets alternate quads): a set then waits on a stage's next phase only after it consumed
// the previous one, which keeps the mbarrier parity waits unambiguous.
constexpr int pstages(bool) { return 4; }
static_assert(pstages(false) % 2 == 0 && pstages(true) % 2 == 0, "weight stages must be even");
constexpr int kMaxMetaE = 512; // experts whose (count, offset, exponents) a CTA keeps in shared memory
constexpr int kASlots = 3;     // A (dequantised quad) slots in TMEM, 64 columns each: quad gq uses slot gq % 3
constexpr int kAccCol = kASlots * 64;
constexpr int kTmemCols = 512;
static_assert(kAccCol + 2 * kMaxN <= kTmemCols, "TMEM columns");
constexpr int kDqWarps = 8;    // warps 4..11: two sets of four (one per TMEM lane quarter), alternate quads
constexpr int kEpiWarps = 4;   // warps 12..15
constexpr int kThreads = 512;
static_assert(kMaxMetaE <= kThreads && kThreads <= 32 * 32, "one expert per thread in the item scan");
constexpr int kBHalf = kMaxN * 128;   // bytes of one half (64 columns) of a token stage
// Token tiles: one TMA box per 64-column half, from the tensor map whose box is the pass's token count
// rounded up to kBoxStep rows (one instruction per half instead of one per 32 rows; a box never
// overruns the kMaxN-row stage).
constexpr int kBoxStep = 32;
constexpr int kNumBoxMaps = kMaxN / kBoxStep;   // box heights 32, 64, ..., kMaxN
static_assert(kMaxN % kBoxStep == 0 && kBHalf % 1024 == 0, "token stage layout");

struct TokenMaps {
    CUtensorMap m[kNumBoxMaps];   // m[i]: boxes of 64 columns x (i + 1) * kBoxStep rows
};

struct PrefillArgs {
    const MbExpert* table;
    const int32_t* e_exp;      // (E, 4): gate|up weight exponent, down weight exponent, activation exponent base
    int E;
    int phase;                 // 1: gate|up -> act (f16), 2: down -> y (f32)
    int NQ;                    // quads of K in the weight tiles (ceil(K / 128))
    int KH;                    // 64-column halves of K (K / 64)
    int RT;                    // row tiles of the matrix
    int MB;                    // M blocks (8 row tiles) per expert
    int block_bytes;
    int max_items;             // an upper bound of the launch's items (sizes the grid)
    const int32_t* counts;
    const int32_t* offsets;
    const int32_t* sorted_rows;   // the token row of each pick, or null: pick p is row p
    const int32_t* row_exp;    // exponents of the rows of x
    int min_rows;
    int O_real;                // phase 1: I (act columns); phase 2: H (y columns)
    __half* act;               // phase 1 output (P, I), K-permuted
    float* y;                  // phase 2 output (P, H)
    // phase 2 output rows elsewhere (expert parallelism): pick p's row goes to
    // y_peers[y_ret[p] >> 24] + (y_ret[p] & 0xffffff) * H instead of y + p * H
    // (an address outside n_peers buffers of peer_rows rows is reported and skipped)
    const int32_t* y_ret;
    float* const* y_peers;
    int n_peers;
    int64_t peer_rows;
    unsigned* status;
    // precise gate|up (affine int4): the weights' f16 rounding (piece 0) or its f16 residual (piece 1), and
    // the gate and up pre-activations written (accumulate 0) or added (1) to pre (P, 2I) f32 instead of act
    int piece;
    float* pre;
    int accumulate;
};

// ---- tcgen05 / TMA helpers -------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(mb_smem_addr(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t cols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem] (kind::f16: f16 inputs, f32 accumulate) and its commit, issued by one
// elected lane of a converged warp (the whole warp runs the MMA loop, so descriptors and addresses stay
// warp-uniform).
__device__ __forceinline__ void tc_mma_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\telect.sync r|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit_elect(uint64_t* bar)
{
    asm volatile(
        "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\telect.sync r|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(mb_smem_addr(bar))
        : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane (no wait).
__device__ __forceinline__ void tmem_st32_nowait(uint32_t taddr, const uint32_t (&v)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]),
        "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]),
        "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
        "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 2-D TMA tile load into shared memory, completing bytes on bar.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            mb_smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(mb_smem_addr(bar))
        : "memory");
}

// Shared-memory descriptor of a K-major 16-bit tile with 128-byte swizzle:
// rows 128 bytes apart, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    return (uint64_t)((saddr & 0x3FFFF) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: kind::f16 with A and B f16 (both K-major), D f32, M=128, N=n.
__device__ __forceinline__ uint32_t idesc_f16(int n)
{
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

// The static sequence of work items every role of a CTA walks: items
// blockIdx.x, blockIdx.x + gridDim.x, ... of all (expert, pass of at most kMaxN
// picks, M block) of the experts in this launch, expert-major, then pass, then
// M block (so items that run at the same time share their token rows).  One
// item is one pass; an expert with many picks spreads its passes over many CTAs.
// meta[e] = (picks, first pick, this launch's weight exponent, activation exponent base) and
// pstart[e] = the first item of expert e (pstart[E] = all items), in shared memory once per CTA.
struct Items {
    const PrefillArgs& a;
    const int4* meta;
    const int* pstart;
    int it;
    int e, mb, n_e, off_e, passes, pass0, wexp, aexp;
    __device__ Items(const PrefillArgs& args, const int4* m, const int* ps)
        : a(args), meta(m), pstart(ps), it((int)blockIdx.x - (int)gridDim.x), e(0) {}
    __device__ bool next()
    {
        it += gridDim.x;
        if (it >= pstart[a.E]) return false;
        while (pstart[e + 1] <= it) ++e;   // items only move forward: the expert whose items hold it
        const int local = it - pstart[e];
        pass0 = local / a.MB;
        mb = local - pass0 * a.MB;
        const int4 m = meta[e];
        n_e = m.x;
        off_e = m.y;
        wexp = m.z;
        aexp = m.w;
        passes = 1;
        return true;
    }
};

// An f16 pair of exact small integers times the group scale (one rounding).
// For the affine int4 format q * scale + bias is formed in f32 and rounded to
// f16 once: a scale and bias rounded to f16 first would put the same error
// on all 32 weights of a group.
template <bool AFF>
__device__ __forceinline__ uint32_t scale_pair(uint32_t q, uint32_t s, float sf, float bf, int piece)
{
    if (AFF) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q));
        const float w0 = fmaf(f.x, sf, bf), w1 = fmaf(f.y, sf, bf);
        if (piece) {            // the residual w - f16(w), exact in f32, rounded to f16
            const float2 h = __half22float2(__floats2half2_rn(w0, w1));
            return pack_f16(w0 - h.x, w1 - h.y);
        }
        return pack_f16(w0, w1);
    }
    return mb_hmul2(q, s);
}

// v[t] = the loaded v[(t - rot) & 3]: undoes a load order rotated by rot.
__device__ __forceinline__ void rotate_back(uint4 (&v)[4], int rot)
{
    const bool r1 = rot & 1, r2 = rot & 2;
    uint4 u[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) u[t] = r1 ? v[(t + 3) & 3] : v[t];
#pragma unroll
    for (int t = 0; t < 4; ++t) v[t] = r2 ? u[(t + 2) & 3] : u[t];
}

// v[k] = p[2k + odd], k < 8, from 16 floats of shared memory (16-byte aligned) in four vector reads.
__device__ __forceinline__ void load_alt8(const float* p, bool odd, float (&v)[8])
{
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const float4 t = *reinterpret_cast<const float4*>(p + 4 * c);
        v[2 * c] = odd ? t.y : t.x;
        v[2 * c + 1] = odd ? t.w : t.z;
    }
}

// ---- the GEMM kernel ----------------------------------------------------------------

template <int FMT>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ PrefillArgs a, const __grid_constant__ TokenMaps bmaps)
{
    constexpr bool Q8 = (FMT == MB_FMT_Q8_F16 || FMT == MB_FMT_Q8_F32);
    constexpr bool F16S = (FMT == MB_FMT_Q4_F16 || FMT == MB_FMT_Q8_F16);
    constexpr bool AFF = (FMT == MB_FMT_Q4K_F32);   // int4 with a per-group bias after the scales
    constexpr int kData = Q8 ? 2048 : 1024;
    constexpr int kPStages = pstages(Q8);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* bst = smem;                                       // [kBStages][2 halves][kMaxN][128 B]
    uint8_t* pst = bst + kBStages * 2 * kBHalf;                // [kPStages][8 tiles][block]
    float* tok_s = reinterpret_cast<float*>(pst + kPStages * 8 * a.block_bytes);   // [2][kMaxN] row scale
    float* tok_a = tok_s + 2 * kMaxN;                          // [2][kMaxN] activation scale (phase 1)
    float** tok_y = reinterpret_cast<float**>(tok_a + 2 * kMaxN);   // [2][kMaxN] output row (phase 2)
    uint64_t* bars = reinterpret_cast<uint64_t*>(tok_y + 2 * kMaxN);
    uint64_t* b_full = bars;                                   // [kBStages]
    uint64_t* b_empty = b_full + kBStages;
    uint64_t* p_full = b_empty + kBStages;                     // [kPStages]
    uint64_t* p_empty = p_full + kPStages;
    uint64_t* a_full = p_empty + kPStages;                     // [kASlots]
    uint64_t* a_empty = a_full + kASlots;
    uint64_t* acc_full = a_empty + kASlots;                    // [2]
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int4* meta = reinterpret_cast<int4*>(tmem_slot + 4);       // [E]
    int* pstart = reinterpret_cast<int*>(meta + a.E);          // [E + 1]
    int* wsum = pstart + a.E + 1;                              // [16] scan of the warps' item counts

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < a.E; e += kThreads) {
        const int* ee = a.e_exp + 4 * e;
        meta[e] = make_int4(a.counts[e], a.offsets[e], ee[a.phase == 1 ? 0 : 1], ee[2]);
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < kBStages; ++i) {
            mb_mbar_init(&b_full[i], 1);
            mb_mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < kPStages; ++i) {
            mb_mbar_init(&p_full[i], 1);
            mb_mbar_init(&p_empty[i], 4);
        }
        for (int i = 0; i < kASlots; ++i) {
            mb_mbar_init(&a_full[i], 4);
            mb_mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mb_mbar_init(&acc_full[i], 1);
            mb_mbar_init(&acc_empty[i], kEpiWarps);
        }
        *abort_flag = 0;
        mb_fence_mbar_init();
    }
    if (warp == 2) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    {
        // pstart: exclusive scan of the experts' item counts (MB items per pass of at most kMaxN picks) over
        // the block, one expert per thread (E <= kMaxMetaE == kThreads)
        int v = 0;
        if ((int)threadIdx.x < a.E) {
            const int n = meta[threadIdx.x].x;
            v = (n >= a.min_rows && n > 0) ? a.MB * ((n + kMaxN - 1) / kMaxN) : 0;
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += t;
        }
        if (lane == 31) wsum[warp] = v;
        __syncthreads();
        if (warp == 0) {
            int s = lane < kThreads / 32 ? wsum[lane] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += t;
            }
            if (lane < kThreads / 32) wsum[lane] = s;
        }
        __syncthreads();
        if ((int)threadIdx.x < a.E) pstart[threadIdx.x + 1] = v + (warp > 0 ? wsum[warp - 1] : 0);
        if (threadIdx.x == 0) pstart[0] = 0;
        __syncthreads();
    }
    const uint32_t tmem = *tmem_slot;
    const int KH = a.KH;
    const int quads = (KH + 1) >> 1;   // quads per pass; the last one has one half when KH is odd

    // Every role counts quads gq over all its items and passes: weight stage gq % kPStages, A slot
    // gq % kASlots, token stage gq % kBStages, dequant set gq % 2.
    if (warp == 0) {
        // ------------------------------------------------------------ weight producer
        {
            Items w(a, meta, pstart);
            int gq = 0;
            bool ok = true;
            while (ok && w.next() && !*abort_flag) {
                const int tiles = min(8, a.RT - w.mb * 8);
                const uint8_t* wbase =
                    reinterpret_cast<const uint8_t*>(a.phase == 1 ? a.table[w.e].gu : a.table[w.e].down);
                for (int pass = 0; ok && pass < w.passes; ++pass) {
                    for (int qd = 0; qd < quads; ++qd, ++gq) {
                        const int ps = (int)(gq % kPStages);
                        if (gq >= kPStages)
                            ok = __all_sync(0xffffffffu, mb_mbar_wait_spin(&p_empty[ps], (uint32_t)(((gq / kPStages) - 1) & 1),
                                                                          a.status, abort_flag));
                        if (!ok) break;
                        if (lane == 0) mb_mbar_arrive_expect_tx(&p_full[ps], (uint32_t)(tiles * a.block_bytes));
                        __syncwarp();
                        if (lane < tiles)   // one lane per row tile: the copies are issued in parallel
                            mb_bulk_g2s(pst + ((size_t)ps * 8 + lane) * a.block_bytes,
                                        wbase + ((size_t)(w.mb * 8 + lane) * a.NQ + qd) * a.block_bytes,
                                        (uint32_t)a.block_bytes, &p_full[ps]);
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ token producer
        {
            Items w(a, meta, pstart);
            int gq = 0;
            bool ok = true;
            while (ok && w.next() && !*abort_flag) {
                for (int pass = 0; ok && pass < w.passes; ++pass) {
                    const int n0 = (w.pass0 + pass) * kMaxN;
                    const int nrows = min(kMaxN, w.n_e - n0);
                    const int nbox = (((nrows + 15) & ~15) + kBoxStep - 1) / kBoxStep;   // box height / kBoxStep
                    const CUtensorMap* bmap = &bmaps.m[nbox - 1];
                    for (int qd = 0; qd < quads; ++qd, ++gq) {
                        const int bs = (int)(gq % kBStages);
                        const int nh = min(2, KH - 2 * qd);
                        if (gq >= kBStages)
                            ok = __all_sync(0xffffffffu, mb_mbar_wait_spin(&b_empty[bs], (uint32_t)(((gq / kBStages) - 1) & 1),
                                                                          a.status, abort_flag));
                        if (!ok) break;
                        if (lane == 0) mb_mbar_arrive_expect_tx(&b_full[bs], (uint32_t)(nh * nbox * kBoxStep * 128));
                        __syncwarp();
                        if (lane < nh)   // one lane per 64-column half
                            tma_load_2d(bst + (size_t)(bs * 2 + lane) * kMaxN * 128, bmap, qd * 128 + lane * 64,
                                        w.off_e + n0, &b_full[bs]);
                    }
                }
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ MMA issuer (whole warp, one lane issues)
        Items w(a, meta, pstart);
        int gq = 0;
        int64_t np = 0;   // passes issued (accumulator buffer np & 1)
        bool ok = true;
        while (ok && w.next()) {
            for (int pass = 0; ok && pass < w.passes; ++pass, ++np) {
                const int nrows = min(kMaxN, w.n_e - (w.pass0 + pass) * kMaxN);
                const uint32_t idesc = idesc_f16((nrows + 15) & ~15);
                const int slot = (int)(np & 1);
                if (np >= 2)
                    ok = __all_sync(0xffffffffu, mb_mbar_wait_spin(&acc_empty[slot], (uint32_t)(((np >> 1) - 1) & 1),
                                                                    a.status, abort_flag));
                tc_fence_after();
                const uint32_t dcol = tmem + kAccCol + slot * kMaxN;
                for (int qd = 0; ok && qd < quads; ++qd, ++gq) {
                    const int as = gq % kASlots, bs = gq % kBStages;
                    const int nh = min(2, KH - 2 * qd);
                    ok = __all_sync(0xffffffffu,
                                    mb_mbar_wait_spin(&a_full[as], (uint32_t)((gq / kASlots) & 1), a.status, abort_flag) &&
                                        mb_mbar_wait_spin(&b_full[bs], (uint32_t)((gq / kBStages) & 1), a.status,
                                                          abort_flag));
                    if (!ok) break;
                    tc_fence_after();
                    for (int hh = 0; hh < nh; ++hh) {
                        const uint32_t bbase = mb_smem_addr(bst + (size_t)(bs * 2 + hh) * kBHalf);
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            tc_mma_ts_elect(dcol, tmem + as * 64 + hh * 32 + j * 8, sw128_desc(bbase + j * 32),
                                            idesc, (qd > 0 || hh > 0 || j > 0) ? 1u : 0u);
                    }
                    tc_commit_elect(&a_empty[as]);
                    tc_commit_elect(&b_empty[bs]);
                }
                tc_commit_elect(&acc_full[slot]);
            }
        }
    } else if (warp >= 4 && warp < 4 + kDqWarps) {
        // ------------------------------------------------------------ dequant (two sets, alternate quads)
        const int q = warp & 3;               // TMEM lane quarter this warp may access
        const int set = (warp - 4) >> 2;      // this set takes the quads gq with gq % 2 == set
        const int L = 32 * q + lane;          // TMEM lane = row of the M block
        int ti, trow;                         // source row tile within the M block, row within it
        if (a.phase == 1) {                   // lanes 32q + s: gate row, 32q + 16 + s: the matching up row
            const int s = lane & 15;
            ti = 2 * q + (s >> 3);
            trow = (s & 7) + ((lane >= 16) ? 8 : 0);
        } else {
            ti = L >> 4;
            trow = L & 15;
        }
        const uint32_t taddr0 = tmem + ((uint32_t)(32 * q) << 16);
        Items w(a, meta, pstart);
        int gq = 0;
        while (w.next()) {
            const int tiles = min(8, a.RT - w.mb * 8);
            const bool row_ok = ti < tiles;
            const float wscale = pow2i(clamp120(w.wexp));
            for (int pass = 0; pass < w.passes; ++pass) {
                for (int qd = 0; qd < quads; ++qd, ++gq) {
                    if ((int)(gq & 1) != set) continue;
                    const int ps = (int)(gq % kPStages);
                    const int nh = min(2, KH - 2 * qd);
                    const int as = gq % kASlots, use = gq / kASlots;   // A slot and its uses so far
                    const uint32_t taddr = taddr0 + as * 64;
                    bool ok = mb_mbar_wait_spin(&p_full[ps], (uint32_t)((gq / kPStages) & 1), a.status, abort_flag);
                    if (use >= 1)
                        ok = mb_mbar_wait_spin(&a_empty[as], (uint32_t)((use - 1) & 1), a.status, abort_flag) && ok;
                    tc_fence_after();
                    const uint8_t* blk = pst + ((size_t)ps * 8 + (row_ok ? ti : 0)) * a.block_bytes;
                    // the quad's four group scales, times 2^wexp, as f16x2 pairs (s, s)
                    uint32_t s2[4];
                    if (F16S) {
                        const uint2 sv = *reinterpret_cast<const uint2*>(blk + kData + trow * 8);
                        const __half2 h01 = *reinterpret_cast<const __half2*>(&sv.x);
                        const __half2 h23 = *reinterpret_cast<const __half2*>(&sv.y);
                        s2[0] = pack_f16(__low2float(h01) * wscale, __low2float(h01) * wscale);
                        s2[1] = pack_f16(__high2float(h01) * wscale, __high2float(h01) * wscale);
                        s2[2] = pack_f16(__low2float(h23) * wscale, __low2float(h23) * wscale);
                        s2[3] = pack_f16(__high2float(h23) * wscale, __high2float(h23) * wscale);
                    } else {
                        const float4 sv = *reinterpret_cast<const float4*>(blk + kData + trow * 16);
                        s2[0] = pack_f16(sv.x * wscale, sv.x * wscale);
                        s2[1] = pack_f16(sv.y * wscale, sv.y * wscale);
                        s2[2] = pack_f16(sv.z * wscale, sv.z * wscale);
                        s2[3] = pack_f16(sv.w * wscale, sv.w * wscale);
                    }
                    // affine int4: the scales and biases in f32, times 2^wexp (exact)
                    float sfl[4] = {0.f, 0.f, 0.f, 0.f}, bfl[4] = {0.f, 0.f, 0.f, 0.f};
                    if (AFF && ok && row_ok) {
                        const float4 sv = *reinterpret_cast<const float4*>(blk + kData + trow * 16);
                        const float4 bv = *reinterpret_cast<const float4*>(blk + kData + 256 + trow * 16);
                        sfl[0] = sv.x * wscale, sfl[1] = sv.y * wscale, sfl[2] = sv.z * wscale, sfl[3] = sv.w * wscale;
                        bfl[0] = bv.x * wscale, bfl[1] = bv.y * wscale, bfl[2] = bv.z * wscale, bfl[3] = bv.w * wscale;
                    }
                    if (!ok || !row_ok) s2[0] = s2[1] = s2[2] = s2[3] = 0u;
                    // half hh covers groups 2hh, 2hh+1; TMEM column 32*hh + 16*gl + 4*t + i of the slot holds
                    // the f16 pair (column 8t+i, column 8t+i+4) of group 2hh+gl.
                    // A row's four 16-byte lane words are read starting at word rot = (trow >> 1) & 3 (so the
                    // eight rows of a quarter-warp hit eight different bank groups) and rotated back.
                    const int rot = (trow >> 1) & 3;
                    uint4 W4[4];
                    if (!Q8) {
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            W4[k] = *reinterpret_cast<const uint4*>(blk + trow * 64 + ((k + rot) & 3) * 16);
                        rotate_back(W4, rot);
                    }
                    for (int hh = 0; hh < nh; ++hh) {
                        uint32_t v[32];
                        if (!Q8) {
                            // int4: lane word t holds word t (columns 8t..8t+7, nibble n = column 8t+n,
                            // u = v + 8) of each of the quad's four groups.
#pragma unroll
                            for (int t = 0; t < 4; ++t) {
                                const uint2 wv = hh ? make_uint2(W4[t].z, W4[t].w) : make_uint2(W4[t].x, W4[t].y);
#pragma unroll
                                for (int gl = 0; gl < 2; ++gl) {
                                    const uint32_t wd = gl ? wv.y : wv.x, w8 = wd >> 8;
                                    const uint32_t sg = s2[2 * hh + gl];
                                    const float sf = sfl[2 * hh + gl], bg = bfl[2 * hh + gl];
                                    uint32_t* o = v + 16 * gl + 4 * t;
                                    // (u - 8) * scale (+ bias for the affine format), each pair exact until then
                                    o[0] = scale_pair<AFF>(
                                        mb_hsub2(mb_lop_and_or(wd, 0x000F000Fu, 0x64006400u), 0x64086408u), sg, sf, bg, a.piece);
                                    o[1] = scale_pair<AFF>(
                                        mb_hfma2(mb_lop_and_or(wd, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD480D480u),
                                        sg, sf, bg, a.piece);
                                    o[2] = scale_pair<AFF>(
                                        mb_hsub2(mb_lop_and_or(w8, 0x000F000Fu, 0x64006400u), 0x64086408u), sg, sf, bg, a.piece);
                                    o[3] = scale_pair<AFF>(
                                        mb_hfma2(mb_lop_and_or(w8, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD480D480u),
                                        sg, sf, bg, a.piece);
                                }
                            }
                        } else {
                            // int8: half hh holds groups 2hh, 2hh+1; lane word t has the 8 columns 8t..8t+7 of
                            // each (group 2hh + gl at byte 8 gl), bytes u = q + 128 in the order
                            // c0 c4 c1 c5 c2 c6 c3 c7: byte pair i is the pair (8t+i, 8t+i+4).
#pragma unroll
                            for (int k = 0; k < 4; ++k)
                                W4[k] = *reinterpret_cast<const uint4*>(blk + hh * 1024 + trow * 64 + ((k + rot) & 3) * 16);
                            rotate_back(W4, rot);
#pragma unroll
                            for (int t = 0; t < 4; ++t) {
                                const uint4 wv = W4[t];
#pragma unroll
                                for (int gl = 0; gl < 2; ++gl) {
                                    const uint32_t w0 = gl ? wv.z : wv.x, w1 = gl ? wv.w : wv.y;
                                    const uint32_t sg = s2[2 * hh + gl];
                                    uint32_t* o = v + 16 * gl + 4 * t;
                                    o[0] = mb_hmul2(mb_hsub2(mb_prmt(w0, 0x00006464u, 0x5140u), 0x64806480u), sg);
                                    o[1] = mb_hmul2(mb_hsub2(mb_prmt(w0, 0x00006464u, 0x5342u), 0x64806480u), sg);
                                    o[2] = mb_hmul2(mb_hsub2(mb_prmt(w1, 0x00006464u, 0x5140u), 0x64806480u), sg);
                                    o[3] = mb_hmul2(mb_hsub2(mb_prmt(w1, 0x00006464u, 0x5342u), 0x64806480u), sg);
                                }
                            }
                        }
                        tmem_st32_nowait(taddr + 32 * hh, v);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mb_mbar_arrive(&a_full[as]);
                        mb_mbar_arrive(&p_empty[ps]);
                    }
                }
            }
        }
    } else if (warp >= 4 + kDqWarps) {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;
        const int L = 32 * q + lane;
        const int et = threadIdx.x - 32 * (4 + kDqWarps);   // 0..127
        const uint32_t lane_addr = (uint32_t)(32 * q) << 16;
        Items w(a, meta, pstart);
        int64_t np = 0;
        while (w.next()) {
            const float wunscale = pow2i(-clamp120(w.wexp));
            for (int pass = 0; pass < w.passes; ++pass, ++np) {
                const int slot = (int)(np & 1);
                const int n0 = (w.pass0 + pass) * kMaxN;
                const int nrows = min(kMaxN, w.n_e - n0);
                const int npad = (nrows + 15) & ~15;
                float* ts = tok_s + slot * kMaxN;
                float* ta = tok_a + slot * kMaxN;
                float** ty = tok_y + slot * kMaxN;
                for (int n = et; n < ((nrows + 31) & ~31); n += 128) {   // padding tokens: scale 0
                    float s0 = 0.f, s1 = 0.f;
                    if (n < nrows) {
                        const int pick = w.off_e + n0 + n;
                        const int rexp = a.row_exp[a.sorted_rows ? a.sorted_rows[pick] : pick];
                        const int ea = clamp120(w.aexp + 2 * rexp);
                        s0 = pow2i(a.phase == 1 ? -clamp120(rexp) : -ea);
                        s1 = pow2i(ea);
                        if (a.phase == 2) {
                            if (a.y_ret) {
                                const uint32_t r = (uint32_t)a.y_ret[pick];
                                const int src = (int)(r >> 24);
                                const int64_t row = (int64_t)(r & 0xffffffu);
                                if (src < a.n_peers && row < a.peer_rows) {
                                    ty[n] = a.y_peers[src] + row * a.O_real;
                                } else {
                                    ty[n] = nullptr;
                                    atomicOr(a.status, MB_STATUS_BADARG);
                                }
                            } else {
                                ty[n] = a.y + (int64_t)pick * a.O_real;
                            }
                        }
                    }
                    ts[n] = s0;
                    ta[n] = s1;
                }
                mb_named_barrier(1, 32 * kEpiWarps);
                const bool ok = mb_mbar_wait_spin(&acc_full[slot], (uint32_t)((np >> 1) & 1), a.status, abort_flag);
                tc_fence_after();
                const uint32_t acol = tmem + lane_addr + kAccCol + slot * kMaxN;
                for (int cb = 0; cb < npad; cb += 32) {
                    uint32_t r[32];
                    tmem_ld32(acol + cb, r);
                    if (!ok) continue;
                    // Batches of 8 tokens (8 token pairs in phase 1): first the batch's scales (and output
                    // rows) as broadcast reads of shared memory, then the values, then the stores, so the eight
                    // independent chains overlap (one epilogue warp per scheduler has nothing else to hide
                    // their latency with).  Reads placed between the global stores would each wait behind the
                    // previous store (the compiler cannot rule out that a store changes them).
                    if (a.phase == 1 && a.pre) {
                        // precise gate|up: lanes s < 16 hold gate row j, lanes 16 + s the up row j; their true
                        // values go to pre[pick][j] and pre[pick][I + j], written or added
                        const int s = lane & 15;
                        const int j = w.mb * 64 + 16 * q + s;
                        const int col = (lane >= 16 ? a.O_real : 0) + j;
                        const float tsv = ts[cb + lane] * wunscale;
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            const int n = cb + i;
                            const float v = __uint_as_float(r[i]) * __shfl_sync(0xffffffffu, tsv, i);
                            if (n < nrows && j < a.O_real) {
                                float* dst = a.pre + (int64_t)(w.off_e + n0 + n) * (2 * a.O_real) + col;
                                *dst = a.accumulate ? *dst + v : v;
                            }
                        }
                    } else if (a.phase == 1) {
                        // lanes s < 16 hold gate row j, lanes 16 + s the up row j: per pair of tokens (i, i+1)
                        // the low lane forms token i and the high lane token i+1; then lanes s and s+4 (columns
                        // j, j+4: adjacent in the K order) store one f16 pair.
                        const int s = lane & 15;
                        const bool hi = lane >= 16;
                        const int j = w.mb * 64 + 16 * q + s;
                        const int jpos = (j & ~7) + 2 * (s & 3);
#pragma unroll
                        for (int i0 = 0; i0 < 32; i0 += 16) {
                            float tsk[8], tak[8];
                            load_alt8(ts + cb + i0, hi, tsk);
                            load_alt8(ta + cb + i0, hi, tak);
                            float gv[8], uv[8];
#pragma unroll
                            for (int k = 0; k < 8; ++k) {
                                const int i = i0 + 2 * k;
                                const float other =
                                    __uint_as_float(__shfl_xor_sync(0xffffffffu, hi ? r[i] : r[i + 1], 16));
                                const float f = tsk[k] * wunscale;
                                gv[k] = (hi ? other : __uint_as_float(r[i])) * f;
                                uv[k] = (hi ? __uint_as_float(r[i + 1]) : other) * f;
                            }
                            float act[8];
#pragma unroll
                            for (int k = 0; k < 8; ++k)
                                act[k] = __fdividef(gv[k], 1.0f + __expf(-gv[k])) * uv[k] * tak[k];
                            uint32_t pk[8];
#pragma unroll
                            for (int k = 0; k < 8; ++k) pk[k] = pack_f16(act[k], __shfl_xor_sync(0xffffffffu, act[k], 4));
#pragma unroll
                            for (int k = 0; k < 8; ++k) {
                                const int n = cb + i0 + 2 * k + (hi ? 1 : 0);
                                if ((s & 4) == 0 && n < nrows && j < a.O_real)
                                    *reinterpret_cast<uint32_t*>(a.act + (int64_t)(w.off_e + n0 + n) * a.O_real +
                                                                 jpos) = pk[k];
                            }
                        }
                    } else {
                        const int o = w.mb * kBM + L;
                        float* const* ty = tok_y + slot * kMaxN + cb;
#pragma unroll
                        for (int i0 = 0; i0 < 32; i0 += 8) {
                            const float4 s0 = *reinterpret_cast<const float4*>(ts + cb + i0);
                            const float4 s1 = *reinterpret_cast<const float4*>(ts + cb + i0 + 4);
                            const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
                            float* dst[8];
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                const ulonglong2 pp = *reinterpret_cast<const ulonglong2*>(ty + i0 + 2 * c);
                                dst[2 * c] = reinterpret_cast<float*>(pp.x);
                                dst[2 * c + 1] = reinterpret_cast<float*>(pp.y);
                            }
#pragma unroll
                            for (int k = 0; k < 8; ++k) {
                                const int n = cb + i0 + k;
                                const float v = __uint_as_float(r[i0 + k]) * sc[k] * wunscale;
                                if (n < nrows && o < a.O_real && dst[k]) dst[k][o] = v;
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mb_mbar_arrive(&acc_empty[slot]);
            }
        }
        if (a.y_ret) __threadfence_system();   // rows stored to other GPUs are seen before what follows the launch
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 2) tmem_dealloc(tmem, kTmemCols);
}

// The picks' tokens in pick order as f16, each row scaled by 2^row_exp[row]
// (K-permuted): xp[p] = f16(x[sorted_rows[p]] * 2^row_exp[sorted_rows[p]]).
__global__ void gather_f16_kernel(const float* __restrict__ x, const int32_t* __restrict__ sorted_rows,
                                  const int32_t* __restrict__ row_exp, int64_t P, int H, __half* __restrict__ xp,
                                  __half* __restrict__ xp_lo)
{
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (c >= H) return;
    for (int64_t p = blockIdx.y; p < P; p += gridDim.y) {   // gridDim.y <= 65535
    const int64_t row = sorted_rows[p];
    const float sc = pow2i(clamp120(row_exp[row]));
    float4 lo = *reinterpret_cast<const float4*>(x + row * H + c);
    float4 hi = *reinterpret_cast<const float4*>(x + row * H + c + 4);
    lo.x *= sc, lo.y *= sc, lo.z *= sc, lo.w *= sc, hi.x *= sc, hi.y *= sc, hi.z *= sc, hi.w *= sc;
    const uint4 h = pack8_perm(lo, hi, 1.0f);
    *reinterpret_cast<uint4*>(xp + p * H + c) = h;
    if (xp_lo) {                // the residual pieces x * 2^e - f16(x * 2^e), in the same order
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
        const float2 c2 = __half22float2(*reinterpret_cast<const __half2*>(&h.z));
        const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&h.w));
        const float4 rl = make_float4(lo.x - a.x, lo.y - b.x, lo.z - c2.x, lo.w - d.x);
        const float4 rh = make_float4(hi.x - a.y, hi.y - b.y, hi.z - c2.y, hi.w - d.y);
        *reinterpret_cast<uint4*>(xp_lo + p * H + c) = pack8_perm(rl, rh, 1.0f);
    }
    }
}

// SiLU(gate) * up of each pick from the f32 pre-activations of the precise gate|up path (one warp per pick),
// scaled by the pick's activation exponent and written as f16 in the K order 0 4 1 5 2 6 3 7.
__global__ void swiglu_act_kernel(const float* __restrict__ pre, int64_t P, int I, const int32_t* __restrict__ offsets,
                                  int E, const int32_t* __restrict__ e_exp, const int32_t* __restrict__ sorted_rows,
                                  const int32_t* __restrict__ row_exp, __half* __restrict__ act)
{
    const int64_t p = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (p >= P) return;
    int lo = 0, hi = E;                       // the expert whose picks [offsets[e], offsets[e+1]) hold p
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (offsets[mid] <= p) lo = mid; else hi = mid;
    }
    const float sc = pow2i(clamp120(e_exp[4 * lo + 2] + 2 * row_exp[sorted_rows[p]]));
    const float* g = pre + p * (2 * (int64_t)I);
    const float* u = g + I;
    for (int c = lane * 8; c < I; c += 256) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float gv = g[c + j];
            v[j] = __fdividef(gv, 1.0f + __expf(-gv)) * u[c + j];
        }
        *reinterpret_cast<uint4*>(act + p * I + c) =
            pack8_perm(make_float4(v[0], v[1], v[2], v[3]), make_float4(v[4], v[5], v[6], v[7]), sc);
    }
}

// ---- host side -----------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_fn(EncodeTiledFn* out)
{
    static std::mutex mu;
    static EncodeTiledFn fn = nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
            return mb_fail(MB_ECUDA, "mb_moe_prefill: cuTensorMapEncodeTiled unavailable");
        fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    *out = fn;
    return MB_OK;
}

// Tensor maps of a (rows, cols) row-major f16 matrix, boxes of 64 columns x 32, 64, ..., kMaxN rows,
// 128-byte swizzle.
int f16_maps(TokenMaps* maps, const void* base, int64_t rows, int64_t cols)
{
    EncodeTiledFn fn;
    int rc = encode_fn(&fn);
    if (rc) return rc;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t estr[2] = {1, 1};
    for (int i = 0; i < kNumBoxMaps; ++i) {
        const cuuint32_t box[2] = {64, (cuuint32_t)((i + 1) * kBoxStep)};
        CUresult r = fn(&maps->m[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return mb_fail(MB_ECUDA, "mb_moe_prefill: cuTensorMapEncodeTiled failed (%d)", (int)r);
    }
    return MB_OK;
}

int block_bytes_of(int fmt)
{
    if (fmt == MB_FMT_Q4K_F32) return 1024 + 256 + 256;
    const bool q8 = fmt == MB_FMT_Q8_F16 || fmt == MB_FMT_Q8_F32;
    const bool f16 = fmt == MB_FMT_Q4_F16 || fmt == MB_FMT_Q8_F16;
    return (q8 ? 2048 : 1024) + 64 * (f16 ? 2 : 4);
}

size_t smem_bytes(int fmt, int block_bytes, int E)
{
    const int ps = pstages(fmt == MB_FMT_Q8_F16 || fmt == MB_FMT_Q8_F32);
    return 1024 + (size_t)kBStages * 2 * kBHalf + (size_t)ps * 8 * block_bytes + 4 * kMaxN * 4 + 2 * kMaxN * 8 +
           (2 * kBStages + 2 * ps + 2 * kASlots + 4) * 8 + 16 + (size_t)E * 16 + (size_t)(E + 1) * 4 + 16 * 4;
}

template <int FMT>
int launch(const PrefillArgs& a, const TokenMaps& maps, cudaStream_t st)
{
    auto kern = prefill_kernel<FMT>;
    const size_t smem = smem_bytes(FMT, a.block_bytes, a.E);
    static thread_local size_t set[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (set[dev & 63] < smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) {
            (void)cudaGetLastError();
            return mb_fail(MB_ECUDA, "mb_moe_prefill: smem attribute: %s", cudaGetErrorString(e));
        }
        set[dev & 63] = smem;
    }
    const int grid = std::max(1, std::min(a.max_items, mb_num_sms()));
    kern<<<grid, kThreads, smem, st>>>(a, maps);
    return mb_check_launch("mb_moe_prefill");
}

int dispatch(int fmt, const PrefillArgs& a, const TokenMaps& map, cudaStream_t st)
{
    switch (fmt) {
    case MB_FMT_Q4_F32: return launch<MB_FMT_Q4_F32>(a, map, st);
    case MB_FMT_Q4_F16: return launch<MB_FMT_Q4_F16>(a, map, st);
    case MB_FMT_Q8_F32: return launch<MB_FMT_Q8_F32>(a, map, st);
    case MB_FMT_Q8_F16: return launch<MB_FMT_Q8_F16>(a, map, st);
    case MB_FMT_Q4K_F32: return launch<MB_FMT_Q4K_F32>(a, map, st);
    default: return mb_fail(MB_EUNSUPPORTED, "mb_moe_prefill: weight format %d", fmt);
    }
}

int64_t r1k(int64_t n) { return (n + 1023) / 1024 * 1024; }

// At most MB * (E + P / kMaxN) items: every expert's passes over P picks in all.
int items_bound(int MB, int E, int64_t P)
{
    return (int)std::min<int64_t>((int64_t)MB * (E + (P + kMaxN - 1) / kMaxN), 1 << 30);
}

// The GEMM launches of one layer over tokens already in f16 rows xp (P x H, pick order, K-permuted, each
// scaled by 2^row_exp): gate|up into a.act (with the precise three-product form when fmt_gu is
// MB_FMT_Q4K_F32: xp_lo the residual rows, pre the f32 pre-activations), then down into the output rows.
int run_gemms(PrefillArgs a, int H, int I, int fmt_gu, int fmt_down, const __half* xp, const __half* xp_lo,
              float* pre, int64_t P, cudaStream_t st)
{
    TokenMaps map;
    // gate|up: K = H, rows 2I (RT = I/8 tiles of 8 gate + 8 up rows) -> act (P, I) f16
    int rc = f16_maps(&map, xp, P, H);
    if (rc) return rc;
    a.phase = 1;
    a.NQ = H / 128;
    a.KH = H / 64;
    a.RT = I / 8;
    a.MB = (a.RT + 7) / 8;
    a.max_items = items_bound(a.MB, a.E, P);
    a.block_bytes = block_bytes_of(fmt_gu);
    a.O_real = I;
    if (fmt_gu != MB_FMT_Q4K_F32) {
        rc = dispatch(fmt_gu, a, map, st);
        if (rc) return rc;
    } else {
        // three products with f16 operands, each exact in its f32 accumulation: W_hi x_hi + W_hi x_lo + W_lo x_hi
        // (W_lo x_lo is below f32 rounding of the sum), then SiLU(gate) * up from the f32 sums
        TokenMaps map_lo;
        rc = f16_maps(&map_lo, xp_lo, P, H);
        if (rc) return rc;
        a.pre = pre;
        const TokenMaps* maps[3] = {&map, &map_lo, &map};
        for (int pass = 0; pass < 3; ++pass) {
            a.piece = pass == 2 ? 1 : 0;
            a.accumulate = pass > 0;
            rc = dispatch(fmt_gu, a, *maps[pass], st);
            if (rc) return rc;
        }
        a.pre = nullptr;
        a.piece = a.accumulate = 0;
        swiglu_act_kernel<<<(unsigned)((P + 7) / 8), 256, 0, st>>>(pre, P, I, a.offsets, a.E, a.e_exp,
                                                                   a.sorted_rows, a.row_exp, a.act);
        rc = mb_check_launch("mb_moe_prefill swiglu");
        if (rc) return rc;
    }

    // down: K = I, rows H -> y (P, H)
    rc = f16_maps(&map, a.act, P, I);
    if (rc) return rc;
    a.phase = 2;
    a.NQ = (I + 127) / 128;
    a.KH = I / 64;
    a.RT = H / 16;
    a.MB = (a.RT + 7) / 8;
    a.max_items = items_bound(a.MB, a.E, P);
    a.block_bytes = block_bytes_of(fmt_down);
    a.O_real = H;
    return dispatch(fmt_down, a, map, st);
}

}  // namespace

// Workspace (from its first 1024-byte boundary): the picks' tokens as f16 (P x H) | the activations as f16
// (P x I) | status word | for the precise gate|up path (affine int4): the tokens' f16 residuals (P x H) and
// the pre-activations (P x 2I) f32.
extern "C" int64_t mb_moe_prefill_workspace_bytes(int64_t P, int H, int I, int fmt_gu)
{
    const int64_t extra = fmt_gu == MB_FMT_Q4K_F32 ? r1k(P * H * 2) + r1k(P * 2 * I * 4) : 0;
    return 1024 + r1k(P * H * 2) + r1k(P * I * 2) + 256 + extra;
}

extern "C" int mb_moe_prefill(const MbExpert* table, const int32_t* e_exp, int E, int H, int I, int gs, int fmt_gu,
                              int fmt_down, const float* x, const int32_t* row_exp, int64_t T, const int32_t* counts,
                              const int32_t* offsets, const int32_t* sorted_rows, int64_t P, int min_rows, float* y,
                              void* workspace, int64_t workspace_bytes, unsigned* status, void* stream)
{
    MB_REQUIRE(table && e_exp && x && row_exp && counts && offsets && sorted_rows && y && workspace,
               "mb_moe_prefill: null pointer");
    MB_REQUIRE(E > 0 && E <= kMaxMetaE && T >= 0 && P >= 0, "mb_moe_prefill: E=%d (at most %d experts)", E,
               kMaxMetaE);
    MB_REQUIRE(H % 128 == 0 && I % 64 == 0 && H > 0 && I > 0,
               "mb_moe_prefill: needs H %% 128 == 0 and I %% 64 == 0 (H=%d I=%d)", H, I);
    MB_REQUIRE(gs % 32 == 0 && H % gs == 0 && I % gs == 0, "mb_moe_prefill: group size %d", gs);
    MB_REQUIRE(((uintptr_t)x & 15) == 0 && ((uintptr_t)workspace & 15) == 0,
               "mb_moe_prefill: x and workspace must be 16-byte aligned");
    MB_REQUIRE(P <= 65536, "mb_moe_prefill: P=%lld above 65536 (the limit of mb_permute)", (long long)P);
    MB_REQUIRE(workspace_bytes >= mb_moe_prefill_workspace_bytes(P, H, I, fmt_gu),
               "mb_moe_prefill: workspace too small");
    if (P == 0) return MB_OK;
    cudaStream_t st = mb_stream(stream);
    uint8_t* ws = reinterpret_cast<uint8_t*>(((uintptr_t)workspace + 1023) & ~(uintptr_t)1023);
    __half* xp = reinterpret_cast<__half*>(ws);
    ws += r1k(P * H * 2);
    __half* act = reinterpret_cast<__half*>(ws);
    ws += r1k(P * I * 2);
    unsigned* ws_status = reinterpret_cast<unsigned*>(ws);
    ws += 256;
    const bool precise = fmt_gu == MB_FMT_Q4K_F32;
    __half* xp_lo = precise ? reinterpret_cast<__half*>(ws) : nullptr;
    float* pre = precise ? reinterpret_cast<float*>(ws + r1k(P * H * 2)) : nullptr;
    if (!status) {
        status = ws_status;
        cudaMemsetAsync(status, 0, sizeof(unsigned), st);
    }

    gather_f16_kernel<<<dim3((H / 8 + 127) / 128, (unsigned)std::min<int64_t>(P, 65535)), 128, 0, st>>>(x, sorted_rows, row_exp, P, H, xp,
                                                                            xp_lo);
    int rc = mb_check_launch("mb_moe_prefill gather");
    if (rc) return rc;

    PrefillArgs a{};
    a.table = table;
    a.e_exp = e_exp;
    a.E = E;
    a.counts = counts;
    a.offsets = offsets;
    a.sorted_rows = sorted_rows;
    a.row_exp = row_exp;
    a.min_rows = min_rows < 1 ? 1 : min_rows;
    a.status = status;
    a.act = act;
    a.y = y;
    return run_gemms(a, H, I, fmt_gu, fmt_down, xp, xp_lo, pre, P, st);
}

// Workspace (from its first 1024-byte boundary): the activations as f16 (P x I) | status word.
extern "C" int64_t mb_moe_prefill_rows_workspace_bytes(int64_t P, int I)
{
    return 1024 + r1k(P * I * 2) + 256;
}

extern "C" int mb_moe_prefill_rows(const MbExpert* table, const int32_t* e_exp, int E, int H, int I, int gs,
                                   int fmt_gu, int fmt_down, const void* xp, const int32_t* row_exp,
                                   const int32_t* counts, const int32_t* offsets, int64_t P, int min_rows, float* y,
                                   const int32_t* y_ret, float* const* y_peers, int n_peers, int64_t peer_rows,
                                   void* workspace, int64_t workspace_bytes, unsigned* status, void* stream)
{
    MB_REQUIRE(table && e_exp && xp && row_exp && counts && offsets && workspace && (y || (y_ret && y_peers)),
               "mb_moe_prefill_rows: null pointer");
    MB_REQUIRE(!y_ret || (n_peers >= 1 && n_peers <= 256 && peer_rows >= 0),
               "mb_moe_prefill_rows: %d result buffers of %lld rows", n_peers, (long long)peer_rows);
    MB_REQUIRE(E > 0 && E <= kMaxMetaE && P >= 0 && P < (1ll << 24),
               "mb_moe_prefill_rows: E=%d (at most %d experts), P=%lld (below 2^24)", E, kMaxMetaE, (long long)P);
    MB_REQUIRE(H % 128 == 0 && I % 64 == 0 && H > 0 && I > 0,
               "mb_moe_prefill_rows: needs H %% 128 == 0 and I %% 64 == 0 (H=%d I=%d)", H, I);
    MB_REQUIRE(gs % 32 == 0 && H % gs == 0 && I % gs == 0, "mb_moe_prefill_rows: group size %d", gs);
    MB_REQUIRE(((uintptr_t)xp & 15) == 0 && ((uintptr_t)workspace & 15) == 0,
               "mb_moe_prefill_rows: xp and workspace must be 16-byte aligned");
    MB_REQUIRE(workspace_bytes >= mb_moe_prefill_rows_workspace_bytes(P, I), "mb_moe_prefill_rows: workspace too small");
    if (fmt_gu == MB_FMT_Q4K_F32)
        return mb_fail(MB_EUNSUPPORTED, "mb_moe_prefill_rows: the precise Q4_K gate|up needs the tokens' f32 rows");
    if (P == 0) return MB_OK;
    cudaStream_t st = mb_stream(stream);
    uint8_t* ws = reinterpret_cast<uint8_t*>(((uintptr_t)workspace + 1023) & ~(uintptr_t)1023);
    __half* act = reinterpret_cast<__half*>(ws);
    ws += r1k(P * I * 2);
    if (!status) {
        status = reinterpret_cast<unsigned*>(ws);
        cudaMemsetAsync(status, 0, sizeof(unsigned), st);
    }
    PrefillArgs a{};
    a.table = table;
    a.e_exp = e_exp;
    a.E = E;
    a.counts = counts;
    a.offsets = offsets;
    a.sorted_rows = nullptr;
    a.row_exp = row_exp;
    a.min_rows = min_rows < 1 ? 1 : min_rows;
    a.status = status;
    a.act = act;
    a.y = y;
    a.y_ret = y_ret;
    a.y_peers = y_peers;
    a.n_peers = n_peers;
    a.peer_rows = peer_rows;
    return run_gemms(a, H, I, fmt_gu, fmt_down, reinterpret_cast<const __half*>(xp), nullptr, nullptr, P, st);
}
