// Prefill: the routed experts as grouped GEMMs on the 5th-generation tensor
// cores (tcgen05), for experts picked by many tokens.
//
// Reference: moelan/experts.py:148-151, 216-219 (GroupQuant / Packed4
// matmul_t with 8 or more rows: widen the matrix to f32, then BLAS x @ W.T),
// run per expert by ExpertStore.compute (experts.py:707-727).
//
// Design (sm_100a), per CTA = (expert, 128 weight rows), all its tokens:
//  * the packed weight tiles (the same HBM tile layout the decode kernels read)
//    are streamed into shared memory with 1-D bulk copies;
//  * four "dequant" warps turn them into f16 ((q - offset) * group scale in
//    f32, times the matrix's power-of-two weight exponent, rounded once) and
//    write them with tcgen05.st straight into tensor memory, where
//    tcgen05.mma reads its A operand: the converted weights never pass
//    through shared memory, whose bandwidth the B operand needs;
//  * the expert's tokens, gathered once per layer into an f16 matrix in pick
//    order (each row times 2^row exponent, so its largest value lies in
//    [2^13, 2^14)), arrive as B by 2-D TMA (128-byte swizzle, K-major);
//  * one thread issues tcgen05.mma (M=128, N <= 192 tokens, K=16, f32 in TMEM);
//    completions are tracked with tcgen05.commit on mbarriers, every wait is
//    bounded;
//  * the same four warps read the accumulators back (tcgen05.ld), undo the
//    power-of-two scalings exactly and form SiLU(gate) * up in f32 (gate|up)
//    or the f32 output rows (down).  The activations go through one more
//    small kernel that rounds each pick's row to f16 with its own exponent.
// f16 rather than bf16 operands: the same tensor-core rate, 3 more mantissa
// bits, and with the exponents above no range is lost.  Tolerance against
// the f32 reference: 2e-3 of each row's max (bf16 operands would give ~7e-3).
#include <cuda.h>

#include <mutex>

#include "mb_common.cuh"

namespace {

constexpr int kBM = 128;      // weight rows per CTA = TMEM lanes
constexpr int kBK = 64;       // K per chunk: one 128-byte swizzled row of f16
constexpr int kMaxN = 192;    // tokens per pass
constexpr int kBStages = 3;   // token (B) chunk stages
constexpr int kPStages = 2;   // packed-weight stages, one 128-column quad each (two K chunks)
constexpr int kTmemCols = 256;
constexpr int kAccCol = 64;   // accumulators at TMEM columns [64, 64 + N); A buffers at [0, 64)
constexpr int kThreads = 192; // warp 0 TMA, warp 1 MMA + TMEM owner, warps 2..5 dequant / epilogue

struct PrefillArgs {
    const MbExpert* table;
    const int32_t* w_exp;   // (E, 2) weight exponents [gate|up, down], or null (0)
    int E;
    int phase;              // 1: gate|up -> act (f32), 2: down -> y (f32)
    int NQ;                 // quads of K in the weight tiles
    int KC;                 // K chunks (K / 64)
    int RT;                 // row tiles of the matrix
    int MB;                 // M blocks (8 row tiles) per expert
    int block_bytes;
    const int32_t* counts;
    const int32_t* offsets;
    const int32_t* tok_rows; // phase 1: sorted_rows (exponent of pick p = tok_exp[tok_rows[p]]); phase 2: null
    const int32_t* tok_exp;  // phase 1: row exponents of x; phase 2: pick exponents of the activations
    int min_rows;
    int O_real;             // phase 1: I (act columns); phase 2: H (y columns)
    float* out;             // phase 1: act (P, I); phase 2: y (P, H)
    int out_ld;
    unsigned* status;
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

__device__ __forceinline__ void tc_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     mb_smem_addr(bar))
                 : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem], kind::f16 (f16 inputs, f32 accumulate).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]),
        "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]),
        "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

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

__device__ __forceinline__ uint32_t pack_f16(float lo, float hi)
{
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// 2^e for -126 <= e <= 127, exact.
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

// ---- the GEMM kernel ----------------------------------------------------------------

template <int FMT>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ PrefillArgs a, const __grid_constant__ CUtensorMap bmap)
{
    constexpr bool Q8 = (FMT == MB_FMT_Q8_F16 || FMT == MB_FMT_Q8_F32);
    constexpr bool F16S = (FMT == MB_FMT_Q4_F16 || FMT == MB_FMT_Q8_F16);
    constexpr int kData = Q8 ? 2048 : 1024;

    const int e = blockIdx.x / a.MB, mb = blockIdx.x - e * a.MB;
    const int n_e = a.counts[e];
    if (n_e < a.min_rows || n_e <= 0) return;
    const int off_e = a.offsets[e];
    const int tiles = min(8, a.RT - mb * 8);     // row tiles of this M block
    const int wexp = a.w_exp ? a.w_exp[2 * e + (a.phase == 1 ? 0 : 1)] : 0;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* bst = smem;                                       // [kBStages][kMaxN][128 B]
    uint8_t* pst = bst + kBStages * kMaxN * 128;               // [kPStages][8 tiles][block]
    float* tok_scale = reinterpret_cast<float*>(pst + kPStages * 8 * a.block_bytes);   // [2][kMaxN]
    uint64_t* bars = reinterpret_cast<uint64_t*>(tok_scale + 2 * kMaxN);
    uint64_t* b_full = bars;                                   // [kBStages]
    uint64_t* b_empty = b_full + kBStages;
    uint64_t* p_full = b_empty + kBStages;                     // [kPStages]
    uint64_t* p_empty = p_full + kPStages;
    uint64_t* a_full = p_empty + kPStages;                     // [2] A buffers in TMEM
    uint64_t* a_empty = a_full + 2;
    uint64_t* acc_full = a_empty + 2;
    uint64_t* acc_empty = acc_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kBStages; ++i) {
            mb_mbar_init(&b_full[i], 1);
            mb_mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < kPStages; ++i) {
            mb_mbar_init(&p_full[i], 1);
            mb_mbar_init(&p_empty[i], 4);
        }
        for (int i = 0; i < 2; ++i) {
            mb_mbar_init(&a_full[i], 4);
            mb_mbar_init(&a_empty[i], 1);
        }
        mb_mbar_init(acc_full, 1);
        mb_mbar_init(acc_empty, 4);
        *abort_flag = 0;
        mb_fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int passes = (n_e + kMaxN - 1) / kMaxN;
    const int KC = a.KC;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            const uint8_t* wbase =
                reinterpret_cast<const uint8_t*>(a.phase == 1 ? a.table[e].gu : a.table[e].down);
            int bs = 0, ps = 0;
            uint32_t bph = 0, pph = 0;
            int64_t bn = 0, pn = 0;
            for (int pass = 0; pass < passes && !*abort_flag; ++pass) {
                const int n0 = pass * kMaxN;
                const int nrows = min(kMaxN, n_e - n0);
                const int nbox = (((nrows + 15) & ~15) + 63) / 64;
                for (int kc = 0; kc < KC; ++kc) {
                    if ((kc & 1) == 0) {  // a new quad of packed weights for the M block
                        if (pn >= kPStages && !mb_mbar_wait(&p_empty[ps], pph ^ 1u, a.status, abort_flag)) break;
                        mb_mbar_arrive_expect_tx(&p_full[ps], (uint32_t)(tiles * a.block_bytes));
                        for (int i = 0; i < tiles; ++i)
                            mb_bulk_g2s(pst + ((size_t)ps * 8 + i) * a.block_bytes,
                                        wbase + ((size_t)(mb * 8 + i) * a.NQ + (kc >> 1)) * a.block_bytes,
                                        (uint32_t)a.block_bytes, &p_full[ps]);
                        ++pn;
                        if (++ps == kPStages) {
                            ps = 0;
                            pph ^= 1u;
                        }
                    }
                    if (bn >= kBStages && !mb_mbar_wait(&b_empty[bs], bph ^ 1u, a.status, abort_flag)) break;
                    mb_mbar_arrive_expect_tx(&b_full[bs], (uint32_t)(nbox * 64 * 128));
                    for (int i = 0; i < nbox; ++i)
                        tma_load_2d(bst + ((size_t)bs * kMaxN + i * 64) * 128, &bmap, kc * kBK, off_e + n0 + i * 64,
                                    &b_full[bs]);
                    ++bn;
                    if (++bs == kBStages) {
                        bs = 0;
                        bph ^= 1u;
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int bs = 0, ab = 0;
            uint32_t bph = 0, abph = 0;
            for (int pass = 0; pass < passes && !*abort_flag; ++pass) {
                const int nrows = min(kMaxN, n_e - pass * kMaxN);
                const int npad = (nrows + 15) & ~15;
                const uint32_t idesc = idesc_f16(npad);
                if (pass > 0 && !mb_mbar_wait(acc_empty, (uint32_t)((pass - 1) & 1), a.status, abort_flag)) break;
                tc_fence_after();
                for (int kc = 0; kc < KC; ++kc) {
                    if (!mb_mbar_wait(&a_full[ab], abph, a.status, abort_flag)) break;
                    if (!mb_mbar_wait(&b_full[bs], bph, a.status, abort_flag)) break;
                    tc_fence_after();
                    const uint32_t bbase = mb_smem_addr(bst + (size_t)bs * kMaxN * 128);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        tc_mma_ts(tmem + kAccCol, tmem + ab * 32 + j * 8, sw128_desc(bbase + j * 32), idesc,
                                  (kc > 0 || j > 0) ? 1u : 0u);
                    tc_commit(&a_empty[ab]);
                    tc_commit(&b_empty[bs]);
                    if (++ab == 2) {
                        ab = 0;
                        abph ^= 1u;
                    }
                    if (++bs == kBStages) {
                        bs = 0;
                        bph ^= 1u;
                    }
                }
                tc_commit(acc_full);
            }
        }
    } else {
        // ------------------------------------------------------------ dequant + epilogue
        const int q = warp & 3;               // TMEM lane quarter this warp may access
        const int L = 32 * q + lane;          // TMEM lane = row of the M block
        const int et = threadIdx.x - 64;      // 0..127 among the four warps
        int ti, trow;                         // source row tile within the M block, row within it
        if (a.phase == 1) {                   // lanes 32q + s: gate row, 32q + 16 + s: the matching up row
            const int s = lane & 15;
            ti = 2 * q + (s >> 3);
            trow = (s & 7) + ((lane >= 16) ? 8 : 0);
        } else {
            ti = L >> 4;
            trow = L & 15;
        }
        const bool row_ok = ti < tiles;
        const uint32_t lane_addr = (uint32_t)(32 * q) << 16;
        const float wscale = pow2i(wexp), wunscale = pow2i(-wexp);
        int ps = 0, ab = 0;
        uint32_t pph = 0, abph = 0;
        int64_t an = 0;
        for (int pass = 0; pass < passes; ++pass) {
            const int n0 = pass * kMaxN;
            const int nrows = min(kMaxN, n_e - n0);
            const int npad = (nrows + 15) & ~15;
            float* tsc = tok_scale + (pass & 1) * kMaxN;
            for (int n = et; n < nrows; n += 128) {
                const int64_t p = off_e + n0 + n;
                tsc[n] = pow2i(-a.tok_exp[a.tok_rows ? a.tok_rows[p] : p]);
            }
            mb_named_barrier(1, 128);
            for (int kc = 0; kc < KC; ++kc) {
                const int h = kc & 1;
                bool ok = true;
                if (h == 0) ok = mb_mbar_wait(&p_full[ps], pph, a.status, abort_flag);
                if (an >= 2) ok = mb_mbar_wait(&a_empty[ab], abph ^ 1u, a.status, abort_flag) && ok;
                tc_fence_after();
                uint32_t v[32];
                const uint8_t* blk = pst + ((size_t)ps * 8 + (row_ok ? ti : 0)) * a.block_bytes;
                float sc[2];
                if (F16S) {
                    const __half2 s2 = *reinterpret_cast<const __half2*>(blk + kData + trow * 8 + 4 * h);
                    sc[0] = __low2float(s2);
                    sc[1] = __high2float(s2);
                } else {
                    const float2 s2 = *reinterpret_cast<const float2*>(blk + kData + trow * 16 + 8 * h);
                    sc[0] = s2.x;
                    sc[1] = s2.y;
                }
                if (!ok || !row_ok) {
                    sc[0] = 0.f;
                    sc[1] = 0.f;
                }
                if (!Q8) {
                    // int4: lane word t holds 4 bytes (8 columns 8t..8t+7, low nibble = even column) of each of
                    // the quad's groups; this chunk takes groups 2h and 2h+1.  Column pair (8t+2b, 8t+2b+1) of
                    // group gl is f16 pair 16*gl + 4t + b of the chunk's 64 columns.
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const uint2 wv = *reinterpret_cast<const uint2*>(blk + trow * 64 + t * 16 + 8 * h);
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const uint32_t x0 = (wv.x >> (8 * b)) & 0xFF, x1 = (wv.y >> (8 * b)) & 0xFF;
                            const float lo0 = __int_as_float(0x4B000000 | (x0 & 15)) - 8388616.0f;
                            const float hi0 = __int_as_float(0x4B000000 | (x0 >> 4)) - 8388616.0f;
                            const float lo1 = __int_as_float(0x4B000000 | (x1 & 15)) - 8388616.0f;
                            const float hi1 = __int_as_float(0x4B000000 | (x1 >> 4)) - 8388616.0f;
                            v[4 * t + b] = pack_f16(lo0 * sc[0] * wscale, hi0 * sc[0] * wscale);
                            v[16 + 4 * t + b] = pack_f16(lo1 * sc[1] * wscale, hi1 * sc[1] * wscale);
                        }
                    }
                } else {
                    // int8: half h holds groups 2h, 2h+1; lane word t has the 8 columns 8t..8t+7 of each in
                    // the order c0 c4 c1 c5 c2 c6 c3 c7 (offset by 128).
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const uint4 wv = *reinterpret_cast<const uint4*>(blk + h * 1024 + trow * 64 + t * 16);
                        const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                        for (int gl = 0; gl < 2; ++gl) {
                            const uint32_t w0 = w[2 * gl], w1 = w[2 * gl + 1];
                            // columns (8t+2i, 8t+2i+1) sit at byte positions (0,2) (4,6) (1,3) (5,7)
                            const uint32_t byt[8] = {w0 & 0xFF, (w0 >> 8) & 0xFF, (w0 >> 16) & 0xFF, w0 >> 24,
                                                     w1 & 0xFF, (w1 >> 8) & 0xFF, (w1 >> 16) & 0xFF, w1 >> 24};
                            const int pa[4] = {0, 4, 1, 5}, pb[4] = {2, 6, 3, 7};
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const float f0 = __int_as_float(0x4B000000 | byt[pa[i]]) - 8388736.0f;
                                const float f1 = __int_as_float(0x4B000000 | byt[pb[i]]) - 8388736.0f;
                                v[16 * gl + 4 * t + i] = pack_f16(f0 * sc[gl] * wscale, f1 * sc[gl] * wscale);
                            }
                        }
                    }
                }
                tmem_st32(tmem + lane_addr + ab * 32, v);
                tc_fence_before();
                __syncwarp();
                const bool quad_done = h == 1 || kc == KC - 1;
                if (lane == 0) {
                    mb_mbar_arrive(&a_full[ab]);
                    if (quad_done) mb_mbar_arrive(&p_empty[ps]);
                }
                ++an;
                if (++ab == 2) {
                    ab = 0;
                    abph ^= 1u;
                }
                if (quad_done && ++ps == kPStages) {
                    ps = 0;
                    pph ^= 1u;
                }
            }
            // epilogue of this pass
            const bool ok = mb_mbar_wait(acc_full, (uint32_t)(pass & 1), a.status, abort_flag);
            tc_fence_after();
            for (int cb = 0; cb < npad; cb += 32) {
                uint32_t r[32];
                tmem_ld32(tmem + lane_addr + kAccCol + cb, r);
                if (!ok) continue;
                if (a.phase == 1) {
                    const int s = lane & 15;
                    const int j = mb * 64 + 16 * q + s;
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int n = cb + i;
                        const float gv = __uint_as_float(r[i]) * tsc[n < kMaxN ? n : 0] * wunscale;
                        const float uv = __shfl_xor_sync(0xffffffffu, gv, 16);
                        if (lane < 16 && n < nrows && j < a.O_real) {
                            const float act = gv / (1.0f + expf(-gv)) * uv;
                            a.out[(int64_t)(off_e + n0 + n) * a.out_ld + j] = act;
                        }
                    }
                } else {
                    const int o = mb * kBM + L;
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int n = cb + i;
                        if (n < nrows && o < a.O_real)
                            a.out[(int64_t)(off_e + n0 + n) * a.out_ld + o] =
                                __uint_as_float(r[i]) * tsc[n] * wunscale;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mb_mbar_arrive(acc_empty);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// The picks' tokens in pick order as f16, each row scaled by 2^row_exp[row]:
// xp[p] = f16(x[sorted_rows[p]] * 2^row_exp[sorted_rows[p]]).
__global__ void gather_f16_kernel(const float* __restrict__ x, const int32_t* __restrict__ sorted_rows,
                                  const int32_t* __restrict__ row_exp, int64_t P, int H, __half* __restrict__ xp)
{
    const int64_t p = blockIdx.y;
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (p >= P || c >= H) return;
    const int64_t row = sorted_rows[p];
    const float sc = pow2i(row_exp[row]);
    const float4 v = *reinterpret_cast<const float4*>(x + row * H + c);
    uint2 o;
    o.x = pack_f16(v.x * sc, v.y * sc);
    o.y = pack_f16(v.z * sc, v.w * sc);
    *reinterpret_cast<uint2*>(xp + p * H + c) = o;
}

// Each pick's activation row to f16 with its own exponent (one warp per pick):
// e = the exponent that maps the row's largest magnitude into [2^13, 2^14).
__global__ void act_to_f16_kernel(const float* __restrict__ act, int64_t P, int I, __half* __restrict__ act16,
                                  int32_t* __restrict__ pick_exp)
{
    const int64_t p = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (p >= P) return;
    const float* row = act + p * I;
    float m = 0.0f;
    for (int c = lane * 4; c < I; c += 128) {
        const float4 v = *reinterpret_cast<const float4*>(row + c);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int e = mb_row_exponent(m);
    const float sc = pow2i(e);
    for (int c = lane * 4; c < I; c += 128) {
        const float4 v = *reinterpret_cast<const float4*>(row + c);
        uint2 o;
        o.x = pack_f16(v.x * sc, v.y * sc);
        o.y = pack_f16(v.z * sc, v.w * sc);
        *reinterpret_cast<uint2*>(act16 + p * I + c) = o;
    }
    if (lane == 0) pick_exp[p] = e;
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

// Tensor map of a (rows, cols) row-major f16 matrix, boxes of 64 columns x 64 rows, 128-byte swizzle.
int f16_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols)
{
    EncodeTiledFn fn;
    int rc = encode_fn(&fn);
    if (rc) return rc;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {64, 64};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return mb_fail(MB_ECUDA, "mb_moe_prefill: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return MB_OK;
}

int block_bytes_of(int fmt)
{
    const bool q8 = fmt == MB_FMT_Q8_F16 || fmt == MB_FMT_Q8_F32;
    const bool f16 = fmt == MB_FMT_Q4_F16 || fmt == MB_FMT_Q8_F16;
    return (q8 ? 2048 : 1024) + 64 * (f16 ? 2 : 4);
}

size_t smem_bytes(int block_bytes)
{
    return 1024 + (size_t)kBStages * kMaxN * 128 + (size_t)kPStages * 8 * block_bytes + 2 * kMaxN * 4 + 16 * 8 +
           64;
}

template <int FMT>
int launch(const PrefillArgs& a, const CUtensorMap& map, cudaStream_t st)
{
    auto kern = prefill_kernel<FMT>;
    const size_t smem = smem_bytes(a.block_bytes);
    static thread_local size_t set[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (set[dev & 63] < smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return mb_fail(MB_ECUDA, "mb_moe_prefill: smem attribute: %s", cudaGetErrorString(e));
        set[dev & 63] = smem;
    }
    kern<<<a.E * a.MB, kThreads, smem, st>>>(a, map);
    return mb_check_launch("mb_moe_prefill");
}

int dispatch(int fmt, const PrefillArgs& a, const CUtensorMap& map, cudaStream_t st)
{
    switch (fmt) {
    case MB_FMT_Q4_F32: return launch<MB_FMT_Q4_F32>(a, map, st);
    case MB_FMT_Q4_F16: return launch<MB_FMT_Q4_F16>(a, map, st);
    case MB_FMT_Q8_F32: return launch<MB_FMT_Q8_F32>(a, map, st);
    case MB_FMT_Q8_F16: return launch<MB_FMT_Q8_F16>(a, map, st);
    default: return mb_fail(MB_EUNSUPPORTED, "mb_moe_prefill: weight format %d", fmt);
    }
}

int64_t r1k(int64_t n) { return (n + 1023) / 1024 * 1024; }

}  // namespace

// Workspace (from its first 1024-byte boundary): the picks' tokens as f16 (P x H) | the activations in f32
// (P x I) | the activations as f16 (P x I) | each pick's activation exponent (P) | status word.
extern "C" int64_t mb_moe_prefill_workspace_bytes(int64_t P, int H, int I)
{
    return 1024 + r1k(P * H * 2) + r1k(P * I * 4) + r1k(P * I * 2) + r1k(P * 4) + 256;
}

extern "C" int mb_moe_prefill(const MbExpert* table, const int32_t* w_exp, int E, int H, int I, int gs, int fmt_gu,
                              int fmt_down, const float* x, const int32_t* row_exp, int64_t T, const int32_t* counts,
                              const int32_t* offsets, const int32_t* sorted_rows, int64_t P, int min_rows, float* y,
                              void* workspace, int64_t workspace_bytes, unsigned* status, void* stream)
{
    MB_REQUIRE(table && x && row_exp && counts && offsets && sorted_rows && y && workspace,
               "mb_moe_prefill: null pointer");
    MB_REQUIRE(E > 0 && E <= 65535 && T >= 0 && P >= 0, "mb_moe_prefill: bad sizes");
    MB_REQUIRE(H % 128 == 0 && I % 64 == 0 && H > 0 && I > 0,
               "mb_moe_prefill: needs H %% 128 == 0 and I %% 64 == 0 (H=%d I=%d)", H, I);
    MB_REQUIRE(gs % 32 == 0 && H % gs == 0 && I % gs == 0, "mb_moe_prefill: group size %d", gs);
    MB_REQUIRE(((uintptr_t)x & 15) == 0 && ((uintptr_t)workspace & 15) == 0,
               "mb_moe_prefill: x and workspace must be 16-byte aligned");
    MB_REQUIRE(P <= 65535, "mb_moe_prefill: P=%lld above 65535", (long long)P);
    MB_REQUIRE(workspace_bytes >= mb_moe_prefill_workspace_bytes(P, H, I), "mb_moe_prefill: workspace too small");
    if (P == 0) return MB_OK;
    cudaStream_t st = mb_stream(stream);
    uint8_t* ws = reinterpret_cast<uint8_t*>(((uintptr_t)workspace + 1023) & ~(uintptr_t)1023);
    __half* xp = reinterpret_cast<__half*>(ws);
    ws += r1k(P * H * 2);
    float* act32 = reinterpret_cast<float*>(ws);
    ws += r1k(P * I * 4);
    __half* act16 = reinterpret_cast<__half*>(ws);
    ws += r1k(P * I * 2);
    int32_t* pick_exp = reinterpret_cast<int32_t*>(ws);
    ws += r1k(P * 4);
    unsigned* ws_status = reinterpret_cast<unsigned*>(ws);
    if (!status) {
        status = ws_status;
        cudaMemsetAsync(status, 0, sizeof(unsigned), st);
    }

    gather_f16_kernel<<<dim3((H / 4 + 255) / 256, (unsigned)P), 256, 0, st>>>(x, sorted_rows, row_exp, P, H, xp);
    int rc = mb_check_launch("mb_moe_prefill gather");
    if (rc) return rc;

    PrefillArgs a{};
    a.table = table;
    a.w_exp = w_exp;
    a.E = E;
    a.counts = counts;
    a.offsets = offsets;
    a.min_rows = min_rows < 1 ? 1 : min_rows;
    a.status = status;

    CUtensorMap map;
    // gate|up: K = H, rows 2I (RT = I/8 tiles of 8 gate + 8 up rows) -> act (P, I) f32
    rc = f16_map(&map, xp, P, H);
    if (rc) return rc;
    a.phase = 1;
    a.NQ = H / 128;
    a.KC = H / kBK;
    a.RT = I / 8;
    a.MB = (a.RT + 7) / 8;
    a.block_bytes = block_bytes_of(fmt_gu);
    a.tok_rows = sorted_rows;
    a.tok_exp = row_exp;
    a.O_real = I;
    a.out = act32;
    a.out_ld = I;
    rc = dispatch(fmt_gu, a, map, st);
    if (rc) return rc;

    act_to_f16_kernel<<<(unsigned)((P + 7) / 8), 256, 0, st>>>(act32, P, I, act16, pick_exp);
    rc = mb_check_launch("mb_moe_prefill act");
    if (rc) return rc;

    // down: K = I, rows H -> y (P, H)
    rc = f16_map(&map, act16, P, I);
    if (rc) return rc;
    a.phase = 2;
    a.NQ = (I + 127) / 128;
    a.KC = I / kBK;
    a.RT = H / 16;
    a.MB = (a.RT + 7) / 8;
    a.block_bytes = block_bytes_of(fmt_down);
    a.tok_rows = nullptr;
    a.tok_exp = pick_exp;
    a.O_real = H;
    a.out = y;
    a.out_ld = H;
    return dispatch(fmt_down, a, map, st);
}
