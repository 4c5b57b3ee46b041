// Fused decode mat-vecs over packed experts: one MoE layer's gate|up, SiLU,
// down for every (expert, pick) of experts picked by few tokens.
//
// Reference: moelan/kernels.py:712-782 (_moe_q4, one call per layer) and the
// per-expert int8 kernels (kernels.py:133-168), all f32.
//
// Design (sm_100a):
//  * Weights live in the device tile layout: 16-row tiles, each a contiguous
//    run of 1 KB (int4) / 2 KB (int8) blocks of 128 columns plus the blocks'
//    group scales.  One producer warp streams a row tile per stage into a
//    shared-memory ring with 1-D bulk copies on the TMA engine (mbarrier
//    completion); the whole working set moves HBM -> SMEM exactly once.
//  * Consumer warps split K: warp w owns quads [w*QPW, w*QPW+QPW) of every
//    tile.  Weights are unpacked to exact f16 (values -8..7 / -128..127) with
//    lop3/prmt + one f16x2 op per pair, and multiplied on the tensor cores by
//    mma.sync m16n8k16 against the activations split into two f16 pieces
//    (x * 2^e = hi + lo, 22 significant bits) laid along K, with f32
//    accumulation: the products are exact, so results match an f32 mat-vec to
//    rounding.  mma.sync is used because its operands come from registers:
//    a decode mat-vec is bound by HBM, and this keeps the unpacked weights
//    out of shared memory entirely (tcgen05 would need them staged).
//  * Each group of 32 columns is accumulated separately and scaled by its
//    group scale in f32; K-split partials are summed through shared memory.
//  * Phase 1 (gate|up) tiles interleave 8 gate rows with the 8 matching up
//    rows, so SiLU(gate) * up is formed in the epilogue and only the
//    activation row (P x I) goes back to HBM, with each pick's max |act|.
//  * Phase 2 (down) writes each pick's unweighted output row; the weighted
//    combine is a separate deterministic kernel.
//  * Work items are (expert, chunk of 8 picks, row tile), split contiguously
//    over a persistent grid so each CTA touches one or two experts.
#include <type_traits>

#include "mb_common.cuh"

namespace {

constexpr int kMaxQPW = 2;         // quads (128 columns) per consumer warp
constexpr int kMaxKW = 8;          // consumer warps
constexpr int kThreadsMax = (kMaxKW + 1) * 32;

struct Fmt {
    int data_bytes;   // per block: 1024 (int4) or 2048 (int8)
    int scale_f16;    // scale element 2 or 4 bytes
    int block_bytes;
};

__host__ __device__ inline Fmt fmt_info(int fmt)
{
    Fmt f;
    f.data_bytes = (fmt == MB_FMT_Q8_F16 || fmt == MB_FMT_Q8_F32) ? 2048 : 1024;
    f.scale_f16 = (fmt == MB_FMT_Q4_F16 || fmt == MB_FMT_Q8_F16) ? 1 : 0;
    f.block_bytes = f.data_bytes + 16 * 4 * (f.scale_f16 ? 2 : 4);
    return f;
}

struct DecodeArgs {
    const MbExpert* table;
    int E;
    int phase;        // 1: gate|up -> act, 2: down -> y
    int K;            // real input columns
    int NQ;           // quads per tile row (K padded to 128)
    int RT;           // row tiles
    int O_real;       // phase 1: I (act columns), phase 2: H (y columns)
    int src_ld;       // floats per input row (x: H, act: I_pad)
    int act_ld;       // I_pad
    int y_ld;         // H
    int QPW, KW;
    int stages, stage_bytes;
    const int32_t* counts;
    const int32_t* offsets;
    const int32_t* sorted_rows;
    const float* x;
    const int32_t* row_exp;
    float* act;
    unsigned* act_max;
    float* y;
    int max_rows;
    unsigned* status;
    // single-matrix mode (mb_matmul_t): one "expert" whose phase-2 matrix is
    // single_w, picked by single_n input rows 0..single_n-1
    const void* single_w;
    int single_n;
};

__device__ __forceinline__ int items_of(int n, int max_rows, int RT)
{
    return (n > 0 && n <= max_rows) ? ((n + 7) >> 3) * RT : 0;
}

// item -> (expert, chunk, row tile) by binary search over the item prefix.
__device__ __forceinline__ void locate(const int64_t* pre, int E, int RT, int64_t item, int& e, int& c, int& rt)
{
    int lo = 0, hi = E;  // pre[lo] <= item < pre[hi]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (pre[mid] <= item) lo = mid;
        else hi = mid;
    }
    e = lo;
    const int rem = (int)(item - pre[lo]);
    c = rem / RT;
    rt = rem - c * RT;
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

template <bool Q8, bool F16S>
__device__ __forceinline__ void scales4(const uint8_t* blk, int data_bytes, int row, float (&s)[4])
{
    if (F16S) {
        const uint2 v = *reinterpret_cast<const uint2*>(blk + data_bytes + row * 8);
        const __half2 a = *reinterpret_cast<const __half2*>(&v.x), b = *reinterpret_cast<const __half2*>(&v.y);
        s[0] = __low2float(a);
        s[1] = __high2float(a);
        s[2] = __low2float(b);
        s[3] = __high2float(b);
    } else {
        const float4 v = *reinterpret_cast<const float4*>(blk + data_bytes + row * 16);
        s[0] = v.x;
        s[1] = v.y;
        s[2] = v.z;
        s[3] = v.w;
    }
}

template <int FMT>
__global__ void __launch_bounds__(kThreadsMax, 1) moe_decode_kernel(const DecodeArgs a)
{
    constexpr bool Q8 = (FMT == MB_FMT_Q8_F16 || FMT == MB_FMT_Q8_F32);
    constexpr bool F16S = (FMT == MB_FMT_Q4_F16 || FMT == MB_FMT_Q8_F16);
    constexpr int kData = Q8 ? 2048 : 1024;
    constexpr int kBlock = kData + 16 * 4 * (F16S ? 2 : 4);

    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem;
    float* red = reinterpret_cast<float*>(smem + (size_t)a.stages * a.stage_bytes);  // [2][KW][16][8]
    uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * a.KW * 128);
    uint64_t* empty = full + a.stages;
    int64_t* pre = reinterpret_cast<int64_t*>(empty + a.stages);                      // [E+1]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(pre + a.E + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nthr = a.KW * 32;

    // ---- item prefix over experts (warp 0), barriers (thread 0)
    if (warp == 0) {
        int64_t run = 0;
        for (int base = 0; base < a.E; base += 32) {
            const int e = base + lane;
            int64_t v = 0;
            if (e < a.E) v = items_of(a.single_n ? (e == 0 ? a.single_n : 0) : a.counts[e], a.max_rows, a.RT);
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t u = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += u;
            }
            if (e < a.E) pre[e + 1] = run + v;
            run += __shfl_sync(0xffffffffu, v, 31);
        }
        if (lane == 0) pre[0] = 0;
    }
    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mb_mbar_init(&full[s], 1);
            mb_mbar_init(&empty[s], a.KW);
        }
        *abort_flag = 0;
        mb_fence_mbar_init();
    }
    __syncthreads();

    const int64_t total = pre[a.E];
    const int64_t lo = total * blockIdx.x / gridDim.x, hi = total * (blockIdx.x + 1) / gridDim.x;

    if (warp == a.KW) {  // ---------------- producer
        if (lane == 0) {
            int64_t it = 0;
            for (int64_t item = lo; item < hi; ++item, ++it) {
                const int s = (int)(it % a.stages);
                const int64_t use = it / a.stages;
                if (use > 0 && !mb_mbar_wait(&empty[s], (uint32_t)((use - 1) & 1), a.status, abort_flag)) break;
                int e, c, rt;
                locate(pre, a.E, a.RT, item, e, c, rt);
                const void* wbase = a.single_w ? a.single_w : (a.phase == 1 ? a.table[e].gu : a.table[e].down);
                const uint8_t* src = reinterpret_cast<const uint8_t*>(wbase) + (int64_t)rt * a.stage_bytes;
                mb_mbar_arrive_expect_tx(&full[s], (uint32_t)a.stage_bytes);
                mb_bulk_g2s(stages + (size_t)s * a.stage_bytes, src, (uint32_t)a.stage_bytes, &full[s]);
            }
        }
        return;
    }

    // ---------------- consumers
    const int q0 = warp * a.QPW;
    const int nq = max(0, min(a.QPW, a.NQ - q0));
    uint32_t bf[kMaxQPW][4][4][2];
    // 2^-e of the input rows this thread's epilogue outputs belong to:
    // phase 1 -> row (tid % 8); phase 2 -> row (o >> 4) of outputs o = tid + m * nthr
    float fs[4];
    int cur_e = -1, cur_c = -1, pbase = 0, nvalid = 0;
    float rmax = 0.0f;     // phase 1: running max |act| of this thread's pick (n = tid % 8)
    int64_t it = 0;

    auto row_exp_of = [&](int n) -> int {
        if (n >= nvalid) return 0;
        if (a.phase == 1) return a.row_exp[a.sorted_rows[pbase + n]];
        return mb_row_exponent(__uint_as_float(a.act_max[pbase + n]));
    };
    auto flush_max = [&]() {
        if (a.phase != 1 || cur_e < 0) return;
        float m = rmax;
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        const int n = tid & 7;
        if (lane < 8 && tid < 64 && n < nvalid) atomicMax(&a.act_max[pbase + n], __float_as_uint(m));
        rmax = 0.0f;
    };

    for (int64_t item = lo; item < hi; ++item, ++it) {
        int e, c, rt;
        locate(pre, a.E, a.RT, item, e, c, rt);
        if (e != cur_e || c != cur_c) {
            flush_max();
            cur_e = e;
            cur_c = c;
            const int n_e = a.single_n ? a.single_n : a.counts[e];
            pbase = (a.single_n ? 0 : a.offsets[e]) + 8 * c;
            nvalid = min(8, n_e - 8 * c);
            if (a.phase == 1) {
                fs[0] = pow2f(-row_exp_of(tid & 7));
            } else {
#pragma unroll
                for (int m = 0; m < 4; ++m) fs[m] = pow2f(-row_exp_of(min(7, (tid + m * nthr) >> 4)));
            }
            // B fragments: input row n = g of the chunk, split into f16 hi/lo of x * 2^e
            const bool valid = g < nvalid;
            const float* src = nullptr;
            float up = 1.0f;
            if (valid) {
                if (a.phase == 1) src = a.x + (int64_t)a.sorted_rows[pbase + g] * a.src_ld;
                else src = a.act + (int64_t)(pbase + g) * a.src_ld;
                up = pow2f(row_exp_of(g));
            }
#pragma unroll
            for (int qi = 0; qi < kMaxQPW; ++qi) {
#pragma unroll
                for (int gi = 0; gi < 4; ++gi) {
                    float v[8];
                    const int col0 = ((q0 + qi) * 4 + gi) * 32 + 8 * t;
                    if (valid && qi < nq && col0 + 8 <= a.K) {
                        const float4 u0 = *reinterpret_cast<const float4*>(src + col0);
                        const float4 u1 = *reinterpret_cast<const float4*>(src + col0 + 4);
                        v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
                        v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
                    } else {
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            v[j] = (valid && qi < nq && col0 + j < a.K) ? src[col0 + j] : 0.0f;
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float xa = v[j] * up, xb = v[j + 4] * up;
                        const __half ha = __float2half_rn(xa), hb = __float2half_rn(xb);
                        const __half la = __float2half_rn(xa - __half2float(ha));
                        const __half lb = __float2half_rn(xb - __half2float(hb));
                        bf[qi][gi][j][0] = mb_pack_h2(ha, hb);
                        bf[qi][gi][j][1] = mb_pack_h2(la, lb);
                    }
                }
            }
        }

        const int s = (int)(it % a.stages);
        const bool ok = mb_mbar_wait(&full[s], (uint32_t)((it / a.stages) & 1), a.status, abort_flag);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (ok) {
            const uint8_t* stage = stages + (size_t)s * a.stage_bytes;
#pragma unroll
            for (int qi = 0; qi < kMaxQPW; ++qi) {
                if (qi < nq) {
                    const uint8_t* blk = stage + (size_t)(q0 + qi) * kBlock;
                    uint32_t wg[8], wh[8];
                    if (Q8) {
                        const uint4 a0 = *reinterpret_cast<const uint4*>(blk + g * 64 + t * 16);
                        const uint4 a1 = *reinterpret_cast<const uint4*>(blk + 1024 + g * 64 + t * 16);
                        const uint4 b0 = *reinterpret_cast<const uint4*>(blk + (g + 8) * 64 + t * 16);
                        const uint4 b1 = *reinterpret_cast<const uint4*>(blk + 1024 + (g + 8) * 64 + t * 16);
                        wg[0] = a0.x; wg[1] = a0.y; wg[2] = a0.z; wg[3] = a0.w;
                        wg[4] = a1.x; wg[5] = a1.y; wg[6] = a1.z; wg[7] = a1.w;
                        wh[0] = b0.x; wh[1] = b0.y; wh[2] = b0.z; wh[3] = b0.w;
                        wh[4] = b1.x; wh[5] = b1.y; wh[6] = b1.z; wh[7] = b1.w;
                    } else {
                        const uint4 a0 = *reinterpret_cast<const uint4*>(blk + g * 64 + t * 16);
                        const uint4 b0 = *reinterpret_cast<const uint4*>(blk + (g + 8) * 64 + t * 16);
                        wg[0] = a0.x; wg[1] = a0.y; wg[2] = a0.z; wg[3] = a0.w;
                        wh[0] = b0.x; wh[1] = b0.y; wh[2] = b0.z; wh[3] = b0.w;
                    }
                    float sg[4], sh[4];
                    scales4<Q8, F16S>(blk, kData, g, sg);
                    scales4<Q8, F16S>(blk, kData, g + 8, sh);
#pragma unroll
                    for (int gi = 0; gi < 4; ++gi) {
                        uint32_t pg[4], ph[4];
                        if (Q8) {
                            unpack_q8(wg[2 * gi], wg[2 * gi + 1], pg);
                            unpack_q8(wh[2 * gi], wh[2 * gi + 1], ph);
                        } else {
                            unpack_q4(wg[gi], pg);
                            unpack_q4(wh[gi], ph);
                        }
                        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            mb_mma_f16(d, pg[j], ph[j], pg[j], ph[j], bf[qi][gi][j][0], bf[qi][gi][j][1], d);
                        acc[0] = fmaf(d[0], sg[gi], acc[0]);
                        acc[1] = fmaf(d[1], sg[gi], acc[1]);
                        acc[2] = fmaf(d[2], sh[gi], acc[2]);
                        acc[3] = fmaf(d[3], sh[gi], acc[3]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mb_mbar_arrive(&empty[s]);

        float* rb = red + ((it & 1) * a.KW + warp) * 128;
        *reinterpret_cast<float2*>(rb + g * 8 + 2 * t) = make_float2(acc[0], acc[1]);
        *reinterpret_cast<float2*>(rb + (g + 8) * 8 + 2 * t) = make_float2(acc[2], acc[3]);
        mb_named_barrier(1, nthr);

        const float* rr = red + (it & 1) * a.KW * 128;
        if (a.phase == 1) {
            for (int o = tid; o < 64; o += nthr) {
                const int jl = o >> 3, n = o & 7;
                float gate = 0.f, upv = 0.f;
                for (int w = 0; w < a.KW; ++w) {
                    gate += rr[w * 128 + jl * 8 + n];
                    upv += rr[w * 128 + (jl + 8) * 8 + n];
                }
                gate *= fs[0];
                upv *= fs[0];
                const float act = gate / (1.0f + expf(-gate)) * upv;
                if (n < nvalid) {
                    a.act[(int64_t)(pbase + n) * a.act_ld + 8 * rt + jl] = act;
                    rmax = fmaxf(rmax, fabsf(act));
                }
            }
        } else {
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int o = tid + m * nthr;
                if (o < 128) {
                    const int row = o & 15, n = o >> 4;
                    float v = 0.f;
                    for (int w = 0; w < a.KW; ++w) v += rr[w * 128 + row * 8 + n];
                    const int orow = 16 * rt + row;
                    if (n < nvalid && orow < a.O_real) a.y[(int64_t)(pbase + n) * a.y_ld + orow] = v * fs[m];
                }
            }
        }
    }
    flush_max();
}

struct Cfg {
    int QPW, KW, NQ, stages, stage_bytes;
    size_t smem;
};

Cfg plan(int fmt, int K, int E, int max_stage_smem)
{
    Cfg c;
    const Fmt f = fmt_info(fmt);
    c.NQ = (K + 127) / 128;
    c.QPW = c.NQ >= 2 ? 2 : 1;
    c.KW = (c.NQ + c.QPW - 1) / c.QPW;
    c.stage_bytes = c.NQ * f.block_bytes;
    c.stages = max_stage_smem / c.stage_bytes;
    if (c.stages > 8) c.stages = 8;
    if (c.stages < 2) c.stages = 2;
    c.smem = (size_t)c.stages * c.stage_bytes + 2 * c.KW * 128 * sizeof(float) + 2 * c.stages * sizeof(uint64_t) +
             (E + 1) * sizeof(int64_t) + 16;
    return c;
}

template <int FMT>
int launch_phase(const DecodeArgs& base, int K, int RT, cudaStream_t st)
{
    DecodeArgs a = base;
    const Cfg c = plan(FMT, K, a.E, 96 * 1024);
    if (c.KW > kMaxKW)
        return mb_fail(MB_EUNSUPPORTED, "mb_moe_decode: K=%d needs %d consumer warps (max %d)", K, c.KW, kMaxKW);
    a.K = K;
    a.NQ = c.NQ;
    a.RT = RT;
    a.QPW = c.QPW;
    a.KW = c.KW;
    a.stages = c.stages;
    a.stage_bytes = c.stage_bytes;
    auto kern = moe_decode_kernel<FMT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c.smem);
    if (e != cudaSuccess) return mb_fail(MB_ECUDA, "mb_moe_decode: smem attribute: %s", cudaGetErrorString(e));
    const int threads = (c.KW + 1) * 32;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, c.smem);
    if (e != cudaSuccess || per_sm < 1) per_sm = 1;
    const int grid = mb_num_sms() * per_sm;
    kern<<<grid, threads, c.smem, st>>>(a);
    return mb_check_launch("mb_moe_decode");
}

template <typename F>
int dispatch_fmt(int fmt, F&& f)
{
    switch (fmt) {
    case MB_FMT_Q4_F32: return f(std::integral_constant<int, MB_FMT_Q4_F32>());
    case MB_FMT_Q4_F16: return f(std::integral_constant<int, MB_FMT_Q4_F16>());
    case MB_FMT_Q8_F32: return f(std::integral_constant<int, MB_FMT_Q8_F32>());
    case MB_FMT_Q8_F16: return f(std::integral_constant<int, MB_FMT_Q8_F16>());
    default: return mb_fail(MB_EUNSUPPORTED, "mb_moe_decode: weight format %d", fmt);
    }
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
    cudaError_t e = cudaMemsetAsync(act_max, 0, P * sizeof(unsigned), st);
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
