// Router logits, softmax top-k, the stable permute by expert and the weighted
// combine (moelan/model.py:154-167, 226-236, 597; the scatter-adds of
// moelan/experts.py and kernels.py).
#include <float.h>

#include <algorithm>
#include <cooperative_groups.h>

#include "mb_common.cuh"

namespace {

// Router logits as a split-K f32 product: CTA (TT tokens, EE experts, 256-column
// K slice) writes the partial dot products of its slice; the top-k kernel adds
// the slices in slice order (deterministic) before the softmax.  Each of the
// 16 x 16 threads holds a (TT/16) x (EE/16) block of (token, expert) sums in
// registers, fed from 32-column chunks of x and the router staged k-major in
// shared memory; a sum runs over its slice's columns in order.
constexpr int kLgK = 256;   // columns per K slice
constexpr int kLgC = 32;    // columns per staged chunk

template <int TT, int EE>
__global__ void __launch_bounds__(256) router_partial_kernel(const float* __restrict__ x,
                                                             const float* __restrict__ router, int64_t T, int H,
                                                             int E, float* __restrict__ part,
                                                             float* __restrict__ part_max)
{
    constexpr int RT = TT / 16, RE = EE / 16;           // sums per thread: RT tokens x RE experts
    constexpr int PT = TT + 4, PE = EE + 4;             // padded rows (floats; 16-byte aligned)
    constexpr int TPR = 256 / TT, CPT = kLgC / TPR;     // |x| max: threads per token row, columns each
    static_assert(RT == 1 || RT == 2 || RT == 4, "token tile");
    static_assert(RE == 1 || RE == 2 || RE == 4, "expert tile");
    __shared__ __align__(16) float xs[kLgC][PT];        // [column][token]
    __shared__ __align__(16) float ws[kLgC][PE];        // [column][expert]
    mb_pdl_wait();
    mb_pdl_trigger();
    const int64_t t0 = (int64_t)blockIdx.x * TT;
    const int e0 = blockIdx.y * EE, ks = blockIdx.z, k0 = ks * kLgK;
    const int kn = min(kLgK, H - k0);
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;    // tokens RT*ty.., experts RE*tx..
    float acc[RT][RE];
#pragma unroll
    for (int a = 0; a < RT; ++a)
#pragma unroll
        for (int b = 0; b < RE; ++b) acc[a][b] = 0.f;
    float xmax = 0.f;
    for (int kc = 0; kc < kn; kc += kLgC) {
        // stage rows x 32 columns of each operand as float4s, transposed to column-major
        for (int i = threadIdx.x; i < TT * (kLgC / 4); i += 256) {
            const int r = i >> 3, c = (i & 7) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t0 + r < T && kc + c < kn) v = *reinterpret_cast<const float4*>(x + (t0 + r) * H + k0 + kc + c);
            xs[c][r] = v.x, xs[c + 1][r] = v.y, xs[c + 2][r] = v.z, xs[c + 3][r] = v.w;
        }
        for (int i = threadIdx.x; i < EE * (kLgC / 4); i += 256) {
            const int r = i >> 3, c = (i & 7) * 4;
            float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e0 + r < E && kc + c < kn)
                u = *reinterpret_cast<const float4*>(router + (int64_t)(e0 + r) * H + k0 + kc + c);
            ws[c][r] = u.x, ws[c + 1][r] = u.y, ws[c + 2][r] = u.z, ws[c + 3][r] = u.w;
        }
        __syncthreads();
#pragma unroll 8
        for (int c = 0; c < kLgC; ++c) {
            float xa[RT], wa[RE];
#pragma unroll
            for (int a = 0; a < RT; ++a) xa[a] = xs[c][RT * ty + a];
#pragma unroll
            for (int b = 0; b < RE; ++b) wa[b] = ws[c][RE * tx + b];
#pragma unroll
            for (int a = 0; a < RT; ++a)
#pragma unroll
                for (int b = 0; b < RE; ++b) acc[a][b] = fmaf(xa[a], wa[b], acc[a][b]);
        }
        if (part_max && blockIdx.y == 0) {
            const int r = threadIdx.x / TPR, c = (threadIdx.x % TPR) * CPT;
#pragma unroll
            for (int q = 0; q < CPT; ++q) xmax = fmaxf(xmax, fabsf(xs[c + q][r]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < RT; ++a) {
        const int64_t t = t0 + RT * ty + a;
        if (t >= T) continue;
#pragma unroll
        for (int b = 0; b < RE; ++b) {
            const int e = e0 + RE * tx + b;
            if (e < E) part[((int64_t)ks * T + t) * E + e] = acc[a][b];
        }
    }
    if (part_max && blockIdx.y == 0) {                        // this slice's largest |x| of each token
#pragma unroll
        for (int o = 1; o < TPR; o <<= 1) xmax = fmaxf(xmax, __shfl_xor_sync(0xffffffffu, xmax, o));
        const int r = threadIdx.x / TPR;
        if (threadIdx.x % TPR == 0 && t0 + r < T) part_max[(int64_t)ks * T + t0 + r] = xmax;
    }
}

// Small batches: CTA (16 tokens, 16 experts, K slice) stages the whole slice of
// both operands in one round trip, token- and expert-major, and each thread
// forms one sum four columns at a time.
__global__ void __launch_bounds__(256) router_partial_small_kernel(const float* __restrict__ x,
                                                                   const float* __restrict__ router, int64_t T,
                                                                   int H, int E, float* __restrict__ part,
                                                                   float* __restrict__ part_max)
{
    __shared__ __align__(16) float xs[16][kLgK + 4];
    __shared__ __align__(16) float ws[16][kLgK + 4];
    mb_pdl_wait();
    mb_pdl_trigger();
    const int64_t t0 = (int64_t)blockIdx.x * 16;
    const int e0 = blockIdx.y * 16, ks = blockIdx.z, k0 = ks * kLgK;
    const int kn = min(kLgK, H - k0);
    for (int i = threadIdx.x; i < 16 * (kLgK / 4); i += 256) {
        const int r = i / (kLgK / 4), c = (i % (kLgK / 4)) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f), u = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t0 + r < T && c < kn) v = *reinterpret_cast<const float4*>(x + (t0 + r) * H + k0 + c);
        if (e0 + r < E && c < kn) u = *reinterpret_cast<const float4*>(router + (int64_t)(e0 + r) * H + k0 + c);
        *reinterpret_cast<float4*>(&xs[r][c]) = v;
        *reinterpret_cast<float4*>(&ws[r][c]) = u;
    }
    __syncthreads();
    const int ti = threadIdx.x >> 4, ej = threadIdx.x & 15;
    float acc = 0.f;
#pragma unroll 8
    for (int c = 0; c < kLgK; c += 4) {
        const float4 xv = *reinterpret_cast<const float4*>(&xs[ti][c]);
        const float4 wv = *reinterpret_cast<const float4*>(&ws[ej][c]);
        acc = fmaf(xv.x, wv.x, acc);
        acc = fmaf(xv.y, wv.y, acc);
        acc = fmaf(xv.z, wv.z, acc);
        acc = fmaf(xv.w, wv.w, acc);
    }
    const int64_t t = t0 + ti;
    if (t < T && e0 + ej < E) part[((int64_t)ks * T + t) * E + e0 + ej] = acc;
    if (part_max && blockIdx.y == 0) {  // this slice's largest |x| of each token
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int r = warp; r < 16; r += 8) {
            float m = 0.f;
            for (int c = lane; c < kLgK; c += 32) m = fmaxf(m, fabsf(xs[r][c]));
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0 && t0 + r < T) part_max[(int64_t)ks * T + t0 + r] = m;
        }
    }
}

__global__ void row_exponent_kernel(const float* __restrict__ x, int64_t T, int H, int32_t* __restrict__ row_exp)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= T) return;
    const float* xr = x + t * H;
    float m = 0.0f;
    for (int h = lane; h < H; h += 32) m = fmaxf(m, fabsf(xr[h]));
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) row_exp[t] = mb_row_exponent(m);
}

// Softmax top-k, one warp per token.  Experts are ranked by logit (softmax is
// monotone), equal logits by lower id -- the order of the reference's stable
// argsort of the probabilities (model.py:154-157) wherever distinct logits give
// distinct probabilities.  Weights are the f32 softmax probabilities of the
// picks, renormalised over the k picks when asked (model.py:164-166).
constexpr int kTopkMaxPerLane = 32;  // E <= 1024

// With nslices > 0 the logits are first summed from nslices partial slices
// (slice s at logits + s*T*E) in slice order, written to out_logits when
// given, and row_exp gets each token's exponent from the slices' maxima.
// PER = experts per lane rounded up to a power of two (E <= 32 * PER).
template <int PER>
__global__ void router_topk_kernel(const float* __restrict__ logits, int nslices, const float* __restrict__ part_max,
                                   float* __restrict__ out_logits, int32_t* __restrict__ row_exp, int64_t T, int E,
                                   int k, int normalize, int32_t* __restrict__ idx, float* __restrict__ w)
{
    mb_pdl_wait();
    mb_pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= T) return;
    constexpr int per = PER;
    float v[PER];
    float m = -FLT_MAX;
    if (nslices > 0) {
        // sum the slices in slice order; four slices' loads per element are in flight at once
#pragma unroll
        for (int i = 0; i < PER; ++i) v[i] = 0.f;
        const int64_t sstride = T * E;
        for (int sl = 0; sl < nslices; sl += 4) {
            const int nl = min(4, nslices - sl);
#pragma unroll
            for (int i = 0; i < PER; ++i) {
                const int e = i * 32 + lane;
                if (i < per && e < E) {
                    const float* src = logits + ((int64_t)sl * T + t) * E + e;
                    const float l0 = src[0];
                    const float l1 = nl > 1 ? src[sstride] : 0.f;
                    const float l2 = nl > 2 ? src[2 * sstride] : 0.f;
                    const float l3 = nl > 3 ? src[3 * sstride] : 0.f;
                    float acc = v[i] + l0;
                    if (nl > 1) acc += l1;
                    if (nl > 2) acc += l2;
                    if (nl > 3) acc += l3;
                    v[i] = acc;
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = i * 32 + lane;
        float val = -INFINITY;
        if (i < per && e < E) {
            if (nslices > 0) {
                val = v[i];
                if (out_logits) out_logits[t * E + e] = val;
            } else {
                val = logits[t * E + e];
            }
            m = fmaxf(m, val);
        }
        v[i] = val;
    }
    if (row_exp && part_max) {
        float xm = 0.f;
        for (int sl = lane; sl < nslices; sl += 32) xm = fmaxf(xm, part_max[(int64_t)sl * T + t]);
        for (int o = 16; o; o >>= 1) xm = fmaxf(xm, __shfl_xor_sync(0xffffffffu, xm, o));
        if (lane == 0) row_exp[t] = mb_row_exponent(xm);
    }
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = i * 32 + lane;
        if (i < per && e < E) sum += expf(v[i] - m);
    }
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    uint32_t taken = 0;  // bit i: element i of this lane already picked
    float my_p = 0.f, psum = 0.f;
    int my_i = -1;
    for (int j = 0; j < k; ++j) {
        float bv = -INFINITY;
        int bi = INT32_MAX;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int e = i * 32 + lane;
            if (i < per && e < E && !((taken >> i) & 1u) && (v[i] > bv || (v[i] == bv && e < bi))) {
                bv = v[i];
                bi = e;
            }
        }
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (bi != INT32_MAX && (bi & 31) == lane) taken |= 1u << (bi >> 5);
        const float p = (bi == INT32_MAX) ? 0.0f : expf(bv - m) / sum;
        if (lane == j) {
            my_p = p;
            my_i = bi;
        }
        psum += p;
    }
    if (lane < k) {
        idx[t * k + lane] = my_i;
        w[t * k + lane] = normalize ? my_p / psum : my_p;
    }
}

// ---- stable counting sort of the T*k picks by expert ---------------------------
// One thread-block cluster of nc CTAs (1 for small P, up to 8): CTA c takes the
// c-th contiguous chunk of picks and each of its warps a contiguous sub-chunk,
// so (CTA, warp, lane) order is pick order and the sort is stable.  Each CTA
// counts its picks per warp in shared memory; after a cluster barrier every
// CTA reads the other CTAs' per-expert totals through distributed shared
// memory, derives the expert offsets (all CTAs compute the same scan) and the
// base of its own picks, and scatters them.  CTA 0 writes the per-expert
// outputs.
constexpr int kPermWarps = 32;
constexpr int kPermBatch = 16;      // picks per lane whose loads are in flight together
constexpr int kPermMaxCluster = 8;  // portable cluster size
constexpr int kPermPerCta = 2048;   // picks per CTA before another CTA joins

__global__ void __launch_bounds__(kPermWarps * 32) permute_kernel(
    const int32_t* __restrict__ idx, const float* __restrict__ w, int64_t P, int k, int E, int32_t* counts,
    int32_t* offsets, int32_t* sorted_rows, float* sorted_w, int32_t* inv, int32_t* uexperts, int32_t* uoffsets,
    int32_t* n_unique)
{
    mb_pdl_wait();
    mb_pdl_trigger();
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int nc = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
    extern __shared__ int32_t sm[];
    int32_t* cnt = sm;                    // [kPermWarps][E]: per-warp counts, then running bases
    int32_t* tot = sm + kPermWarps * E;   // [E]: this CTA's counts per expert (read by the other CTAs)
    int32_t* gtot = tot + E;              // [E]: the cluster's counts per expert
    int32_t* bef = gtot + E;              // [E]: picks of expert e in lower-ranked CTAs, then this CTA's base
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < kPermWarps * E; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    const int64_t per_cta = ((P + nc - 1) / nc + 31) / 32 * 32;
    const int64_t clo = min(P, (int64_t)rank * per_cta), chi = min(P, clo + per_cta);
    const int64_t chunk = ((chi - clo + kPermWarps - 1) / kPermWarps + 31) / 32 * 32;
    const int64_t lo = min(chi, clo + warp * chunk), hi = min(chi, lo + chunk);
    int32_t* my = cnt + warp * E;
    // a warp walks its sub-chunk kPermBatch x 32 picks at a time, all their loads issued first
    for (int64_t b0 = lo; b0 < hi; b0 += 32 * kPermBatch) {
        int ev[kPermBatch];
#pragma unroll
        for (int j = 0; j < kPermBatch; ++j) {
            const int64_t i = b0 + 32 * j + lane;
            ev[j] = i < hi ? idx[i] : -1;
        }
#pragma unroll
        for (int j = 0; j < kPermBatch; ++j) {
            if (b0 + 32 * j >= hi) break;                 // warp-uniform
            const int64_t i = b0 + 32 * j + lane;
            const bool valid = i < hi;
            const int e = ev[j];
            const unsigned act = __ballot_sync(0xffffffffu, valid);
            if (valid) {
                const unsigned peers = __match_any_sync(act, e);
                if (e >= 0 && e < E && lane == __ffs(peers) - 1) my[e] += __popc(peers);
            }
            __syncwarp();
        }
    }
    __syncthreads();
    // this CTA's totals and per-warp bases within the CTA
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int32_t run = 0;
        for (int q = 0; q < kPermWarps; ++q) {
            const int32_t c = cnt[q * E + e];
            cnt[q * E + e] = run;
            run += c;
        }
        tot[e] = run;
    }
    if (nc > 1) {
        cluster.sync();                               // every CTA's totals are visible
        for (int e = threadIdx.x; e < E; e += blockDim.x) {
            int32_t all = 0, before = 0;
            for (int c = 0; c < nc; ++c) {
                const int32_t v = cluster.map_shared_rank(tot, c)[e];
                all += v;
                before += c < rank ? v : 0;
            }
            gtot[e] = all;
            bef[e] = before;
        }
        cluster.sync();                               // no CTA reads another's memory after this
    } else {
        __syncthreads();
        for (int e = threadIdx.x; e < E; e += blockDim.x) {
            gtot[e] = tot[e];
            bef[e] = 0;
        }
        __syncthreads();
    }
    {  // exclusive scan of the totals over experts, and the compact list of used experts
        __shared__ int32_t wsum[kPermWarps], wcnt[kPermWarps];
        const int e = threadIdx.x;                    // blockDim.x = 1024 >= E
        const int32_t c = e < E ? gtot[e] : 0;
        int32_t inc = c, used = (c > 0);
        for (int o = 1; o < 32; o <<= 1) {
            const int32_t u = __shfl_up_sync(0xffffffffu, inc, o), v = __shfl_up_sync(0xffffffffu, used, o);
            if (lane >= o) {
                inc += u;
                used += v;
            }
        }
        if (lane == 31) {
            wsum[warp] = inc;
            wcnt[warp] = used;
        }
        __syncthreads();
        if (warp == 0) {
            int32_t s1 = wsum[lane], s2 = wcnt[lane];
            for (int o = 1; o < 32; o <<= 1) {
                const int32_t u = __shfl_up_sync(0xffffffffu, s1, o), v = __shfl_up_sync(0xffffffffu, s2, o);
                if (lane >= o) {
                    s1 += u;
                    s2 += v;
                }
            }
            wsum[lane] = s1;
            wcnt[lane] = s2;
        }
        __syncthreads();
        const int32_t excl = inc - c + (warp ? wsum[warp - 1] : 0);
        const int32_t uidx = used - (c > 0) + (warp ? wcnt[warp - 1] : 0);
        if (e < E) {
            if (rank == 0) {
                offsets[e] = excl;
                if (counts) counts[e] = c;
                if (c > 0) {
                    if (uexperts) uexperts[uidx] = e;
                    if (uoffsets) uoffsets[uidx] = excl;
                }
                if (e == E - 1) {
                    offsets[E] = excl + c;
                    if (uoffsets) uoffsets[uidx + (c > 0)] = excl + c;
                    if (n_unique) *n_unique = uidx + (c > 0);
                }
            }
            bef[e] += excl;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int32_t base = bef[e];
        for (int q = 0; q < kPermWarps; ++q) cnt[q * E + e] += base;
    }
    __syncthreads();
    for (int64_t b0 = lo; b0 < hi; b0 += 32 * kPermBatch) {
        int ev[kPermBatch];
        float wv[kPermBatch];
#pragma unroll
        for (int j = 0; j < kPermBatch; ++j) {
            const int64_t i = b0 + 32 * j + lane;
            ev[j] = i < hi ? idx[i] : -1;
            wv[j] = (i < hi && w) ? w[i] : 1.0f;
        }
#pragma unroll
        for (int j = 0; j < kPermBatch; ++j) {
            if (b0 + 32 * j >= hi) break;                 // warp-uniform
            const int64_t i = b0 + 32 * j + lane;
            const bool valid = i < hi;
            const int e = ev[j];
            const unsigned act = __ballot_sync(0xffffffffu, valid);
            int32_t pos = -1;
            unsigned peers = 0;
            if (valid && e >= 0 && e < E) {
                peers = __match_any_sync(act, e);
                pos = my[e] + __popc(peers & ((1u << lane) - 1u));
            } else if (valid) {
                peers = __match_any_sync(act, e);
            }
            __syncwarp();
            if (valid && e >= 0 && e < E) {
                if (lane == __ffs(peers) - 1) my[e] += __popc(peers);
                sorted_rows[pos] = (int32_t)(i / k);
                if (sorted_w) sorted_w[pos] = wv[j];
            }
            if (valid && inv) inv[i] = pos;
            __syncwarp();
        }
    }
}

// out[r] (+)= sum_i pair_w[i] * y[pair_idx[i]] in entry order; one thread per
// 4 columns of a row.  Rows with up to 8 entries issue all their loads first.
__global__ void combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ row_ptr,
                               const int32_t* __restrict__ pair_idx, const float* __restrict__ pair_w, int64_t T,
                               int k, int H, int accumulate, float* __restrict__ out)
{
    mb_pdl_wait();
    mb_pdl_trigger();
    const int64_t r = blockIdx.y;
    const int h = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (h >= H) return;
    const int64_t i0 = row_ptr ? row_ptr[r] : r * k;
    const int64_t i1 = row_ptr ? row_ptr[r + 1] : r * k + k;
    float4 acc = accumulate ? *reinterpret_cast<const float4*>(out + r * H + h) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t b = i0; b < i1; b += 8) {
        int32_t p[8];
        float wt[8];
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            p[j] = (b + j < i1) ? pair_idx[b + j] : -1;
            wt[j] = (b + j < i1) ? pair_w[b + j] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
            v[j] = p[j] >= 0 ? *reinterpret_cast<const float4*>(y + (int64_t)p[j] * H + h) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (p[j] < 0) continue;
            acc.x = fmaf(wt[j], v[j].x, acc.x);
            acc.y = fmaf(wt[j], v[j].y, acc.y);
            acc.z = fmaf(wt[j], v[j].z, acc.z);
            acc.w = fmaf(wt[j], v[j].w, acc.w);
        }
    }
    *reinterpret_cast<float4*>(out + r * H + h) = acc;
}

}  // namespace

static int router_slices(int H) { return (H + kLgK - 1) / kLgK; }

static int launch_topk(const float* logits, int nslices, const float* part_max, float* out_logits, int32_t* row_exp,
                       int64_t T, int E, int k, int normalize, int32_t* idx, float* w, cudaStream_t st)
{
    const dim3 grid((unsigned)((T + 7) / 8)), block(256);
    const int per = (E + 31) / 32;
    auto kern = per <= 1 ? router_topk_kernel<1>
              : per <= 2 ? router_topk_kernel<2>
              : per <= 4 ? router_topk_kernel<4>
              : per <= 8 ? router_topk_kernel<8>
              : per <= 16 ? router_topk_kernel<16>
                          : router_topk_kernel<32>;
    const cudaError_t e = mb_launch_pdl(kern, grid, block, 0, st, logits, nslices, part_max, out_logits, row_exp, T,
                                        E, k, normalize, idx, w);
    if (e != cudaSuccess) return mb_fail(MB_ECUDA, "router top-k launch: %s", cudaGetErrorString(e));
    return MB_OK;
}

__global__ void sum_slices_kernel(const float* __restrict__ part, int nslices, const float* __restrict__ part_max,
                                  int64_t T, int E, float* __restrict__ logits, int32_t* __restrict__ row_exp)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < T * E) {
        float v = 0.f;
        for (int sl = 0; sl < nslices; ++sl) v += part[(int64_t)sl * T * E + i];
        logits[i] = v;
    }
    if (row_exp && i < T) {
        float m = 0.f;
        for (int sl = 0; sl < nslices; ++sl) m = fmaxf(m, part_max[(int64_t)sl * T + i]);
        row_exp[i] = mb_row_exponent(m);
    }
}

static int launch_partial(const float* x, const float* router, int64_t T, int H, int E, float* part,
                          float* part_max, cudaStream_t st)
{
    MB_REQUIRE(x && router && part, "router logits: null pointer");
    MB_REQUIRE(T >= 0 && H > 0 && E > 0 && H % 4 == 0, "router logits: bad shape (H must be a multiple of 4)");
    MB_REQUIRE(((uintptr_t)x & 15) == 0 && ((uintptr_t)router & 15) == 0, "router logits: x/router not 16-byte aligned");
    MB_REQUIRE((T + 15) / 16 <= 0x7fffffff && (E + 15) / 16 <= 65535, "router logits: too large");
    if (T == 0) return MB_OK;
    cudaError_t e;
    if (T >= 512) {
        const dim3 grid((unsigned)((T + 63) / 64), (E + 63) / 64, router_slices(H));
        e = mb_launch_pdl(router_partial_kernel<64, 64>, grid, dim3(256), 0, st, x, router, T, H, E, part, part_max);
    } else {
        const dim3 grid((unsigned)((T + 15) / 16), (E + 15) / 16, router_slices(H));
        e = mb_launch_pdl(router_partial_small_kernel, grid, dim3(256), 0, st, x, router, T, H, E, part, part_max);
    }
    if (e != cudaSuccess) return mb_fail(MB_ECUDA, "router logits launch: %s", cudaGetErrorString(e));
    return MB_OK;
}

extern "C" int64_t mb_router_workspace_bytes(int64_t T, int H, int E)
{
    const int64_t ns = router_slices(H);
    return ((ns * T * E * 4 + 255) / 256) * 256 + ((ns * T * 4 + 255) / 256) * 256;
}

extern "C" int mb_router_logits(const float* x, const float* router, int64_t T, int H, int E, float* logits,
                                int32_t* row_exp, void* workspace, int64_t workspace_bytes, void* stream)
{
    MB_REQUIRE(logits && workspace, "mb_router_logits: null pointer");
    MB_REQUIRE(workspace_bytes >= mb_router_workspace_bytes(T, H, E), "mb_router_logits: workspace too small");
    const int ns = router_slices(H);
    float* part = reinterpret_cast<float*>(workspace);
    float* pmax = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + (((int64_t)ns * T * E * 4 + 255) / 256) * 256);
    int rc = launch_partial(x, router, T, H, E, part, pmax, mb_stream(stream));
    if (rc || T == 0) return rc;
    sum_slices_kernel<<<(unsigned)((T * E + 255) / 256), 256, 0, mb_stream(stream)>>>(part, ns, pmax, T, E, logits,
                                                                                     row_exp);
    return mb_check_launch("mb_router_logits");
}

extern "C" int mb_router_route(const float* x, const float* router, int64_t T, int H, int E, int k, int normalize,
                               float* logits, int32_t* row_exp, int32_t* idx, float* w, void* workspace,
                               int64_t workspace_bytes, void* stream)
{
    MB_REQUIRE(idx && w && workspace, "mb_router_route: null pointer");
    MB_REQUIRE(E <= 32 * kTopkMaxPerLane && k > 0 && k <= E && k <= 32, "mb_router_route: E=%d k=%d", E, k);
    MB_REQUIRE(workspace_bytes >= mb_router_workspace_bytes(T, H, E), "mb_router_route: workspace too small");
    const int ns = router_slices(H);
    float* part = reinterpret_cast<float*>(workspace);
    float* pmax = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + (((int64_t)ns * T * E * 4 + 255) / 256) * 256);
    int rc = launch_partial(x, router, T, H, E, part, pmax, mb_stream(stream));
    if (rc || T == 0) return rc;
    rc = launch_topk(part, ns, pmax, logits, row_exp, T, E, k, normalize, idx, w, mb_stream(stream));
    if (rc) return rc;
    return mb_check_launch("mb_router_route");
}

extern "C" int mb_row_exponents(const float* x, int64_t T, int H, int32_t* row_exp, void* stream)
{
    MB_REQUIRE(x && row_exp, "mb_row_exponents: null pointer");
    if (T == 0) return MB_OK;
    row_exponent_kernel<<<(unsigned)((T + 7) / 8), 256, 0, mb_stream(stream)>>>(x, T, H, row_exp);
    return mb_check_launch("mb_row_exponents");
}

extern "C" int mb_router_topk(const float* logits, int64_t T, int E, int k, int normalize, int32_t* idx, float* w,
                              void* stream)
{
    MB_REQUIRE(logits && idx && w, "mb_router_topk: null pointer");
    MB_REQUIRE(E > 0 && E <= 32 * kTopkMaxPerLane, "mb_router_topk: E=%d outside 1..1024", E);
    MB_REQUIRE(k > 0 && k <= E && k <= 32, "mb_router_topk: k=%d outside 1..min(E,32)", k);
    if (T == 0) return MB_OK;
    const int rc = launch_topk(logits, 0, nullptr, nullptr, nullptr, T, E, k, normalize, idx, w, mb_stream(stream));
    if (rc) return rc;
    return mb_check_launch("mb_router_topk");
}

extern "C" int mb_permute(const int32_t* idx, const float* w, int64_t T, int k, int E, int32_t* counts,
                          int32_t* offsets, int32_t* sorted_rows, float* sorted_w, int32_t* inv, int32_t* uexperts,
                          int32_t* uoffsets, int32_t* n_unique, void* stream)
{
    MB_REQUIRE(idx && offsets && sorted_rows, "mb_permute: null pointer");
    MB_REQUIRE(E > 0 && E <= 1024 && k > 0, "mb_permute: E=%d k=%d", E, k);
    const int64_t P = T * k;
    MB_REQUIRE(P >= 0 && P <= 65536, "mb_permute: T*k=%lld outside 0..65536", (long long)P);
    const size_t smem = sizeof(int32_t) * ((size_t)kPermWarps * E + 3 * (size_t)E);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return mb_fail(MB_ECUDA, "mb_permute: %s", cudaGetErrorString(e));
    }
    const int nc = (int)std::min<int64_t>(kPermMaxCluster, std::max<int64_t>(1, (P + kPermPerCta - 1) / kPermPerCta));
    if (nc == 1) {  // one CTA: no cluster
        const cudaError_t e = mb_launch_pdl(permute_kernel, dim3(1), dim3(kPermWarps * 32), smem, mb_stream(stream), idx,
                                            w, P, k, E, counts, offsets, sorted_rows, sorted_w, inv, uexperts,
                                            uoffsets, n_unique);
        if (e != cudaSuccess) return mb_fail(MB_ECUDA, "mb_permute launch: %s", cudaGetErrorString(e));
        return MB_OK;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nc);
    cfg.blockDim = dim3(kPermWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = mb_stream(stream);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = nc;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // see mb_launch_pdl
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t le = cudaLaunchKernelEx(&cfg, permute_kernel, idx, w, P, k, E, counts, offsets, sorted_rows, sorted_w,
                                        inv, uexperts, uoffsets, n_unique);
    if (le != cudaSuccess) return mb_fail(MB_ECUDA, "mb_permute launch: %s", cudaGetErrorString(le));
    return mb_check_launch("mb_permute");
}

extern "C" int mb_unpermute_combine(const float* y, const int32_t* row_ptr, const int32_t* pair_idx,
                                    const float* pair_w, int64_t T, int k, int H, int accumulate, float* out,
                                    void* stream)
{
    MB_REQUIRE(y && pair_idx && pair_w && out, "mb_unpermute_combine: null pointer");
    MB_REQUIRE(H % 4 == 0 && ((uintptr_t)y & 15) == 0 && ((uintptr_t)out & 15) == 0,
               "mb_unpermute_combine: H must be a multiple of 4 and y/out 16-byte aligned");
    MB_REQUIRE(T <= 65535, "mb_unpermute_combine: T=%lld above 65535", (long long)T);
    if (T == 0) return MB_OK;
    dim3 grid((H / 4 + 255) / 256, (unsigned)T);
    const cudaError_t e = mb_launch_pdl(combine_kernel, grid, dim3(256), 0, mb_stream(stream), y, row_ptr, pair_idx,
                                        pair_w, T, k, H, accumulate, out);
    if (e != cudaSuccess) return mb_fail(MB_ECUDA, "mb_unpermute_combine launch: %s", cudaGetErrorString(e));
    return mb_check_launch("mb_unpermute_combine");
}
