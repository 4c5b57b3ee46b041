// Router logits, softmax top-k, the stable permute by expert and the weighted
// combine (moelan/model.py:154-167, 226-236, 597; the scatter-adds of
// moelan/experts.py and kernels.py).
#include <float.h>

#include "mb_common.cuh"

namespace {

constexpr int kLogitTokens = 8;   // tokens per CTA of the logits kernel
constexpr int kLogitExperts = 8;  // experts per CTA (one per warp)

// logits[t][e] = sum_h x[t][h] * router[e][h].  CTAs with blockIdx.x == 0
// also write each token's row exponent (its largest |x|) when asked.
__global__ void __launch_bounds__(256) router_logits_kernel(const float* __restrict__ x,
                                                            const float* __restrict__ router, int64_t T, int H, int E,
                                                            float* __restrict__ logits, int32_t* __restrict__ row_exp)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * kLogitExperts + warp;
    const int64_t t0 = (int64_t)blockIdx.y * kLogitTokens;
    const int nt = (int)((T - t0) < kLogitTokens ? (T - t0) : kLogitTokens);
    const bool vec = (H & 3) == 0;
    if (e < E) {
        float acc[kLogitTokens];
#pragma unroll
        for (int i = 0; i < kLogitTokens; ++i) acc[i] = 0.0f;
        const float* w = router + (int64_t)e * H;
        if (vec) {
            for (int h = lane * 4; h < H; h += 128) {
                const float4 wv = *reinterpret_cast<const float4*>(w + h);
#pragma unroll
                for (int i = 0; i < kLogitTokens; ++i) {
                    if (i < nt) {
                        const float4 xv = *reinterpret_cast<const float4*>(x + (t0 + i) * H + h);
                        acc[i] = fmaf(wv.x, xv.x, fmaf(wv.y, xv.y, fmaf(wv.z, xv.z, fmaf(wv.w, xv.w, acc[i]))));
                    }
                }
            }
        } else {
            for (int h = lane; h < H; h += 32) {
                const float wv = w[h];
#pragma unroll
                for (int i = 0; i < kLogitTokens; ++i)
                    if (i < nt) acc[i] = fmaf(wv, x[(t0 + i) * H + h], acc[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < kLogitTokens; ++i) {
            float v = acc[i];
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && i < nt) logits[(t0 + i) * E + e] = v;
        }
    }
    if (row_exp && blockIdx.x == 0 && warp < nt) {
        const float* xr = x + (t0 + warp) * H;
        float m = 0.0f;
        for (int h = lane; h < H; h += 32) m = fmaxf(m, fabsf(xr[h]));
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) row_exp[t0 + warp] = mb_row_exponent(m);
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

__global__ void router_topk_kernel(const float* __restrict__ logits, int64_t T, int E, int k, int normalize,
                                   int32_t* __restrict__ idx, float* __restrict__ w)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    if (t >= T) return;
    const float* lg = logits + t * E;
    const int per = (E + 31) / 32;
    float v[kTopkMaxPerLane];
    float m = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < kTopkMaxPerLane; ++i) {
        const int e = i * 32 + lane;
        v[i] = (i < per && e < E) ? lg[e] : -INFINITY;
        if (i < per && e < E) m = fmaxf(m, v[i]);
    }
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < kTopkMaxPerLane; ++i) {
        const int e = i * 32 + lane;
        if (i < per && e < E) sum += expf(v[i] - m);
    }
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    uint32_t taken = 0;  // bit i: element i of this lane already picked
    float pk[32];
    int ik[32];
    float psum = 0.0f;
    for (int j = 0; j < k; ++j) {
        float bv = -INFINITY;
        int bi = INT32_MAX;
#pragma unroll
        for (int i = 0; i < kTopkMaxPerLane; ++i) {
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
        if (j < 32) {
            pk[j] = p;
            ik[j] = bi;
        }
        psum += p;
    }
    if (lane == 0) {
        for (int j = 0; j < k && j < 32; ++j) {
            idx[t * k + j] = ik[j];
            w[t * k + j] = normalize ? pk[j] / psum : pk[j];
        }
    }
}

// ---- stable counting sort of the T*k picks by expert ---------------------------
constexpr int kPermWarps = 32;

__global__ void __launch_bounds__(kPermWarps * 32) permute_kernel(
    const int32_t* __restrict__ idx, const float* __restrict__ w, int64_t P, int k, int E, int32_t* counts,
    int32_t* offsets, int32_t* sorted_rows, float* sorted_w, int32_t* inv, int32_t* uexperts, int32_t* uoffsets,
    int32_t* n_unique)
{
    extern __shared__ int32_t sm[];
    int32_t* cnt = sm;                    // [kPermWarps][E]: per-warp counts, then running bases
    int32_t* tot = sm + kPermWarps * E;   // [E + 1]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < kPermWarps * E; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    const int64_t chunk = ((P + kPermWarps - 1) / kPermWarps + 31) / 32 * 32;
    const int64_t lo = warp * chunk, hi = (lo + chunk < P) ? lo + chunk : P;
    int32_t* my = cnt + warp * E;
    for (int64_t b = lo; b < hi; b += 32) {
        const int64_t i = b + lane;
        const bool valid = i < hi;
        const int e = valid ? idx[i] : -1;
        const unsigned act = __ballot_sync(0xffffffffu, valid);
        if (valid) {
            const unsigned peers = __match_any_sync(act, e);
            if (e >= 0 && e < E && lane == __ffs(peers) - 1) my[e] += __popc(peers);
        }
        __syncwarp();
    }
    __syncthreads();
    // totals and per-warp bases
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int32_t run = 0;
        for (int q = 0; q < kPermWarps; ++q) {
            const int32_t c = cnt[q * E + e];
            cnt[q * E + e] = run;
            run += c;
        }
        tot[e] = run;
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // exclusive scan over experts (E <= 1024: serial is fine)
        int32_t run = 0, u = 0;
        for (int e = 0; e < E; ++e) {
            const int32_t c = tot[e];
            offsets[e] = run;
            if (counts) counts[e] = c;
            if (c > 0) {
                if (uexperts) uexperts[u] = e;
                if (uoffsets) uoffsets[u] = run;
                ++u;
            }
            tot[e] = run;
            run += c;
        }
        offsets[E] = run;
        if (uoffsets) uoffsets[u] = run;
        if (n_unique) *n_unique = u;
        tot[E] = run;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int32_t base = tot[e];
        for (int q = 0; q < kPermWarps; ++q) cnt[q * E + e] += base;
    }
    __syncthreads();
    for (int64_t b = lo; b < hi; b += 32) {
        const int64_t i = b + lane;
        const bool valid = i < hi;
        const int e = valid ? idx[i] : -1;
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
            if (sorted_w) sorted_w[pos] = w ? w[i] : 1.0f;
        }
        if (valid && inv) inv[i] = pos;
        __syncwarp();
    }
}

// out[r] (+)= sum_i pair_w[i] * y[pair_idx[i]]; one CTA row-slice per (row, 1024 columns).
__global__ void combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ row_ptr,
                               const int32_t* __restrict__ pair_idx, const float* __restrict__ pair_w, int64_t T,
                               int k, int H, int accumulate, float* __restrict__ out)
{
    const int64_t r = blockIdx.y;
    const int h = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (h >= H) return;
    const int64_t i0 = row_ptr ? row_ptr[r] : r * k;
    const int64_t i1 = row_ptr ? row_ptr[r + 1] : r * k + k;
    float4 acc = accumulate ? *reinterpret_cast<const float4*>(out + r * H + h) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t i = i0; i < i1; ++i) {
        const int32_t p = pair_idx[i];
        if (p < 0) continue;
        const float wt = pair_w[i];
        const float4 v = *reinterpret_cast<const float4*>(y + (int64_t)p * H + h);
        acc.x = fmaf(wt, v.x, acc.x);
        acc.y = fmaf(wt, v.y, acc.y);
        acc.z = fmaf(wt, v.z, acc.z);
        acc.w = fmaf(wt, v.w, acc.w);
    }
    *reinterpret_cast<float4*>(out + r * H + h) = acc;
}

}  // namespace

extern "C" int mb_router_logits(const float* x, const float* router, int64_t T, int H, int E, float* logits,
                                int32_t* row_exp, void* stream)
{
    MB_REQUIRE(x && router && logits, "mb_router_logits: null pointer");
    MB_REQUIRE(T >= 0 && H > 0 && E > 0, "mb_router_logits: bad shape");
    if (T == 0) return MB_OK;
    MB_REQUIRE(T / kLogitTokens < 65535, "mb_router_logits: T too large");
    dim3 grid((E + kLogitExperts - 1) / kLogitExperts, (unsigned)((T + kLogitTokens - 1) / kLogitTokens));
    router_logits_kernel<<<grid, 256, 0, mb_stream(stream)>>>(x, router, T, H, E, logits, row_exp);
    return mb_check_launch("mb_router_logits");
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
    router_topk_kernel<<<(unsigned)((T + 7) / 8), 256, 0, mb_stream(stream)>>>(logits, T, E, k, normalize, idx, w);
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
    const size_t smem = sizeof(int32_t) * ((size_t)kPermWarps * E + E + 1);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return mb_fail(MB_ECUDA, "mb_permute: %s", cudaGetErrorString(e));
    }
    permute_kernel<<<1, kPermWarps * 32, smem, mb_stream(stream)>>>(idx, w, P, k, E, counts, offsets, sorted_rows,
                                                                    sorted_w, inv, uexperts, uoffsets, n_unique);
    return mb_check_launch("mb_permute");
}

extern "C" int mb_unpermute_combine(const float* y, const int32_t* row_ptr, const int32_t* pair_idx,
                                    const float* pair_w, int64_t T, int k, int H, int accumulate, float* out,
                                    void* stream)
{
    MB_REQUIRE(y && pair_idx && pair_w && out, "mb_unpermute_combine: null pointer");
    MB_REQUIRE(H % 4 == 0 && ((uintptr_t)y & 15) == 0 && ((uintptr_t)out & 15) == 0,
               "mb_unpermute_combine: H must be a multiple of 4 and y/out 16-byte aligned");
    MB_REQUIRE(T < 65536 * 1024LL, "mb_unpermute_combine: T too large");
    if (T == 0) return MB_OK;
    dim3 grid((H / 4 + 255) / 256, (unsigned)T);
    combine_kernel<<<grid, 256, 0, mb_stream(stream)>>>(y, row_ptr, pair_idx, pair_w, T, k, H, accumulate, out);
    return mb_check_launch("mb_unpermute_combine");
}
