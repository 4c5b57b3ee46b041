// The reference's other routers, one warp per token.
//
// * route_grouped (moelan/model.py:170-201): DeepSeek V2 / V3 routing.  Scores
//   are the softmax or the sigmoid of the logits; the choice is the score plus
//   an optional per-expert bias (V3's e_score_correction_bias).  With
//   group-limited methods only the topk_group best groups of experts stay
//   (V2 group_limited_greedy: a group's best choice; V3 noaux_tc: the sum of
//   its two best), the others' choices become 0.  The k best choices are
//   picked and weighted by their scores, normalised (V3 also scaled) or
//   scaled.
// * route_sparsemixer (moelan/model.py:204-223): PhiMoE's top-2.  Each pick
//   is the best remaining expert, weighted by its softmax over the experts
//   whose logit lies within a relative 2*eps of it; the second pick masks the
//   first.
//
// Orders follow the reference's stable argsorts: equal values go to the lower
// index.  Each lane holds experts lane, lane + 32, ... (E <= 32 * PER); a
// warp's choices also go to shared memory for the per-group scan.
#include <cfloat>

#include "mb_common.cuh"

namespace {

constexpr int kWarps = 8;          // tokens per CTA
constexpr int kMaxExperts = 1024;

// The index of the largest v over the warp's experts not yet taken (ties: lower
// index), and its value; every lane gets both.
template <int PER>
__device__ __forceinline__ int warp_argmax(const float (&v)[PER], uint32_t taken, int E, int lane, float* best)
{
    float bv = -INFINITY;
    int bi = INT32_MAX;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = i * 32 + lane;
        if (e < E && !((taken >> i) & 1u) && (v[i] > bv || (v[i] == bv && e < bi))) {
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
    *best = bv;
    return bi;
}

// numpy's sum of n <= 128 contiguous f32 values (pairwise: eight running sums
// when n >= 8, combined as a tree, then the tail; a plain running sum below 8).
__device__ float np_sum(const float* a, int n)
{
    if (n < 8) {
        float r = 0.0f;
        for (int i = 0; i < n; ++i) r += a[i];
        return r;
    }
    float r[8];
    for (int j = 0; j < 8; ++j) r[j] = a[j];
    int i = 8;
    for (; i < n - n % 8; i += 8)
        for (int j = 0; j < 8; ++j) r[j] += a[i + j];
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res += a[i];
    return res;
}

template <int PER>
__global__ void __launch_bounds__(kWarps * 32) router_grouped_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias, int64_t T, int E, int k, int sigmoid,
    int method, int n_group, int topk_group, int normalize, float scaling, int32_t* __restrict__ idx,
    float* __restrict__ w)
{
    mb_pdl_wait();
    mb_pdl_trigger();
    __shared__ float s_choice[kWarps][32 * PER];
    __shared__ float s_w[kWarps][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * kWarps + warp;
    if (t >= T) return;
    float sc[PER], ch[PER];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = i * 32 + lane;
        sc[i] = e < E ? logits[t * E + e] : -INFINITY;
        m = fmaxf(m, sc[i]);
    }
    if (sigmoid) {
#pragma unroll
        for (int i = 0; i < PER; ++i) sc[i] = __fdiv_rn(1.0f, 1.0f + expf(-sc[i]));
    } else {   // softmax: subtract the row maximum, exponentiate, divide by the sum
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            sc[i] = (i * 32 + lane) < E ? expf(sc[i] - m) : 0.0f;
            sum += sc[i];
        }
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
        for (int i = 0; i < PER; ++i) sc[i] = __fdiv_rn(sc[i], sum);
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = i * 32 + lane;
        ch[i] = e < E ? (bias ? sc[i] + bias[e] : sc[i]) : -INFINITY;
    }
    if (method >= 1 && n_group > 1) {
        // group scores from the choices in shared memory: lane g scans group g
#pragma unroll
        for (int i = 0; i < PER; ++i)
            if (i * 32 + lane < E) s_choice[warp][i * 32 + lane] = ch[i];
        __syncwarp();
        const int gsz = E / n_group;
        float gscore = -INFINITY;
        for (int g = lane; g < n_group; g += 32) {   // n_group <= 32
            float b1 = -INFINITY, b2 = -INFINITY;
            for (int j = 0; j < gsz; ++j) {
                const float c = s_choice[warp][g * gsz + j];
                if (c > b1) {
                    b2 = b1;
                    b1 = c;
                } else if (c > b2) {
                    b2 = c;
                }
            }
            gscore = method == 2 ? b1 + b2 : b1;
        }
        // the topk_group best groups (ties: lower group first); the others' choices become 0
        uint32_t kept = 0;
        float gv[1] = {gscore};
        uint32_t gtaken = 0;
        for (int j = 0; j < topk_group; ++j) {
            float bv;
            const int g = warp_argmax<1>(gv, gtaken, n_group, lane, &bv);
            if (g == lane) gtaken = 1u;
            kept |= 1u << g;
        }
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int e = i * 32 + lane;
            if (e < E && !((kept >> (e / gsz)) & 1u)) ch[i] = 0.0f;
        }
    }
    // the k best choices, weighted by their scores
    uint32_t taken = 0;
    for (int j = 0; j < k; ++j) {
        float bv;
        const int e = warp_argmax<PER>(ch, taken, E, lane, &bv);
        const int owner = e & 31, slot = e >> 5;
        float sv = 0.0f;
#pragma unroll
        for (int i = 0; i < PER; ++i)
            if (i == slot) sv = sc[i];
        sv = __shfl_sync(0xffffffffu, sv, owner);
        if (lane == owner) taken |= 1u << slot;
        if (lane == 0) {
            idx[t * k + j] = e;
            s_w[warp][j] = sv;
        }
    }
    __syncwarp();
    if (lane == 0) {
        float* wr = s_w[warp];
        if (k > 1 && normalize) {
            const float den = np_sum(wr, k) + 1e-20f;
            for (int j = 0; j < k; ++j) {
                float v = __fdiv_rn(wr[j], den);
                if (method == 2) v *= scaling;
                w[t * k + j] = v;
            }
        } else {
            for (int j = 0; j < k; ++j) w[t * k + j] = wr[j] * scaling;
        }
    }
}

template <int PER>
__global__ void __launch_bounds__(kWarps * 32) router_sparsemixer_kernel(const float* __restrict__ logits, int64_t T,
                                                                        int E, float thr, int32_t* __restrict__ idx,
                                                                        float* __restrict__ w)
{
    mb_pdl_wait();
    mb_pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * kWarps + warp;
    if (t >= T) return;
    float s[PER], left[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = i * 32 + lane;
        s[i] = e < E ? logits[t * E + e] : -INFINITY;
        left[i] = s[i];
    }
    uint32_t none = 0;
    for (int j = 0; j < 2; ++j) {
        float best;
        const int top = warp_argmax<PER>(left, none, E, lane, &best);
        // softmax over the experts within the band, at the pick: exp(0) / sum(exp(v - best))
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            if (i * 32 + lane >= E) continue;
            const float rel = __fdiv_rn(best - s[i], fmaxf(fabsf(s[i]), best));
            const bool far = rel > thr;   // a NaN (0 / 0) is not far
            if (!far && left[i] != -INFINITY) sum += expf(left[i] - best);
        }
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            idx[t * 2 + j] = top;
            w[t * 2 + j] = __fdiv_rn(1.0f, sum);
        }
        if (lane == (top & 31)) {
#pragma unroll
            for (int i = 0; i < PER; ++i)
                if (i == (top >> 5)) left[i] = -INFINITY;
        }
    }
}

}  // namespace

extern "C" int mb_router_grouped(const float* logits, const float* bias, int64_t T, int E, int k, int sigmoid,
                                 int method, int n_group, int topk_group, int normalize, float scaling, int32_t* idx,
                                 float* w, void* stream)
{
    MB_REQUIRE(logits && idx && w, "mb_router_grouped: null pointer");
    MB_REQUIRE(T >= 0 && E > 0 && E <= kMaxExperts && k > 0 && k <= E && k <= 32,
               "mb_router_grouped: T=%lld E=%d k=%d (E <= %d, k <= 32)", (long long)T, E, k, kMaxExperts);
    MB_REQUIRE(method >= 0 && method <= 2, "mb_router_grouped: method %d", method);
    if (method >= 1 && n_group > 1)
        MB_REQUIRE(n_group <= 32 && E % n_group == 0 && topk_group >= 1 && topk_group <= n_group,
                   "mb_router_grouped: %d groups of %d experts, keep %d", n_group, E, topk_group);
    if (T == 0) return MB_OK;
    const int per = (E + 31) / 32;
    const dim3 grid((unsigned)((T + kWarps - 1) / kWarps)), block(kWarps * 32);
    cudaStream_t st = mb_stream(stream);
    cudaError_t e;
#define MB_GROUPED(P)                                                                                               \
    e = mb_launch_pdl(router_grouped_kernel<P>, grid, block, 0, st, logits, bias, T, E, k, sigmoid, method, n_group, \
                      topk_group, normalize, scaling, idx, w)
    if (per <= 1) MB_GROUPED(1);
    else if (per <= 2) MB_GROUPED(2);
    else if (per <= 4) MB_GROUPED(4);
    else if (per <= 8) MB_GROUPED(8);
    else if (per <= 16) MB_GROUPED(16);
    else MB_GROUPED(32);
#undef MB_GROUPED
    if (e != cudaSuccess) return mb_fail(MB_ECUDA, "mb_router_grouped launch: %s", cudaGetErrorString(e));
    return MB_OK;
}

extern "C" int mb_router_sparsemixer(const float* logits, int64_t T, int E, double eps, int32_t* idx, float* w,
                                     void* stream)
{
    MB_REQUIRE(logits && idx && w, "mb_router_sparsemixer: null pointer");
    MB_REQUIRE(T >= 0 && E >= 2 && E <= kMaxExperts, "mb_router_sparsemixer: T=%lld E=%d", (long long)T, E);
    if (T == 0) return MB_OK;
    const float thr = (float)(2.0 * eps);   // the reference compares its f32 ratios with 2 * eps (made f32)
    const int per = (E + 31) / 32;
    const dim3 grid((unsigned)((T + kWarps - 1) / kWarps)), block(kWarps * 32);
    cudaStream_t st = mb_stream(stream);
    cudaError_t e;
#define MB_SPARSE(P) e = mb_launch_pdl(router_sparsemixer_kernel<P>, grid, block, 0, st, logits, T, E, thr, idx, w)
    if (per <= 1) MB_SPARSE(1);
    else if (per <= 2) MB_SPARSE(2);
    else if (per <= 4) MB_SPARSE(4);
    else if (per <= 8) MB_SPARSE(8);
    else if (per <= 16) MB_SPARSE(16);
    else MB_SPARSE(32);
#undef MB_SPARSE
    if (e != cudaSuccess) return mb_fail(MB_ECUDA, "mb_router_sparsemixer launch: %s", cudaGetErrorString(e));
    return MB_OK;
}
