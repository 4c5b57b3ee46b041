// Expert parallelism over the GPUs of one node through peer memory.
//
// The reference's multi-machine design (moelan/coordinator.py:475-535) sends
// each worker one request per layer carrying only the rows routed to that
// worker's experts, and adds the partial sums it gets back.  Here the workers
// are the GPUs of one node, one process each, and the rows move by stores
// into the other GPUs' memory over NVLink, from inside the kernels that make
// and consume them:
//
//  * every rank owns one receive arena (plain cudaMalloc memory) that the
//    other ranks' processes map through CUDA IPC handles (mb_peer_*);
//  * mb_ep_dispatch: every rank routes its own tokens; once the per-expert
//    pick counts of all ranks are known on the device (an all-gather of E
//    integers per rank), each rank's rows have a fixed place in their
//    expert's rank's receive rows (grouped by local expert, within an expert
//    by source rank, within a source in the source's pick order).  The
//    kernel computes that place and stores the token row there, already as
//    the grouped GEMM's f16 operand, with the row's exponent and a return
//    address (source rank, source pick);
//  * the grouped GEMM (mb_moe_prefill_rows) runs the rank's experts over its
//    receive rows and its epilogue stores each output row straight into the
//    source rank's result rows at the return address;
//  * each rank combines its own picks' results locally, in each token's
//    fixed pick order (the same sum as on one GPU).
// No host round trip and no size known only on the device: every buffer is
// sized for the worst case (all picks of all ranks on one rank), so the
// whole step can be captured in a CUDA graph.  The peer stores are plain
// global stores; no TMA copy touches another GPU's memory.
#include <string.h>

#include <algorithm>

#include "mb_common.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) == MB_PEER_HANDLE_BYTES, "IPC handle size");

extern "C" int mb_peer_alloc(int64_t bytes, void** ptr, void* handle)
{
    MB_REQUIRE(bytes > 0 && ptr && handle, "mb_peer_alloc: bad arguments");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, (size_t)bytes);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return mb_fail(MB_ECUDA, "mb_peer_alloc: cudaMalloc(%lld): %s", (long long)bytes, cudaGetErrorString(e));
    }
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        cudaFree(p);
        return mb_fail(MB_ECUDA, "mb_peer_alloc: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    }
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return MB_OK;
}

extern "C" int mb_peer_open(const void* handle, void** ptr)
{
    MB_REQUIRE(handle && ptr, "mb_peer_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return mb_fail(MB_ECUDA, "mb_peer_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    }
    *ptr = p;
    return MB_OK;
}

extern "C" int mb_peer_close(void* ptr)
{
    MB_REQUIRE(ptr, "mb_peer_close: null pointer");
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return mb_fail(MB_ECUDA, "mb_peer_close: %s", cudaGetErrorString(e));
    }
    return MB_OK;
}

extern "C" int mb_peer_free(void* ptr)
{
    MB_REQUIRE(ptr, "mb_peer_free: null pointer");
    const cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return mb_fail(MB_ECUDA, "mb_peer_free: %s", cudaGetErrorString(e));
    }
    return MB_OK;
}

namespace {

constexpr int kDispatchThreads = 256;

// One CTA: the receive plan from the all-gathered counts (redundantly in every CTA, E x G integers), then one
// warp per pick of this rank's tokens.
__global__ void __launch_bounds__(kDispatchThreads)
    ep_dispatch_kernel(const float* __restrict__ x, const int32_t* __restrict__ row_exp, int64_t T, int H,
                       const int32_t* __restrict__ idx, const int32_t* __restrict__ inv, int k,
                       const int32_t* __restrict__ offsets, const int32_t* __restrict__ counts_all, int E, int G,
                       int rank, __half* const* __restrict__ recv_rows, int32_t* const* __restrict__ recv_exp,
                       int32_t* const* __restrict__ recv_ret, int64_t cap, int32_t* __restrict__ local_counts,
                       int32_t* __restrict__ local_offsets, unsigned* __restrict__ status)
{
    extern __shared__ int32_t plan_s[];
    int32_t* tot = plan_s;        // [E] picks of every rank for expert e
    int32_t* roff = plan_s + E;   // [E] receive row of this rank's first pick for expert e, at e's rank
    const int El = E / G;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int t = 0, before = 0;
        for (int s = 0; s < G; ++s) {
            const int c = counts_all[(int64_t)s * E + e];
            t += c;
            if (s < rank) before += c;
        }
        tot[e] = t;
        roff[e] = before;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int base = 0;
        for (int f = (e / El) * El; f < e; ++f) base += tot[f];
        roff[e] += base;
    }
    if (blockIdx.x == 0) {
        for (int j = threadIdx.x; j <= El; j += blockDim.x) {
            int base = 0;
            for (int f = 0; f < j; ++f) base += tot[rank * El + f];
            if (j < El) local_counts[j] = tot[rank * El + j];
            local_offsets[j] = base;
        }
    }
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int wpb = blockDim.x >> 5;
    const int64_t P = T * k;
    for (int64_t p = (int64_t)blockIdx.x * wpb + (threadIdx.x >> 5); p < P; p += (int64_t)gridDim.x * wpb) {
        const int e = idx[p];
        if (e < 0 || e >= E) {
            if (lane == 0) atomicOr(status, MB_STATUS_BADARG);
            continue;
        }
        const int64_t row = (int64_t)roff[e] + (inv[p] - offsets[e]);
        if (row < 0 || row >= cap) {
            if (lane == 0) atomicOr(status, MB_STATUS_BADARG);
            continue;
        }
        const int d = e / El;
        const int64_t t = p / k;
        const int rexp = row_exp[t];
        const float sc = pow2i(clamp120(rexp));
        const float* src = x + t * H;
        __half* dst = recv_rows[d] + row * H;
        for (int c = lane * 8; c < H; c += 256) {
            const float4 lo = *reinterpret_cast<const float4*>(src + c);
            const float4 hi = *reinterpret_cast<const float4*>(src + c + 4);
            *reinterpret_cast<uint4*>(dst + c) = pack8_perm(lo, hi, sc);
        }
        if (lane == 0) {
            recv_exp[d][row] = rexp;
            recv_ret[d][row] = (int32_t)(((uint32_t)rank << 24) | (uint32_t)p);
        }
    }
    __threadfence_system();   // the stores to other GPUs are seen before what follows this launch
}

}  // namespace

extern "C" int mb_ep_dispatch(const float* x, const int32_t* row_exp, int64_t T, int H, const int32_t* idx,
                              const int32_t* inv, int k, const int32_t* offsets, const int32_t* counts_all, int E,
                              int G, int rank, void* const* recv_rows, int32_t* const* recv_exp,
                              int32_t* const* recv_ret, int64_t cap, int32_t* local_counts, int32_t* local_offsets,
                              unsigned* status, void* stream)
{
    MB_REQUIRE(x && row_exp && idx && inv && offsets && counts_all && recv_rows && recv_exp && recv_ret &&
                   local_counts && local_offsets && status,
               "mb_ep_dispatch: null pointer");
    MB_REQUIRE(G >= 1 && G <= 128 && rank >= 0 && rank < G, "mb_ep_dispatch: rank %d of %d (at most 128)", rank, G);
    MB_REQUIRE(E > 0 && E % G == 0 && E <= 4096, "mb_ep_dispatch: E=%d experts over %d ranks", E, G);
    MB_REQUIRE(T >= 0 && k > 0 && T * k < (1 << 24), "mb_ep_dispatch: T*k=%lld picks (below 2^24)",
               (long long)(T * k));
    MB_REQUIRE(H > 0 && H % 128 == 0, "mb_ep_dispatch: H=%d (a multiple of 128)", H);
    MB_REQUIRE(cap >= 0 && cap < (1ll << 31), "mb_ep_dispatch: cap=%lld", (long long)cap);
    MB_REQUIRE(((uintptr_t)x & 15) == 0, "mb_ep_dispatch: x must be 16-byte aligned");
    cudaStream_t st = mb_stream(stream);
    const int64_t P = T * k;
    const int wpb = kDispatchThreads / 32;
    const int64_t want = (P + wpb - 1) / wpb;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)mb_num_sms() * 4));
    ep_dispatch_kernel<<<grid, kDispatchThreads, 2 * E * sizeof(int32_t), st>>>(
        x, row_exp, T, H, idx, inv, k, offsets, counts_all, E, G, rank, reinterpret_cast<__half* const*>(recv_rows),
        recv_exp, recv_ret, cap, local_counts, local_offsets, status);
    return mb_check_launch("mb_ep_dispatch");
}
