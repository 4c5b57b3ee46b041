// Shared helpers for the sm_100a kernels of the routed-expert path.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/moelan_b200.h"

// ---- host-side error reporting -------------------------------------------------

// Records a message for mb_last_error() (thread-local) and returns `code`.
int mb_fail(int code, const char* fmt, ...);

// Returns MB_OK, or records the pending CUDA launch error and returns MB_ECUDA.
int mb_check_launch(const char* what);

// Programmatic dependent launch.  A kernel launched by mb_launch_pdl may start
// while the kernel before it in the stream is still running (its CTAs are
// placed as that kernel's CTAs leave the SMs); it calls mb_pdl_wait() before
// the first read of anything that kernel wrote, which returns once that kernel
// has completed and its writes are visible (at once when there is no such
// kernel).  mb_pdl_trigger() lets the next kernel start launching.
__device__ __forceinline__ void mb_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void mb_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t mb_launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 Args&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
    // a refused launch also records itself as the thread's last CUDA error; it is
    // reported through the return value, so clear it here, or the next
    // mb_check_launch (of an unrelated call) would report it again
    if (e != cudaSuccess) (void)cudaGetLastError();
    return e;
}

#define MB_REQUIRE(cond, ...)                                  \
    do {                                                       \
        if (!(cond)) return mb_fail(MB_EINVAL, __VA_ARGS__);   \
    } while (0)

static inline cudaStream_t mb_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device).
int mb_num_sms();

// ---- device-side status word ---------------------------------------------------
// Kernels never trap: a wait that runs out sets a bit in a caller-visible
// status word and the kernel finishes its loops without waiting any more.
#define MB_STATUS_TIMEOUT 1u
#define MB_STATUS_BADARG 2u

// ---- f16 token rows ---------------------------------------------------------------
// The grouped GEMM reads its tokens as f16 rows, each scaled by 2^row_exp and
// stored in the K order 0 4 1 5 2 6 3 7 within every 8 columns (the order its
// tensor-core operand tiles expect); the token gather and the expert-parallel
// dispatch both write them with these helpers.

__device__ __forceinline__ uint32_t pack_f16(float lo, float hi)
{
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// 2^e for -126 <= e <= 127, exact.
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

__device__ __forceinline__ int clamp120(int e) { return e < -120 ? -120 : (e > 120 ? 120 : e); }

// Eight f32 values as four f16 pairs in the K order 0 4 1 5 2 6 3 7.
__device__ __forceinline__ uint4 pack8_perm(const float4 lo, const float4 hi, float sc)
{
    uint4 o;
    o.x = pack_f16(lo.x * sc, hi.x * sc);
    o.y = pack_f16(lo.y * sc, hi.y * sc);
    o.z = pack_f16(lo.z * sc, hi.z * sc);
    o.w = pack_f16(lo.w * sc, hi.w * sc);
    return o;
}

// Upper bound for one bounded wait, in nanoseconds of %globaltimer.
#define MB_WAIT_LIMIT_NS 2000000000ull

__device__ __forceinline__ uint64_t mb_globaltimer()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t mb_smem_addr(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier + bulk copy (TMA engine, 1-D) ------------------------------------

__device__ __forceinline__ void mb_mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(mb_smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mb_fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mb_mbar_arrive(uint64_t* bar)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(mb_smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mb_mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     mb_smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mb_mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(mb_smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that may park the thread in hardware for up to `ns` nanoseconds
// (woken early when the phase completes), so waiting warps issue nothing.
__device__ __forceinline__ bool mb_mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(mb_smem_addr(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of `bar` to complete, for at most MB_WAIT_LIMIT_NS.
// On time-out sets MB_STATUS_TIMEOUT in *status and *abort_flag and returns false.
// Once *abort_flag is set (by any thread of the CTA) it returns false at once.
__device__ __forceinline__ bool mb_mbar_wait(uint64_t* bar, uint32_t parity, unsigned* status,
                                             volatile int* abort_flag)
{
    if (mb_mbar_try_wait(bar, parity)) return true;
    // back off with __nanosleep so waiting warps leave the issue slots (and the
    // special-register pipe) to the warps doing work; read the timer rarely
    uint64_t t0 = 0;
    uint32_t ns = 20;
    for (uint32_t i = 0;; ++i) {
        __nanosleep(ns);
        if (ns < 320) ns <<= 1;
        if (mb_mbar_try_wait(bar, parity)) return true;
        if ((i & 15u) == 15u) {
            if (*abort_flag) return false;
            const uint64_t now = mb_globaltimer();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > MB_WAIT_LIMIT_NS) {
                atomicOr(status, MB_STATUS_TIMEOUT);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// mb_mbar_wait for tight hand-offs: polls try_wait (which itself parks the
// thread in hardware for a short while) without sleeping in between, reading
// the timer and the abort flag every 1024 polls; same bound and status.
__device__ __forceinline__ bool mb_mbar_wait_spin(uint64_t* bar, uint32_t parity, unsigned* status,
                                                  volatile int* abort_flag)
{
    uint64_t t0 = 0;
    for (uint32_t i = 1;; ++i) {
        if (mb_mbar_try_wait(bar, parity)) return true;
        if ((i & 1023u) == 0) {
            if (*abort_flag) return false;
            const uint64_t now = mb_globaltimer();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > MB_WAIT_LIMIT_NS) {
                atomicOr(status, MB_STATUS_TIMEOUT);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// Global -> shared bulk copy on the TMA engine, completing `bytes` on `bar`.
// dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void mb_bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            mb_smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(mb_smem_addr(bar))
        : "memory");
}

// L2 policies for the copies above: data read once (weights streamed through
// the kernel) goes first when L2 needs room; data read again (token or
// activation rows reused by many tiles) is kept.
__device__ __forceinline__ uint64_t mb_policy_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t mb_policy_evict_last()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// mb_bulk_g2s with an L2 policy from mb_policy_*.
__device__ __forceinline__ void mb_bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                 uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(mb_smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(mb_smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void mb_named_barrier(int id, int nthreads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- small numeric helpers -----------------------------------------------------

// IEEE half from its bits, decoded the way moelan/kernels.py:244-255 does it
// (exponent 31 -> +-inf whatever the payload), exact.
__device__ __forceinline__ float mb_f16_ref(uint32_t h)
{
    const uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF;
    float v;
    if (e == 0)
        v = __fmul_rn((float)m, 5.9604644775390625e-08f);
    else if (e == 31)
        v = __int_as_float(0x7f800000);
    else
        v = __uint_as_float(((e + 112u) << 23) | (m << 13));
    return (h & 0x8000) ? -v : v;
}

// mma.sync m16n8k16, f16 x f16 -> f32, accumulating in place: D += A*B.
// (No volatile: independent MMAs may be interleaved by the compiler.)
__device__ __forceinline__ void mb_mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A*B (zero accumulator).
__device__ __forceinline__ void mb_mma_f16_zero(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                uint32_t b0, uint32_t b1)
{
    const float z = 0.0f;
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

__device__ __forceinline__ uint32_t mb_lop_and_or(uint32_t a, uint32_t mask, uint32_t orv)
{
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));  // (a & b) | c
    return r;
}

__device__ __forceinline__ uint32_t mb_hsub2(uint32_t a, uint32_t b)
{
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t mb_hfma2(uint32_t a, uint32_t b, uint32_t c)
{
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ uint32_t mb_hmul2(uint32_t a, uint32_t b)
{
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t mb_prmt(uint32_t a, uint32_t b, uint32_t sel)
{
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ __forceinline__ uint32_t mb_pack_h2(__half lo, __half hi)
{
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// The power-of-two exponent e that maps a row whose largest magnitude is
// `amax` into [2^13, 2^14): the row is split into f16 hi + lo pieces of
// x * 2^e for the tensor-core mat-vec.
__device__ __forceinline__ int mb_row_exponent(float amax)
{
    if (!(amax > 0.0f) || !(amax < 3.0e38f)) return 0;
    int ex;
    frexpf(amax, &ex);
    int e = 14 - ex;
    return e < -120 ? -120 : (e > 120 ? 120 : e);
}
