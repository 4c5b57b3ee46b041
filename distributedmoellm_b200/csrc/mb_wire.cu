// Activation rows in the reference's wire formats, on the device.
//
// moelan sends the rows routed to a worker and the rows it sends back in one
// of three formats (moelan/protocol.py:96-123): f32, f16 (numpy's
// round-to-nearest-even conversion) or int8 with one f32 scale per group of 64
// values (the whole row when its width is not a multiple of 64): scale =
// max|group| / 127 (1 for an all-zero group), q = clip(rint(x / scale), ±127).
// A GPU worker can copy the encoded bytes to the device as they arrive and
// widen them there, and encode its results before the copy back, so the
// host↔device copies carry the compressed sizes.
//
// One warp per (row, group): each lane takes two values of a 64-value group
// (coalesced 8-byte loads), the group maximum is a warp reduction, and every
// result is rounded exactly once as numpy rounds it (__fdiv_rn, rintf, which
// rounds half to even, and __fmul_rn on decode).
#include "mb_common.cuh"

namespace {

constexpr int kWireGroup = 64;

// int8 encode: warp (row r, group g) of width gw (64, or the row width d when d % 64 != 0)
__global__ void encode_int8_kernel(const float* __restrict__ a, int64_t n, int d, int gw, int8_t* __restrict__ q,
                                   float* __restrict__ scales)
{
    const int lane = threadIdx.x & 31;
    const int ng = d / gw;
    const int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (w >= n * ng) return;
    const int64_t r = w / ng;
    const int g = (int)(w - r * ng);
    const float* src = a + r * d + (int64_t)g * gw;
    float m = 0.0f;
    for (int j = lane; j < gw; j += 32) m = fmaxf(m, fabsf(src[j]));
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = __fdiv_rn(m, 127.0f);
    if (s == 0.0f) s = 1.0f;
    int8_t* dst = q + r * d + (int64_t)g * gw;
    for (int j = lane; j < gw; j += 32) {
        float v = rintf(__fdiv_rn(src[j], s));
        v = fminf(fmaxf(v, -127.0f), 127.0f);
        dst[j] = (int8_t)(int)v;
    }
    if (lane == 0) scales[r * ng + g] = s;
}

__global__ void encode_f16_kernel(const float* __restrict__ a, int64_t count, __half* __restrict__ h)
{
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
        h[i] = __float2half_rn(a[i]);
}

__global__ void decode_int8_kernel(const int8_t* __restrict__ q, const float* __restrict__ scales, int64_t n, int d,
                                   int gw, float* __restrict__ out)
{
    const int ng = d / gw;
    const int64_t count = n * d;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / d;
        const int c = (int)(i - r * d);
        out[i] = __fmul_rn((float)q[i], scales[r * ng + c / gw]);
    }
}

__global__ void decode_f16_kernel(const __half* __restrict__ h, int64_t count, float* __restrict__ out)
{
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __half2float(h[i]);
}

int wire_grid(int64_t count, int block)
{
    int64_t g = (count + block - 1) / block;
    const int64_t cap = (int64_t)mb_num_sms() * 8;
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace

extern "C" int mb_wire_group(int d) { return d % kWireGroup == 0 ? kWireGroup : d; }

extern "C" int mb_encode_rows(const float* a, int64_t n, int d, int wire, void* q, float* scales, void* stream)
{
    MB_REQUIRE(a && q && n >= 0 && d > 0, "mb_encode_rows: bad arguments");
    MB_REQUIRE(wire == MB_WIRE_F16 || wire == MB_WIRE_INT8, "mb_encode_rows: wire format %d", wire);
    MB_REQUIRE(wire != MB_WIRE_INT8 || scales, "mb_encode_rows: int8 needs the scales buffer");
    if (n == 0) return MB_OK;
    cudaStream_t st = mb_stream(stream);
    if (wire == MB_WIRE_F16) {
        encode_f16_kernel<<<wire_grid(n * d, 256), 256, 0, st>>>(a, n * d, reinterpret_cast<__half*>(q));
    } else {
        const int gw = mb_wire_group(d);
        const int64_t warps = n * (d / gw);
        encode_int8_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(a, n, d, gw, reinterpret_cast<int8_t*>(q),
                                                                       scales);
    }
    return mb_check_launch("mb_encode_rows");
}

extern "C" int mb_decode_rows(const void* q, const float* scales, int64_t n, int d, int wire, float* out,
                              void* stream)
{
    MB_REQUIRE(q && out && n >= 0 && d > 0, "mb_decode_rows: bad arguments");
    MB_REQUIRE(wire == MB_WIRE_F16 || wire == MB_WIRE_INT8, "mb_decode_rows: wire format %d", wire);
    MB_REQUIRE(wire != MB_WIRE_INT8 || scales, "mb_decode_rows: int8 needs the scales");
    if (n == 0) return MB_OK;
    cudaStream_t st = mb_stream(stream);
    if (wire == MB_WIRE_F16)
        decode_f16_kernel<<<wire_grid(n * d, 256), 256, 0, st>>>(reinterpret_cast<const __half*>(q), n * d, out);
    else
        decode_int8_kernel<<<wire_grid(n * d, 256), 256, 0, st>>>(reinterpret_cast<const int8_t*>(q), scales, n, d,
                                                                  mb_wire_group(d), out);
    return mb_check_launch("mb_decode_rows");
}
