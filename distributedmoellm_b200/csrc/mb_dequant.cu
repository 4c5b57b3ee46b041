// Bit-exact dequantisation of packed expert weights to f32.
//
// Each value is produced with the reference's single rounding (products and
// sums written with __fmul_rn/__fadd_rn/__fsub_rn so nvcc cannot contract
// them into FMAs):
//   int4  moelan/kernels.py:215-228   f32(nibble - 8) * s
//   int8  moelan/kernels.py:230-237   f32(q) * s
//   GGUF  moelan/kernels.py:262-476   llama.cpp block formats
#include <algorithm>

#include "mb_common.cuh"

namespace {

template <bool F16>
__device__ __forceinline__ float load_scale(const void* s, int64_t i)
{
    if (F16) return __half2float(reinterpret_cast<const __half*>(s)[i]);
    return reinterpret_cast<const float*>(s)[i];
}

template <bool F16>
__global__ void q4_dequant_kernel(const uint8_t* __restrict__ raw, const void* __restrict__ s, int64_t rows,
                                  int64_t cols, int gs, uint8_t xr, float* __restrict__ out)
{
    const int64_t C = cols / 2, ng = cols / gs;
    const int64_t n = rows * C;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = i / C, b = i - o * C;
        const float sc = load_scale<F16>(s, o * ng + (2 * b) / gs);
        const int v = raw[i] ^ xr;
        float2 r;
        r.x = __fmul_rn((float)((v & 15) - 8), sc);
        r.y = __fmul_rn((float)((v >> 4) - 8), sc);
        *reinterpret_cast<float2*>(out + o * cols + 2 * b) = r;
    }
}

template <bool F16>
__global__ void q8_dequant_kernel(const int8_t* __restrict__ q, const void* __restrict__ s, int64_t rows,
                                  int64_t cols, int gs, float* __restrict__ out)
{
    const int64_t ng = cols / gs, n = rows * cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = i / cols, c = i - o * cols;
        out[i] = __fmul_rn((float)q[i], load_scale<F16>(s, o * ng + c / gs));
    }
}

// ---- GGUF: one thread decodes one 32-value segment of one row ------------------

__device__ __forceinline__ float f16b(const uint8_t* p) { return mb_f16_ref((uint32_t)p[0] | ((uint32_t)p[1] << 8)); }
__device__ __forceinline__ int i8(uint8_t b) { return (int)(int8_t)b; }
__device__ __forceinline__ uint32_t u32le(const uint8_t* p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// (scale, min) pair j of a K-quant super-block (moelan/kernels.py:310-316).
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* s, int& sc, int& m)
{
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

__device__ __forceinline__ void gguf_segment(const uint8_t* row, int qtype, int64_t seg, float* v)
{
    switch (qtype) {
    case 8: {  // Q8_0, kernels.py:262-268
        const uint8_t* p = row + seg * 34;
        const float d = f16b(p);
        for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(d, (float)i8(p[2 + j]));
        break;
    }
    case 2: {  // Q4_0, kernels.py:270-278
        const uint8_t* p = row + seg * 18;
        const float d = f16b(p);
        for (int j = 0; j < 16; ++j) {
            const int q = p[2 + j];
            v[j] = __fmul_rn(d, (float)((q & 15) - 8));
            v[j + 16] = __fmul_rn(d, (float)((q >> 4) - 8));
        }
        break;
    }
    case 3: {  // Q4_1, kernels.py:280-289
        const uint8_t* p = row + seg * 20;
        const float d = f16b(p), mn = f16b(p + 2);
        for (int j = 0; j < 16; ++j) {
            const int q = p[4 + j];
            v[j] = __fadd_rn(__fmul_rn(d, (float)(q & 15)), mn);
            v[j + 16] = __fadd_rn(__fmul_rn(d, (float)(q >> 4)), mn);
        }
        break;
    }
    case 6:
    case 7: {  // Q5_0 / Q5_1, kernels.py:291-308
        const bool wm = qtype == 7;
        const uint8_t* p = row + seg * (wm ? 24 : 22);
        const float d = f16b(p);
        const float mn = wm ? f16b(p + 2) : 0.0f;
        const uint8_t* h = p + (wm ? 4 : 2);
        const int64_t qh = (int64_t)u32le(h);
        const uint8_t* qs = h + 4;
        const int off = wm ? 0 : 16;
        for (int j = 0; j < 16; ++j) {
            const int64_t q = qs[j];
            const int64_t x0 = ((q & 15) | (((qh >> j) << 4) & 0x10)) - off;
            const int64_t x1 = ((q >> 4) | ((qh >> (j + 12)) & 0x10)) - off;
            v[j] = __fadd_rn(__fmul_rn(d, (float)x0), mn);
            v[j + 16] = __fadd_rn(__fmul_rn(d, (float)x1), mn);
        }
        break;
    }
    case 12:
    case 13: {  // Q4_K / Q5_K, kernels.py:318-361
        const bool q5 = qtype == 13;
        const int64_t b = seg >> 3;
        const int s8 = (int)(seg & 7), k = s8 >> 1, hi = s8 & 1;
        const uint8_t* p = row + b * (q5 ? 176 : 144);
        const float d = f16b(p), dmin = f16b(p + 2);
        int sc, m;
        scale_min_k4(s8, p + 4, sc, m);
        const float ds = __fmul_rn(d, (float)sc), ms = __fmul_rn(dmin, (float)m);
        const uint8_t* q = p + (q5 ? 48 : 16) + 32 * k;
        const int ubit = 1 << (2 * k + hi);
        for (int l = 0; l < 32; ++l) {
            int u = hi ? (q[l] >> 4) : (q[l] & 15);
            if (q5 && (p[16 + l] & ubit)) u += 16;
            v[l] = __fsub_rn(__fmul_rn(ds, (float)u), ms);
        }
        break;
    }
    case 14: {  // Q6_K, kernels.py:363-387
        const int64_t b = seg >> 3;
        const int s8 = (int)(seg & 7), n = s8 >> 2, m4 = s8 & 3;
        const uint8_t* p = row + b * 210;
        const float d = f16b(p + 208);
        const uint8_t *ql = p + 64 * n, *qh = p + 128 + 32 * n, *sc = p + 192 + 8 * n;
        for (int l = 0; l < 32; ++l) {
            const int s = l / 16;
            const int a = ql[l], c = ql[l + 32], h = qh[l];
            int q;
            switch (m4) {
            case 0: q = ((a & 15) | (((h >> 0) & 3) << 4)) - 32; break;
            case 1: q = ((c & 15) | (((h >> 2) & 3) << 4)) - 32; break;
            case 2: q = ((a >> 4) | (((h >> 4) & 3) << 4)) - 32; break;
            default: q = ((c >> 4) | (((h >> 6) & 3) << 4)) - 32; break;
            }
            v[l] = __fmul_rn(d, (float)(i8(sc[s + 2 * m4]) * q));
        }
        break;
    }
    case 10: {  // Q2_K, kernels.py:389-414
        const int64_t b = seg >> 3;
        const int s8 = (int)(seg & 7), n = s8 >> 2, j = s8 & 3;
        const uint8_t* p = row + b * 84;
        const float d = f16b(p + 80), dmin = f16b(p + 82);
        const uint8_t* q = p + 16 + 32 * n;
        const int shift = 2 * j;
        for (int half = 0; half < 2; ++half) {
            const int s = p[8 * n + 2 * j + half];
            const float dl = __fmul_rn(d, (float)(s & 15)), ml = __fmul_rn(dmin, (float)(s >> 4));
            for (int l = 0; l < 16; ++l)
                v[16 * half + l] = __fsub_rn(__fmul_rn(dl, (float)((q[l + 16 * half] >> shift) & 3)), ml);
        }
        break;
    }
    case 11: {  // Q3_K, kernels.py:416-453
        const int64_t b = seg >> 3;
        const int s8 = (int)(seg & 7), n = s8 >> 2, j = s8 & 3;
        const uint8_t* p = row + b * 110;
        const float d = f16b(p + 108);
        const int64_t km1 = 0x03030303, km2 = 0x0F0F0F0F;
        const int64_t a0 = u32le(p + 96), a1 = u32le(p + 100), t = u32le(p + 104);
        const uint8_t *hm = p, *q = p + 32 + 32 * n;
        const int shift = 2 * j, mbit = 1 << (4 * n + j);
        for (int half = 0; half < 2; ++half) {
            const int i = 8 * n + 2 * j + half, w = i >> 2, kk = i & 3;
            int64_t word;
            switch (w) {
            case 0: word = (a0 & km2) | (((t >> 0) & km1) << 4); break;
            case 1: word = (a1 & km2) | (((t >> 2) & km1) << 4); break;
            case 2: word = ((a0 >> 4) & km2) | (((t >> 4) & km1) << 4); break;
            default: word = ((a1 >> 4) & km2) | (((t >> 6) & km1) << 4); break;
            }
            const int scale = (int)((word >> (8 * kk)) & 0xFF) - 32;
            const float dl = __fmul_rn(d, (float)scale);
            for (int l = 0; l < 16; ++l) {
                const int x = ((q[l + 16 * half] >> shift) & 3) - ((hm[l + 16 * half] & mbit) ? 0 : 4);
                v[16 * half + l] = __fmul_rn(dl, (float)x);
            }
        }
        break;
    }
    default:
        break;
    }
}

__global__ void gguf_dequant_kernel(const uint8_t* __restrict__ raw, int qtype, int64_t rows, int64_t row_bytes,
                                    int64_t cols, float* __restrict__ out)
{
    const int64_t nseg = cols / 32, n = rows * nseg;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = i / nseg, seg = i - o * nseg;
        float v[32];
        gguf_segment(raw + o * row_bytes, qtype, seg, v);
        float4* dst = reinterpret_cast<float4*>(out + o * cols + seg * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
}

// x @ W.T straight from GGUF blocks for a few input rows (decode): one warp per
// weight row, each lane decoding 32-value segments with the bit-exact block
// decoders above and dotting them with up to NR input rows in f32.  QT: the
// ggml type id (a compile-time constant, so each decoder is specialised).
template <int QT, int NR>
__global__ void __launch_bounds__(256) gguf_mv_kernel(const uint8_t* __restrict__ raw, int64_t rows,
                                                      int64_t row_bytes, int64_t cols, const float* __restrict__ x,
                                                      int n, float* __restrict__ y)
{
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t nseg = cols / 32;
    for (int64_t o = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); o < rows; o += warps) {
        const uint8_t* row = raw + o * row_bytes;
        float acc[NR];
#pragma unroll
        for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
        for (int64_t seg = lane; seg < nseg; seg += 32) {
            float v[32];
            gguf_segment(row, QT, seg, v);
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                if (r < n) {
                    const float4* xp = reinterpret_cast<const float4*>(x + (int64_t)r * cols + seg * 32);
                    float s = 0.0f;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 u = __ldg(xp + j);
                        s = fmaf(v[4 * j], u.x, s);
                        s = fmaf(v[4 * j + 1], u.y, s);
                        s = fmaf(v[4 * j + 2], u.z, s);
                        s = fmaf(v[4 * j + 3], u.w, s);
                    }
                    acc[r] += s;
                }
            }
        }
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            float a = acc[r];
#pragma unroll
            for (int off = 16; off; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
            if (lane == 0 && r < n) y[(int64_t)r * rows + o] = a;
        }
    }
}

int grid_for(int64_t n, int block)
{
    int64_t g = (n + block - 1) / block;
    const int64_t cap = (int64_t)mb_num_sms() * 16;
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

bool gguf_block(int qtype, int* vals, int* bytes)
{
    switch (qtype) {
    case 2: *vals = 32; *bytes = 18; return true;
    case 3: *vals = 32; *bytes = 20; return true;
    case 6: *vals = 32; *bytes = 22; return true;
    case 7: *vals = 32; *bytes = 24; return true;
    case 8: *vals = 32; *bytes = 34; return true;
    case 10: *vals = 256; *bytes = 84; return true;
    case 11: *vals = 256; *bytes = 110; return true;
    case 12: *vals = 256; *bytes = 144; return true;
    case 13: *vals = 256; *bytes = 176; return true;
    case 14: *vals = 256; *bytes = 210; return true;
    default: return false;
    }
}

}  // namespace

extern "C" int mb_q4_dequant(const uint8_t* raw, const void* scales, int scale_f16, int64_t rows, int64_t cols,
                             int gs, uint8_t xor_mask, float* out, void* stream)
{
    MB_REQUIRE(raw && scales && out, "mb_q4_dequant: null pointer");
    MB_REQUIRE(rows >= 0 && cols >= 0 && gs >= 2 && gs % 2 == 0 && cols % gs == 0,
               "mb_q4_dequant: bad shape rows=%lld cols=%lld gs=%d", (long long)rows, (long long)cols, gs);
    MB_REQUIRE(((uintptr_t)out & 7) == 0, "mb_q4_dequant: out must be 8-byte aligned");
    const int64_t n = rows * (cols / 2);
    if (n == 0) return MB_OK;
    if (scale_f16)
        q4_dequant_kernel<true><<<grid_for(n, 256), 256, 0, mb_stream(stream)>>>(raw, scales, rows, cols, gs,
                                                                                 xor_mask, out);
    else
        q4_dequant_kernel<false><<<grid_for(n, 256), 256, 0, mb_stream(stream)>>>(raw, scales, rows, cols, gs,
                                                                                  xor_mask, out);
    return mb_check_launch("mb_q4_dequant");
}

extern "C" int mb_q8_dequant(const int8_t* q, const void* scales, int scale_f16, int64_t rows, int64_t cols, int gs,
                             float* out, void* stream)
{
    MB_REQUIRE(q && scales && out, "mb_q8_dequant: null pointer");
    MB_REQUIRE(rows >= 0 && cols >= 0 && gs >= 1 && cols % gs == 0, "mb_q8_dequant: bad shape");
    const int64_t n = rows * cols;
    if (n == 0) return MB_OK;
    if (scale_f16)
        q8_dequant_kernel<true><<<grid_for(n, 256), 256, 0, mb_stream(stream)>>>(q, scales, rows, cols, gs, out);
    else
        q8_dequant_kernel<false><<<grid_for(n, 256), 256, 0, mb_stream(stream)>>>(q, scales, rows, cols, gs, out);
    return mb_check_launch("mb_q8_dequant");
}

extern "C" int mb_gguf_dequant(const uint8_t* raw, int qtype, int64_t rows, int64_t row_bytes, int64_t cols,
                               float* out, void* stream)
{
    int vals = 0, bytes = 0;
    MB_REQUIRE(raw && out, "mb_gguf_dequant: null pointer");
    if (!gguf_block(qtype, &vals, &bytes)) return mb_fail(MB_EUNSUPPORTED, "mb_gguf_dequant: GGUF type %d", qtype);
    MB_REQUIRE(cols % vals == 0 && row_bytes == cols / vals * bytes,
               "mb_gguf_dequant: cols=%lld row_bytes=%lld do not fit type %d", (long long)cols,
               (long long)row_bytes, qtype);
    MB_REQUIRE(((uintptr_t)out & 15) == 0, "mb_gguf_dequant: out must be 16-byte aligned");
    const int64_t n = rows * (cols / 32);
    if (n == 0) return MB_OK;
    gguf_dequant_kernel<<<grid_for(n, 128), 128, 0, mb_stream(stream)>>>(raw, qtype, rows, row_bytes, cols, out);
    return mb_check_launch("mb_gguf_dequant");
}

// x @ W.T for a GGUF block-quantised W (rows, row_bytes), a few input rows at a
// time: moelan/kernels.py:981-998 gguf_matmul_t (fused per-type mat-vecs
// _mv_q8_0 482-497, _mv_q4_k 499-527, _mv_q5_k, _mv_q2_k, _mv_q3_k, _mv_q6_k
// 529-676, and the row-decoding _gguf_mm for the other types), every type of
// mb_gguf_dequant.  x (n, cols) f32, y (n, rows) f32, both 16-byte aligned.
extern "C" int mb_gguf_matmul_t(const uint8_t* raw, int qtype, int64_t rows, int64_t row_bytes, int64_t cols,
                                const float* x, int64_t n, float* y, void* stream)
{
    int vals = 0, bytes = 0;
    MB_REQUIRE(raw && x && y, "mb_gguf_matmul_t: null pointer");
    if (!gguf_block(qtype, &vals, &bytes)) return mb_fail(MB_EUNSUPPORTED, "mb_gguf_matmul_t: GGUF type %d", qtype);
    MB_REQUIRE(rows >= 0 && n >= 0 && cols > 0 && cols % vals == 0 && row_bytes == cols / vals * bytes,
               "mb_gguf_matmul_t: cols=%lld row_bytes=%lld do not fit type %d", (long long)cols,
               (long long)row_bytes, qtype);
    MB_REQUIRE(((uintptr_t)x & 15) == 0, "mb_gguf_matmul_t: x must be 16-byte aligned");
    if (rows == 0 || n == 0) return MB_OK;
    cudaStream_t st = mb_stream(stream);
    const int grid = grid_for(rows * 32, 256);
    for (int64_t r0 = 0; r0 < n; r0 += 8) {
        const int nr = (int)std::min<int64_t>(8, n - r0);
        const float* xr = x + r0 * cols;
        float* yr = y + r0 * rows;
#define MB_GGUF_MV(QT)                                                                                      \
    case QT:                                                                                                \
        if (nr == 1) gguf_mv_kernel<QT, 1><<<grid, 256, 0, st>>>(raw, rows, row_bytes, cols, xr, nr, yr);   \
        else if (nr <= 4) gguf_mv_kernel<QT, 4><<<grid, 256, 0, st>>>(raw, rows, row_bytes, cols, xr, nr, yr); \
        else gguf_mv_kernel<QT, 8><<<grid, 256, 0, st>>>(raw, rows, row_bytes, cols, xr, nr, yr);            \
        break;
        switch (qtype) {
            MB_GGUF_MV(2)
            MB_GGUF_MV(3)
            MB_GGUF_MV(6)
            MB_GGUF_MV(7)
            MB_GGUF_MV(8)
            MB_GGUF_MV(10)
            MB_GGUF_MV(11)
            MB_GGUF_MV(12)
            MB_GGUF_MV(13)
            MB_GGUF_MV(14)
        default: break;
        }
#undef MB_GGUF_MV
        const int rc = mb_check_launch("mb_gguf_matmul_t");
        if (rc) return rc;
    }
    return MB_OK;
}
