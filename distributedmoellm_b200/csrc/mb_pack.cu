// The device tile layout made on the device from the bytes moelan keeps.
//
// moelan holds an int4 matrix as colibri bytes (raw (O, K/2): two's-complement
// nibbles, low nibble = even column, or XOR-ed with 0x88 in its resident form;
// scales (O, K/gs)) (moelan/experts.py:170-236), an int8 matrix as GroupQuant
// (q (O, K), scales (O, K/gs)) (experts.py:125-167) and GGUF Q4_K rows as
// 144-byte super-blocks (moelan/kernels.py:310-336).  These kernels write the
// tile layout the decode and prefill kernels read, byte for byte what the
// host-side layout functions produce:
//  * rows are cut into 16-row tiles (a gate|up matrix of 2I rows interleaves
//    8 gate rows with the 8 matching up rows per tile), columns into quads of
//    128; a block (tile, quad) holds the quad's values then its 16 x 4 group
//    scales (f16 or f32), padding rows and columns zero weights and scales;
//  * int4: byte 64 r + 16 t + 4 grp + b of a block is byte 16 grp + 4 t + b of
//    row r's quad, nibbles offset by 8 (u = v + 8);
//  * int8: byte 1024 h + 64 r + 16 t + 8 gp + j is column 64 h + 32 gp + 8 t +
//    (0 4 1 5 2 6 3 7)[j] of row r's quad, offset by 128;
//  * affine int4 (Q4_K): the int4 block of the nibbles q, scales d*sc, then
//    16 x 4 f32 biases 8 * d*sc - dmin*m (each product rounded once).
// One CTA per block; the source rows are read where they lie (no staging).
#include "mb_common.cuh"

namespace {

// Source row of tile row tr (-1: padding): gate|up matrices (inter > 0)
// interleave 8 gate rows (j) and the 8 matching up rows (inter + j).
__device__ __forceinline__ int src_row(int tr, int O, int inter)
{
    if (inter > 0) {
        const int rt = tr >> 4, r = tr & 15;
        const int j = rt * 8 + (r & 7);
        if (j >= inter) return -1;
        return r < 8 ? j : inter + j;
    }
    return tr < O ? tr : -1;
}

template <bool F16S>
__device__ __forceinline__ void put_scale(uint8_t* dst, int i, float v)
{
    if (F16S) reinterpret_cast<__half*>(dst)[i] = __float2half_rn(v);
    else reinterpret_cast<float*>(dst)[i] = v;
}

template <bool F16S>
__device__ __forceinline__ float get_scale(const void* s, int64_t i)
{
    if (F16S) return __half2float(reinterpret_cast<const __half*>(s)[i]);
    return reinterpret_cast<const float*>(s)[i];
}

// int4 colibri bytes -> tiles.  grid (NQ, RT), 256 threads.
template <bool F16S>
__global__ void pack_q4_kernel(const uint8_t* __restrict__ raw, const void* __restrict__ s, int O, int K, int gs,
                               uint8_t xr, int inter, uint8_t* __restrict__ tiles)
{
    const int q = blockIdx.x, rt = blockIdx.y, NQ = gridDim.x;
    constexpr int kBlock = 1024 + 64 * (F16S ? 2 : 4);
    uint8_t* blk = tiles + ((int64_t)rt * NQ + q) * kBlock;
    const int tid = threadIdx.x;
    const int KB = K / 2;   // bytes per source row
    {   // one 4-byte word per thread: row r, lane t, group grp
        const int r = tid >> 4, t = (tid >> 2) & 3, grp = tid & 3;
        const int row = src_row(rt * 16 + r, O, inter);
        const int c0 = q * 64 + grp * 16 + t * 4;   // byte of the source row
        uint32_t wv = 0x88888888u;
        if (row >= 0) {
            const uint8_t* src = raw + (int64_t)row * KB;
            uint32_t b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) b[i] = c0 + i < KB ? (uint32_t)(src[c0 + i] ^ xr) : 0x88u;
            wv = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
        }
        reinterpret_cast<uint32_t*>(blk)[r * 16 + t * 4 + grp] = wv;
    }
    if (tid < 64) {   // scales [16 rows][4 groups]
        const int r = tid >> 2, grp = tid & 3;
        const int row = src_row(rt * 16 + r, O, inter);
        const int col = (q * 4 + grp) * 32;
        float v = 0.0f;
        if (row >= 0 && col < K) v = get_scale<F16S>(s, (int64_t)row * (K / gs) + col / gs);
        put_scale<F16S>(blk + 1024, r * 4 + grp, v);
    }
}

// int8 GroupQuant -> tiles.  grid (NQ, RT), 256 threads.
template <bool F16S>
__global__ void pack_q8_kernel(const int8_t* __restrict__ qv, const void* __restrict__ s, int O, int K, int gs,
                               int inter, uint8_t* __restrict__ tiles)
{
    const int q = blockIdx.x, rt = blockIdx.y, NQ = gridDim.x;
    constexpr int kBlock = 2048 + 64 * (F16S ? 2 : 4);
    uint8_t* blk = tiles + ((int64_t)rt * NQ + q) * kBlock;
    const int tid = threadIdx.x;
    // 512 words: half h, row r, lane t, group position gp, word jw (bytes j = 4 jw .. 4 jw + 3)
    for (int wi = tid; wi < 512; wi += blockDim.x) {
        const int h = wi >> 8, r = (wi >> 4) & 15, t = (wi >> 2) & 3, gp = (wi >> 1) & 1, jw = wi & 1;
        const int row = src_row(rt * 16 + r, O, inter);
        const int c0 = q * 128 + h * 64 + gp * 32 + t * 8;
        // bytes j = 4 jw .. 4 jw + 3 hold columns c0 + (0 4 1 5 | 2 6 3 7)
        const int cs[4] = {jw * 2, 4 + jw * 2, jw * 2 + 1, 5 + jw * 2};
        uint32_t wv = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int c = c0 + cs[i];
            const uint32_t u = (row >= 0 && c < K) ? (uint32_t)((uint8_t)qv[(int64_t)row * K + c] ^ 0x80u) : 0x80u;
            wv |= u << (8 * i);
        }
        reinterpret_cast<uint32_t*>(blk)[h * 256 + r * 16 + t * 4 + gp * 2 + jw] = wv;
    }
    if (tid < 64) {
        const int r = tid >> 2, grp = tid & 3;
        const int row = src_row(rt * 16 + r, O, inter);
        const int col = (q * 4 + grp) * 32;
        float v = 0.0f;
        if (row >= 0 && col < K) v = get_scale<F16S>(s, (int64_t)row * (K / gs) + col / gs);
        put_scale<F16S>(blk + 2048, r * 4 + grp, v);
    }
}

// (scale, min) pair j of a K-quant super-block (moelan/kernels.py:310-316).
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t* sb, int& sc, int& m)
{
    if (j < 4) {
        sc = sb[j] & 63;
        m = sb[j + 4] & 63;
    } else {
        sc = (sb[j + 4] & 0xF) | ((sb[j - 4] >> 6) << 4);
        m = (sb[j + 4] >> 4) | ((sb[j] >> 6) << 4);
    }
}

// GGUF Q4_K rows -> affine int4 tiles.  grid (NQ, RT), 256 threads; K a multiple of 256.
__global__ void pack_q4k_kernel(const uint8_t* __restrict__ raw, int O, int K, int inter, uint8_t* __restrict__ tiles)
{
    const int q = blockIdx.x, rt = blockIdx.y, NQ = gridDim.x;
    constexpr int kBlock = 1024 + 256 + 256;
    uint8_t* blk = tiles + ((int64_t)rt * NQ + q) * kBlock;
    const int tid = threadIdx.x;
    const int64_t rb = (int64_t)(K / 256) * 144;   // bytes per row
    {
        const int r = tid >> 4, t = (tid >> 2) & 3, grp = tid & 3;
        const int row = src_row(rt * 16 + r, O, inter);
        uint32_t wv = 0x88888888u;
        const int col0 = q * 128 + grp * 32 + t * 8;   // 8 columns: bytes pack columns (2m, 2m + 1)
        if (row >= 0 && col0 < K) {
            const uint8_t* sb = raw + (int64_t)row * rb + (int64_t)(col0 / 256) * 144;
            const int cc = col0 % 256, c = cc / 64, hi = (cc % 64) / 32, l0 = cc % 32;
            wv = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t a = (sb[16 + 32 * c + l0 + 2 * i] >> (4 * hi)) & 15u;
                const uint32_t b = (sb[16 + 32 * c + l0 + 2 * i + 1] >> (4 * hi)) & 15u;
                wv |= (a | (b << 4)) << (8 * i);
            }
        }
        reinterpret_cast<uint32_t*>(blk)[r * 16 + t * 4 + grp] = wv;
    }
    if (tid < 64) {
        const int r = tid >> 2, grp = tid & 3;
        const int row = src_row(rt * 16 + r, O, inter);
        const int col = (q * 4 + grp) * 32;
        float scale = 0.0f, bias = 0.0f;
        if (row >= 0 && col < K) {
            const uint8_t* sb = raw + (int64_t)row * rb + (int64_t)(col / 256) * 144;
            const float d = mb_f16_ref((uint32_t)sb[0] | ((uint32_t)sb[1] << 8));
            const float dmin = mb_f16_ref((uint32_t)sb[2] | ((uint32_t)sb[3] << 8));
            int sc, m;
            q4k_scale_min((col % 256) / 32, sb + 4, sc, m);
            scale = __fmul_rn(d, (float)sc);
            bias = __fsub_rn(__fmul_rn(8.0f, scale), __fmul_rn(dmin, (float)m));
        }
        reinterpret_cast<float*>(blk + 1024)[r * 4 + grp] = scale;
        reinterpret_cast<float*>(blk + 1280)[r * 4 + grp] = bias;
    }
}

int tile_rows(int O, int inter) { return inter > 0 ? 2 * ((inter + 7) / 8 * 8) : (O + 15) / 16 * 16; }

}  // namespace

extern "C" int64_t mb_tiles_bytes(int fmt, int O, int K, int inter)
{
    int block;
    switch (fmt) {
    case MB_FMT_Q4_F32: block = 1024 + 256; break;
    case MB_FMT_Q4_F16: block = 1024 + 128; break;
    case MB_FMT_Q8_F32: block = 2048 + 256; break;
    case MB_FMT_Q8_F16: block = 2048 + 128; break;
    case MB_FMT_Q4K_F32: block = 1024 + 512; break;
    default: return -1;
    }
    if (O <= 0 || K <= 0) return -1;
    return (int64_t)tile_rows(O, inter) / 16 * ((K + 127) / 128) * block;
}

extern "C" int mb_pack_q4(const uint8_t* raw, const void* scales, int scale_f16, int O, int K, int gs,
                          uint8_t xor_mask, int inter, void* tiles, void* stream)
{
    MB_REQUIRE(raw && scales && tiles, "mb_pack_q4: null pointer");
    MB_REQUIRE(O > 0 && K > 0 && gs >= 32 && gs % 32 == 0 && K % gs == 0, "mb_pack_q4: O=%d K=%d gs=%d", O, K, gs);
    MB_REQUIRE(inter == 0 || O == 2 * inter, "mb_pack_q4: a gate|up matrix has 2 * inter rows");
    MB_REQUIRE(((uintptr_t)tiles & 15) == 0, "mb_pack_q4: tiles must be 16-byte aligned");
    const dim3 grid((K + 127) / 128, tile_rows(O, inter) / 16);
    if (scale_f16)
        pack_q4_kernel<true><<<grid, 256, 0, mb_stream(stream)>>>(raw, scales, O, K, gs, xor_mask, inter,
                                                                  reinterpret_cast<uint8_t*>(tiles));
    else
        pack_q4_kernel<false><<<grid, 256, 0, mb_stream(stream)>>>(raw, scales, O, K, gs, xor_mask, inter,
                                                                   reinterpret_cast<uint8_t*>(tiles));
    return mb_check_launch("mb_pack_q4");
}

extern "C" int mb_pack_q8(const int8_t* q, const void* scales, int scale_f16, int O, int K, int gs, int inter,
                          void* tiles, void* stream)
{
    MB_REQUIRE(q && scales && tiles, "mb_pack_q8: null pointer");
    MB_REQUIRE(O > 0 && K > 0 && gs >= 32 && gs % 32 == 0 && K % gs == 0, "mb_pack_q8: O=%d K=%d gs=%d", O, K, gs);
    MB_REQUIRE(inter == 0 || O == 2 * inter, "mb_pack_q8: a gate|up matrix has 2 * inter rows");
    MB_REQUIRE(((uintptr_t)tiles & 15) == 0, "mb_pack_q8: tiles must be 16-byte aligned");
    const dim3 grid((K + 127) / 128, tile_rows(O, inter) / 16);
    if (scale_f16)
        pack_q8_kernel<true><<<grid, 256, 0, mb_stream(stream)>>>(q, scales, O, K, gs, inter,
                                                                  reinterpret_cast<uint8_t*>(tiles));
    else
        pack_q8_kernel<false><<<grid, 256, 0, mb_stream(stream)>>>(q, scales, O, K, gs, inter,
                                                                   reinterpret_cast<uint8_t*>(tiles));
    return mb_check_launch("mb_pack_q8");
}

extern "C" int mb_pack_q4k(const uint8_t* raw, int O, int K, int inter, void* tiles, void* stream)
{
    MB_REQUIRE(raw && tiles, "mb_pack_q4k: null pointer");
    MB_REQUIRE(O > 0 && K > 0 && K % 256 == 0, "mb_pack_q4k: O=%d K=%d (K a multiple of 256)", O, K);
    MB_REQUIRE(inter == 0 || O == 2 * inter, "mb_pack_q4k: a gate|up matrix has 2 * inter rows");
    MB_REQUIRE(((uintptr_t)tiles & 15) == 0, "mb_pack_q4k: tiles must be 16-byte aligned");
    const dim3 grid((K + 127) / 128, tile_rows(O, inter) / 16);
    pack_q4k_kernel<<<grid, 256, 0, mb_stream(stream)>>>(raw, O, K, inter, reinterpret_cast<uint8_t*>(tiles));
    return mb_check_launch("mb_pack_q4k");
}
