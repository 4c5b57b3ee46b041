/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement of moelan's routed-expert arithmetic (the reference is
 * pure Python + numba; its kernels live in moelan/kernels.py).  This file is
 * the checker that the CUDA path is compared against, and the CPU baseline
 * that bench.py times beside it.  Nothing in the product links or calls it.
 *
 * Every function names the reference lines it restates.  The restatement
 * keeps the reference's order of float operations where the reference pins
 * it (dequantisation is bit-exact: one rounding per value, no contraction --
 * this file is built with -ffp-contract=off), and keeps its summation
 * structure (per-group partial sums, then the group scale) for the fused
 * mat-vecs, whose numba originals run with fastmath and are therefore only
 * reproducible to rounding.
 *
 * Parallelism mirrors the reference: numba's prange over output rows becomes
 * an OpenMP loop over output rows.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- scalar helpers --------------------------------------------------- */

/* IEEE half from two little-endian bytes, as moelan/kernels.py:244-255 does
 * it: exponent 31 maps to +-inf whatever the payload (no NaN). */
static inline float or_f16(uint8_t lo, uint8_t hi)
{
    int h = (int)lo | ((int)hi << 8);
    int e = (h >> 10) & 0x1F;
    int m = h & 0x3FF;
    double v;
    if (e == 0)
        v = (double)m * 5.9604644775390625e-08; /* m * 2^-24, exact */
    else if (e == 31)
        v = INFINITY;
    else
        v = ldexp((double)(1024 + m), e - 25);
    return (float)((h & 0x8000) ? -v : v);
}

static inline int or_i8(uint8_t b) { return (int)(int8_t)b; } /* kernels.py:257-260 */

static inline uint32_t or_u32(const uint8_t *p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

int or_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void or_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0)
        omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ---- group-scaled int4 / int8 dequantisation ------------------------- */

/* moelan/kernels.py:215-228 (_q4_dequant): b = raw ^ xor; the low nibble is
 * the even column, the high nibble the odd one; value = f32(nibble - 8) * s. */
void or_q4_dequant(const uint8_t *raw, const float *s, int64_t O, int64_t K, int gs,
                   uint8_t xr, float *out)
{
    const int64_t ng = K / gs, half = gs / 2, C = K / 2;
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < O; ++o) {
        for (int64_t g = 0; g < ng; ++g) {
            const float sc = s[o * ng + g];
            for (int64_t j = 0; j < half; ++j) {
                const int b = raw[o * C + g * half + j] ^ xr;
                out[o * K + g * gs + 2 * j] = (float)((b & 15) - 8) * sc;
                out[o * K + g * gs + 2 * j + 1] = (float)((b >> 4) - 8) * sc;
            }
        }
    }
}

/* moelan/kernels.py:230-237 (_q8_dequant): f32(q) * s per group. */
void or_q8_dequant(const int8_t *q, const float *s, int64_t O, int64_t K, int gs, float *out)
{
    const int64_t ng = K / gs;
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < O; ++o)
        for (int64_t i = 0; i < K; ++i)
            out[o * K + i] = (float)q[o * K + i] * s[o * ng + i / gs];
}

/* ---- GGUF block decoders (llama.cpp formats, as moelan/kernels.py:262-476) */

static void dq_q8_0(const uint8_t *row, int64_t cols, float *out) /* kernels.py:262-268 */
{
    for (int64_t b = 0; b < cols / 32; ++b) {
        const uint8_t *p = row + b * 34;
        const float d = or_f16(p[0], p[1]);
        for (int j = 0; j < 32; ++j)
            out[b * 32 + j] = d * (float)or_i8(p[2 + j]);
    }
}

static void dq_q4_0(const uint8_t *row, int64_t cols, float *out) /* kernels.py:270-278 */
{
    for (int64_t b = 0; b < cols / 32; ++b) {
        const uint8_t *p = row + b * 18;
        const float d = or_f16(p[0], p[1]);
        for (int j = 0; j < 16; ++j) {
            const int q = p[2 + j];
            out[b * 32 + j] = d * (float)((q & 15) - 8);
            out[b * 32 + j + 16] = d * (float)((q >> 4) - 8);
        }
    }
}

static void dq_q4_1(const uint8_t *row, int64_t cols, float *out) /* kernels.py:280-289 */
{
    for (int64_t b = 0; b < cols / 32; ++b) {
        const uint8_t *p = row + b * 20;
        const float d = or_f16(p[0], p[1]), mn = or_f16(p[2], p[3]);
        for (int j = 0; j < 16; ++j) {
            const int q = p[4 + j];
            out[b * 32 + j] = d * (float)(q & 15) + mn;
            out[b * 32 + j + 16] = d * (float)(q >> 4) + mn;
        }
    }
}

static void dq_q5(const uint8_t *row, int64_t cols, float *out, int with_min) /* kernels.py:291-308 */
{
    const int size = with_min ? 24 : 22;
    for (int64_t b = 0; b < cols / 32; ++b) {
        const uint8_t *p = row + b * size;
        const float d = or_f16(p[0], p[1]);
        const float mn = with_min ? or_f16(p[2], p[3]) : 0.0f;
        const uint8_t *h = p + (with_min ? 4 : 2);
        const int64_t qh = (int64_t)or_u32(h);
        const uint8_t *qs = h + 4;
        const int off = with_min ? 0 : 16;
        for (int j = 0; j < 16; ++j) {
            const int64_t q = qs[j];
            const int64_t x0 = ((q & 15) | (((qh >> j) << 4) & 0x10)) - off;
            const int64_t x1 = ((q >> 4) | ((qh >> (j + 12)) & 0x10)) - off;
            out[b * 32 + j] = d * (float)x0 + mn;
            out[b * 32 + j + 16] = d * (float)x1 + mn;
        }
    }
}

/* 6-bit (scale, min) pair j of a K-quant super-block (kernels.py:310-316). */
static inline void scale_min_k4(int j, const uint8_t *s, int *sc, int *m)
{
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static void dq_q4_k(const uint8_t *row, int64_t cols, float *out) /* kernels.py:318-336 */
{
    for (int64_t b = 0; b < cols / 256; ++b) {
        const uint8_t *p = row + b * 144;
        const float d = or_f16(p[0], p[1]), dmin = or_f16(p[2], p[3]);
        const uint8_t *q = p + 16;
        float *y = out + b * 256;
        for (int k = 0; k < 4; ++k) {
            int sc, m;
            scale_min_k4(2 * k, p + 4, &sc, &m);
            const float d1 = d * (float)sc, m1 = dmin * (float)m;
            scale_min_k4(2 * k + 1, p + 4, &sc, &m);
            const float d2 = d * (float)sc, m2 = dmin * (float)m;
            for (int l = 0; l < 32; ++l) {
                y[l] = d1 * (float)(q[l] & 15) - m1;
                y[32 + l] = d2 * (float)(q[l] >> 4) - m2;
            }
            q += 32;
            y += 64;
        }
    }
}

static void dq_q5_k(const uint8_t *row, int64_t cols, float *out) /* kernels.py:338-361 */
{
    for (int64_t b = 0; b < cols / 256; ++b) {
        const uint8_t *p = row + b * 176;
        const float d = or_f16(p[0], p[1]), dmin = or_f16(p[2], p[3]);
        const uint8_t *qh = p + 16, *ql = p + 48;
        float *y = out + b * 256;
        int u1 = 1, u2 = 2;
        for (int k = 0; k < 4; ++k) {
            int sc, m;
            scale_min_k4(2 * k, p + 4, &sc, &m);
            const float d1 = d * (float)sc, m1 = dmin * (float)m;
            scale_min_k4(2 * k + 1, p + 4, &sc, &m);
            const float d2 = d * (float)sc, m2 = dmin * (float)m;
            for (int l = 0; l < 32; ++l) {
                y[l] = d1 * (float)((ql[l] & 15) + ((qh[l] & u1) ? 16 : 0)) - m1;
                y[32 + l] = d2 * (float)((ql[l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2;
            }
            ql += 32;
            y += 64;
            u1 <<= 2;
            u2 <<= 2;
        }
    }
}

static void dq_q6_k(const uint8_t *row, int64_t cols, float *out) /* kernels.py:363-387 */
{
    for (int64_t b = 0; b < cols / 256; ++b) {
        const uint8_t *p = row + b * 210;
        const float d = or_f16(p[208], p[209]);
        const uint8_t *ql = p, *qh = p + 128, *sc = p + 192;
        float *y = out + b * 256;
        for (int n = 0; n < 2; ++n) {
            for (int l = 0; l < 32; ++l) {
                const int s = l / 16;
                const int a = ql[l], c = ql[l + 32], h = qh[l];
                const int q1 = ((a & 15) | (((h >> 0) & 3) << 4)) - 32;
                const int q2 = ((c & 15) | (((h >> 2) & 3) << 4)) - 32;
                const int q3 = ((a >> 4) | (((h >> 4) & 3) << 4)) - 32;
                const int q4 = ((c >> 4) | (((h >> 6) & 3) << 4)) - 32;
                y[l] = d * (float)(or_i8(sc[s]) * q1);
                y[l + 32] = d * (float)(or_i8(sc[s + 2]) * q2);
                y[l + 64] = d * (float)(or_i8(sc[s + 4]) * q3);
                y[l + 96] = d * (float)(or_i8(sc[s + 6]) * q4);
            }
            y += 128;
            ql += 64;
            qh += 32;
            sc += 8;
        }
    }
}

static void dq_q2_k(const uint8_t *row, int64_t cols, float *out) /* kernels.py:389-414 */
{
    for (int64_t b = 0; b < cols / 256; ++b) {
        const uint8_t *p = row + b * 84;
        const float d = or_f16(p[80], p[81]), dmin = or_f16(p[82], p[83]);
        const uint8_t *q = p + 16;
        float *y = out + b * 256;
        int i = 0;
        for (int n = 0; n < 2; ++n) {
            int shift = 0;
            for (int j = 0; j < 4; ++j) {
                int s = p[i++];
                float dl = d * (float)(s & 15), ml = dmin * (float)(s >> 4);
                for (int l = 0; l < 16; ++l)
                    *y++ = dl * (float)((q[l] >> shift) & 3) - ml;
                s = p[i++];
                dl = d * (float)(s & 15);
                ml = dmin * (float)(s >> 4);
                for (int l = 0; l < 16; ++l)
                    *y++ = dl * (float)((q[l + 16] >> shift) & 3) - ml;
                shift += 2;
            }
            q += 32;
        }
    }
}

static void dq_q3_k(const uint8_t *row, int64_t cols, float *out) /* kernels.py:416-453 */
{
    const int64_t km1 = 0x03030303, km2 = 0x0F0F0F0F;
    for (int64_t b = 0; b < cols / 256; ++b) {
        const uint8_t *p = row + b * 110;
        const float d = or_f16(p[108], p[109]);
        const int64_t a0 = or_u32(p + 96), a1 = or_u32(p + 100), t = or_u32(p + 104);
        const int64_t words[4] = {(a0 & km2) | (((t >> 0) & km1) << 4), (a1 & km2) | (((t >> 2) & km1) << 4),
                                  ((a0 >> 4) & km2) | (((t >> 4) & km1) << 4),
                                  ((a1 >> 4) & km2) | (((t >> 6) & km1) << 4)};
        int scales[16];
        for (int w = 0; w < 4; ++w)
            for (int k = 0; k < 4; ++k)
                scales[w * 4 + k] = (int)((words[w] >> (8 * k)) & 0xFF) - 32;
        const uint8_t *hm = p, *q = p + 32;
        float *y = out + b * 256;
        int m = 1, i = 0;
        for (int n = 0; n < 2; ++n) {
            int shift = 0;
            for (int j = 0; j < 4; ++j) {
                float dl = d * (float)scales[i++];
                for (int l = 0; l < 16; ++l) {
                    const int v = ((q[l] >> shift) & 3) - ((hm[l] & m) ? 0 : 4);
                    *y++ = dl * (float)v;
                }
                dl = d * (float)scales[i++];
                for (int l = 0; l < 16; ++l) {
                    const int v = ((q[l + 16] >> shift) & 3) - ((hm[l + 16] & m) ? 0 : 4);
                    *y++ = dl * (float)v;
                }
                shift += 2;
                m <<= 1;
            }
            q += 32;
        }
    }
}

/* One row of any supported block type (kernels.py:455-476).  Returns 0, or -1
 * for an unknown type id. */
static int gguf_row(const uint8_t *row, int qtype, int64_t cols, float *out)
{
    switch (qtype) {
    case 8: dq_q8_0(row, cols, out); return 0;
    case 12: dq_q4_k(row, cols, out); return 0;
    case 14: dq_q6_k(row, cols, out); return 0;
    case 13: dq_q5_k(row, cols, out); return 0;
    case 2: dq_q4_0(row, cols, out); return 0;
    case 3: dq_q4_1(row, cols, out); return 0;
    case 6: dq_q5(row, cols, out, 0); return 0;
    case 7: dq_q5(row, cols, out, 1); return 0;
    case 10: dq_q2_k(row, cols, out); return 0;
    case 11: dq_q3_k(row, cols, out); return 0;
    default: return -1;
    }
}

/* moelan/kernels.py:693-697 (_gguf_dequant): (rows, row_bytes) -> (rows, cols). */
int or_gguf_dequant(const uint8_t *raw, int qtype, int64_t rows, int64_t row_bytes, int64_t cols, float *out)
{
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (int64_t o = 0; o < rows; ++o)
        bad |= gguf_row(raw + o * row_bytes, qtype, cols, out + o * cols) ? 1 : 0;
    return bad ? -1 : 0;
}

/* ---- mat-vecs straight from packed bytes ------------------------------ */

/* x @ W.T for colibri int4 (moelan/kernels.py:85-106 _q4, and the host
 * correction of q4_matmul_t, kernels.py:1018-1027): nibbles are read unsigned
 * (u = v + 8), each group's partial sum is scaled, and 8 * sum_g s * sum(x in g)
 * is taken off. */
void or_q4_matmul_t(const float *x, int64_t n, const uint8_t *raw, const float *s, int64_t O, int64_t K,
                    int gs, uint8_t xr, float *y)
{
    const int64_t ng = K / gs, half = gs / 2, C = K / 2;
    float *xsum = (float *)malloc(sizeof(float) * (size_t)(n * ng));
    for (int64_t r = 0; r < n; ++r)
        for (int64_t g = 0; g < ng; ++g) {
            float a = 0.0f;
            for (int64_t i = 0; i < gs; ++i)
                a += x[r * K + g * gs + i];
            xsum[r * ng + g] = a;
        }
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < O; ++o) {
        for (int64_t r = 0; r < n; ++r) {
            const float *xr_ = x + r * K;
            float acc = 0.0f, corr = 0.0f;
            for (int64_t g = 0; g < ng; ++g) {
                float part = 0.0f;
                const uint8_t *b0 = raw + o * C + g * half;
                const float *xg = xr_ + g * gs;
#pragma omp simd reduction(+ : part)
                for (int64_t j = 0; j < half; ++j) {
                    const int b = b0[j] ^ xr;
                    part += (float)(b & 15) * xg[2 * j] + (float)(b >> 4) * xg[2 * j + 1];
                }
                acc += part * s[o * ng + g];
                corr += s[o * ng + g] * xsum[r * ng + g];
            }
            y[r * O + o] = acc - 8.0f * corr;
        }
    }
    free(xsum);
}

/* x @ W.T for group-scaled int8 (moelan/kernels.py:152-168 _q8). */
void or_q8_matmul_t(const float *x, int64_t n, const int8_t *q, const float *s, int64_t O, int64_t K, int gs,
                    float *y)
{
    const int64_t ng = K / gs;
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < O; ++o) {
        for (int64_t r = 0; r < n; ++r) {
            float acc = 0.0f;
            for (int64_t g = 0; g < ng; ++g) {
                float part = 0.0f;
                const int8_t *qg = q + o * K + g * gs;
                const float *xg = x + r * K + g * gs;
#pragma omp simd reduction(+ : part)
                for (int64_t i = 0; i < gs; ++i)
                    part += (float)qg[i] * xg[i];
                acc += part * s[o * ng + g];
            }
            y[r * O + o] = acc;
        }
    }
}

/* Fused GGUF mat-vecs.  Q8_0: moelan/kernels.py:482-497 (_mv_q8_0); Q4_K:
 * kernels.py:499-527 (_mv_q4_k) with xs = per-32 sums of x.  Other types go
 * through the row decoder and a dot product (kernels.py:678-691 _gguf_mm).
 * Returns -1 for an unknown type. */
int or_gguf_matmul_t(const float *x, int64_t n, const uint8_t *raw, int qtype, int64_t O, int64_t row_bytes,
                     int64_t cols, float *y)
{
    if (qtype == 8) {
#pragma omp parallel for schedule(static)
        for (int64_t o = 0; o < O; ++o) {
            const uint8_t *row = raw + o * row_bytes;
            for (int64_t r = 0; r < n; ++r) {
                float acc = 0.0f;
                for (int64_t b = 0; b < cols / 32; ++b) {
                    const uint8_t *p = row + b * 34;
                    float s = 0.0f;
                    for (int j = 0; j < 32; ++j)
                        s += (float)or_i8(p[2 + j]) * x[r * cols + b * 32 + j];
                    acc += or_f16(p[0], p[1]) * s;
                }
                y[r * O + o] = acc;
            }
        }
        return 0;
    }
    if (qtype == 12) {
        const int64_t ns = cols / 32;
        float *xs = (float *)malloc(sizeof(float) * (size_t)(n * ns));
        for (int64_t r = 0; r < n; ++r)
            for (int64_t g = 0; g < ns; ++g) {
                float a = 0.0f;
                for (int i = 0; i < 32; ++i)
                    a += x[r * cols + g * 32 + i];
                xs[r * ns + g] = a;
            }
#pragma omp parallel for schedule(static)
        for (int64_t o = 0; o < O; ++o) {
            const uint8_t *row = raw + o * row_bytes;
            for (int64_t r = 0; r < n; ++r) {
                float acc = 0.0f;
                for (int64_t b = 0; b < cols / 256; ++b) {
                    const uint8_t *p = row + b * 144;
                    const float d = or_f16(p[0], p[1]), dmin = or_f16(p[2], p[3]);
                    for (int k = 0; k < 4; ++k) {
                        int sc1, m1, sc2, m2;
                        scale_min_k4(2 * k, p + 4, &sc1, &m1);
                        scale_min_k4(2 * k + 1, p + 4, &sc2, &m2);
                        const uint8_t *q = p + 16 + k * 32;
                        const int64_t x0 = b * 256 + k * 64;
                        float s1 = 0.0f, s2 = 0.0f;
                        for (int l = 0; l < 32; ++l) {
                            s1 += (float)(q[l] & 15) * x[r * cols + x0 + l];
                            s2 += (float)(q[l] >> 4) * x[r * cols + x0 + 32 + l];
                        }
                        const int64_t g = x0 / 32;
                        acc += d * ((float)sc1 * s1 + (float)sc2 * s2) -
                               dmin * ((float)m1 * xs[r * ns + g] + (float)m2 * xs[r * ns + g + 1]);
                    }
                }
                y[r * O + o] = acc;
            }
        }
        free(xs);
        return 0;
    }
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (int64_t o = 0; o < O; ++o) {
        float *w = (float *)malloc(sizeof(float) * (size_t)cols);
        if (gguf_row(raw + o * row_bytes, qtype, cols, w))
            bad = 1;
        else
            for (int64_t r = 0; r < n; ++r) {
                float acc = 0.0f;
                for (int64_t i = 0; i < cols; ++i)
                    acc += w[i] * x[r * cols + i];
                y[r * O + o] = acc;
            }
        free(w);
    }
    return bad ? -1 : 0;
}

/* ---- one MoE layer's int4 experts in one call ------------------------ */

/* moelan/kernels.py:712-782 (_moe_q4) called as kernels.py:942-968 (moe_q4).
 *   xs    (n, H)   the distinct input rows (x[uniq] in the reference)
 *   ptrs  (k, 4)   addresses of each expert's gate|up bytes, their f32
 *                  scales, down bytes, their f32 scales
 *   xors  (k,)     0 for resident (offset) copies, 0x88 for raw nibbles
 *   poff  (k+1,)   pairs of expert e are poff[e]..poff[e+1]
 *   prow  (P,)     row of xs for each pair; pw (P,) its gate weight
 *   part  (n, H)   += sum over pairs of w * expert(x)
 * Gate|up: 2I rows over H; SiLU(gate) * up; down: H rows over I.  Nibbles are
 * unsigned (u = v + 8) and 8 * sum_g s * sum(x in g) is taken off (744-745,
 * 769-777).  Pairs are added in pair order (778-782). */
void or_moe_q4(const float *xs, int64_t n, const int64_t *ptrs, const uint8_t *xors, const int64_t *poff,
               int64_t k, const int64_t *prow, const float *pw, int64_t H, int64_t I, int gs, float *part)
{
    const int64_t P = poff[k];
    const int64_t O1 = 2 * I, C1 = H / 2, G1 = H / gs, C2 = I / 2, G2 = I / gs, half = gs / 2;
    float *xsum = (float *)malloc(sizeof(float) * (size_t)(n * G1));
    float *h = (float *)malloc(sizeof(float) * (size_t)(P * O1));
    float *act = (float *)malloc(sizeof(float) * (size_t)(P * I));
    float *asum = (float *)malloc(sizeof(float) * (size_t)(P * G2));
    float *y = (float *)malloc(sizeof(float) * (size_t)(P * H));
    for (int64_t r = 0; r < n; ++r)
        for (int64_t g = 0; g < G1; ++g) {
            float a = 0.0f;
            for (int64_t i = 0; i < gs; ++i)
                a += xs[r * H + g * gs + i];
            xsum[r * G1 + g] = a;
        }
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < k * O1; ++t) {
        const int64_t e = t / O1, o = t - e * O1;
        const uint8_t *raw = (const uint8_t *)(intptr_t)ptrs[e * 4 + 0];
        const float *sc = (const float *)(intptr_t)ptrs[e * 4 + 1];
        const uint8_t xr = xors[e];
        for (int64_t p = poff[e]; p < poff[e + 1]; ++p) {
            const float *xr_ = xs + prow[p] * H;
            float acc = 0.0f, corr = 0.0f;
            for (int64_t g = 0; g < G1; ++g) {
                float pt = 0.0f;
                const uint8_t *b0 = raw + o * C1 + g * half;
                const float *xg = xr_ + g * gs;
#pragma omp simd reduction(+ : pt)
                for (int64_t j = 0; j < half; ++j) {
                    const int b = b0[j] ^ xr;
                    pt += (float)(b & 15) * xg[2 * j] + (float)(b >> 4) * xg[2 * j + 1];
                }
                acc += pt * sc[o * G1 + g];
                corr += sc[o * G1 + g] * xsum[prow[p] * G1 + g];
            }
            h[p * O1 + o] = acc - 8.0f * corr;
        }
    }
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < P; ++p) {
        for (int64_t j = 0; j < I; ++j) {
            const float g0 = h[p * O1 + j];
            act[p * I + j] = g0 / (1.0f + expf(-g0)) * h[p * O1 + I + j];
        }
        for (int64_t g = 0; g < G2; ++g) {
            float a = 0.0f;
            for (int64_t i = 0; i < gs; ++i)
                a += act[p * I + g * gs + i];
            asum[p * G2 + g] = a;
        }
    }
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < k * H; ++t) {
        const int64_t e = t / H, o = t - e * H;
        const uint8_t *raw = (const uint8_t *)(intptr_t)ptrs[e * 4 + 2];
        const float *sc = (const float *)(intptr_t)ptrs[e * 4 + 3];
        const uint8_t xr = xors[e];
        for (int64_t p = poff[e]; p < poff[e + 1]; ++p) {
            const float *a = act + p * I;
            float acc = 0.0f, corr = 0.0f;
            for (int64_t g = 0; g < G2; ++g) {
                float pt = 0.0f;
                const uint8_t *b0 = raw + o * C2 + g * half;
                const float *ag = a + g * gs;
#pragma omp simd reduction(+ : pt)
                for (int64_t j = 0; j < half; ++j) {
                    const int b = b0[j] ^ xr;
                    pt += (float)(b & 15) * ag[2 * j] + (float)(b >> 4) * ag[2 * j + 1];
                }
                acc += pt * sc[o * G2 + g];
                corr += sc[o * G2 + g] * asum[p * G2 + g];
            }
            y[p * H + o] = acc - 8.0f * corr;
        }
    }
    for (int64_t p = 0; p < P; ++p) {
        const float w = pw[p];
        float *dst = part + prow[p] * H;
        for (int64_t j = 0; j < H; ++j)
            dst[j] += w * y[p * H + j];
    }
    free(xsum);
    free(h);
    free(act);
    free(asum);
    free(y);
}
