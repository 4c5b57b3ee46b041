/*
 * moelan_b200.h -- C ABI of libmoelan_b200.so, the sm_100a routed-expert path.
 *
 * Every entry point takes plain device pointers and sizes, a CUDA stream
 * (cudaStream_t passed as void*, never the legacy default stream's special
 * handles other than 0), and returns 0 (MB_OK) or an error code; the message
 * of the last error on the calling thread is mb_last_error().  Calls are
 * stream-ordered and asynchronous; no entry point synchronises the device.
 * The library allocates nothing: scratch comes from caller-provided workspace
 * whose size the *_workspace_bytes functions return.  Buffers are owned by
 * the caller and must stay alive until the stream has run the call.
 *
 * Kernels are launched with programmatic dependent launch and release their
 * successor at entry: a kernel of the caller's that follows one of ours on the
 * same stream with programmatic stream serialisation must execute
 * griddepcontrol.wait (cudaGridDependencySynchronize) before it reads our
 * outputs.  Ordinary launches, copies and events order as usual.
 *
 * Each entry point names the reference (moelan) interface it replaces.
 * Reference paths are relative to the moelan project root.
 */
#ifndef MOELAN_B200_H
#define MOELAN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    MB_OK = 0,
    MB_EINVAL = 1,       /* bad argument (shape, alignment, null pointer) */
    MB_ECUDA = 2,        /* a CUDA runtime error */
    MB_EUNSUPPORTED = 3, /* a format or size this build does not handle */
    MB_EDEVICE = 4       /* a kernel reported a failure in its status word */
};

/* Weight formats of the device tile layout (16-row tiles of 128-column quads,
 * built by distributedmoellm_b200/layout.py). */
enum {
    MB_FMT_Q4_F32 = 1, /* int4, two nibbles per byte, group scales f32 */
    MB_FMT_Q4_F16 = 2, /* int4, group scales f16 */
    MB_FMT_Q8_F32 = 3, /* int8, group scales f32 */
    MB_FMT_Q8_F16 = 4, /* int8, group scales f16 (also GGUF Q8_0 blocks) */
    MB_FMT_Q4K_F32 = 5 /* int4 u with value (u - 8) * scale + bias, f32 scales and biases per group of 32
                          (GGUF Q4_K: scale = d*sc, bias = 8*scale - dmin*m) */
};

/* Wire formats of activation rows (moelan/protocol.py:96 WIRE_FORMATS; f32 rows need no conversion). */
enum {
    MB_WIRE_F16 = 1, /* f16, round to nearest even */
    MB_WIRE_INT8 = 2 /* int8, one f32 scale per group of mb_wire_group(d) values */
};

const char *mb_last_error(void);
int mb_version(void);
/* MB_OK when the current device is an sm_100 part this build runs on. */
int mb_device_check(void);

/* ---- the device tile layout, made on the device ----------------------------- */

/* Bytes of one matrix (O rows, K columns) in the tile layout of format fmt;
 * inter > 0 for a gate|up matrix of 2 * inter rows.  -1 for a bad argument. */
int64_t mb_tiles_bytes(int fmt, int O, int K, int inter);

/* Tiles (MB_FMT_Q4_F16 when scale_f16, else MB_FMT_Q4_F32) from moelan's int4
 * bytes as they are (moelan/experts.py:170-236 Packed4: raw (O, K/2), scales
 * (O, K/gs); xor_mask 0x88 for two's-complement nibbles, 0 for the XOR-ed
 * resident form, as mb_q4_dequant), so a caller holding those arrays needs no
 * host re-layout.  Byte-identical to the layout distributedmoellm_b200/layout.py
 * writes.  tiles: mb_tiles_bytes(fmt, O, K, inter) bytes, 16-byte aligned. */
int mb_pack_q4(const uint8_t *raw, const void *scales, int scale_f16, int O, int K, int gs, uint8_t xor_mask,
               int inter, void *tiles, void *stream);

/* Tiles (MB_FMT_Q8_F16 / MB_FMT_Q8_F32) from moelan's GroupQuant int8 (q (O, K),
 * scales (O, K/gs); moelan/experts.py:125-167), or from GGUF Q8_0 values and
 * their f16 block scales. */
int mb_pack_q8(const int8_t *q, const void *scales, int scale_f16, int O, int K, int gs, int inter, void *tiles,
               void *stream);

/* Affine int4 tiles (MB_FMT_Q4K_F32) from GGUF Q4_K rows as stored (O rows of
 * K/256 144-byte super-blocks; moelan/kernels.py:310-336): nibbles q, scales
 * d*sc, biases 8*d*sc - dmin*m. */
int mb_pack_q4k(const uint8_t *raw, int O, int K, int inter, void *tiles, void *stream);

/* ---- dequantisation (bit-exact) -------------------------------------------- */

/* moelan/kernels.py:971 q4_dequant(raw, s, gs, offset, out) -> _q4_dequant
 * (kernels.py:215-228).  raw (rows, cols/2) u8, scales (rows, cols/gs) f32 or
 * f16 (scale_f16 != 0), xor_mask 0x88 for two's-complement nibbles, 0 for the
 * XOR-ed resident form.  out (rows, cols) f32. */
int mb_q4_dequant(const uint8_t *raw, const void *scales, int scale_f16, int64_t rows, int64_t cols, int gs,
                  uint8_t xor_mask, float *out, void *stream);

/* moelan/kernels.py:976 q8_dequant(q, s, gs, out) -> _q8_dequant (kernels.py:230-237). */
int mb_q8_dequant(const int8_t *q, const void *scales, int scale_f16, int64_t rows, int64_t cols, int gs,
                  float *out, void *stream);

/* moelan/kernels.py:1001 gguf_dequant(raw, qtype, out) and moelan/gguf.py:258
 * dequantize -> _gguf_dequant (kernels.py:693-697).  qtype: ggml type id
 * (2 Q4_0, 3 Q4_1, 6 Q5_0, 7 Q5_1, 8 Q8_0, 10 Q2_K, 11 Q3_K, 12 Q4_K, 13 Q5_K,
 * 14 Q6_K). */
int mb_gguf_dequant(const uint8_t *raw, int qtype, int64_t rows, int64_t row_bytes, int64_t cols, float *out,
                    void *stream);

/* moelan/kernels.py:981 gguf_matmul_t(x, raw, qtype, cols): x @ W.T straight
 * from the GGUF blocks of W (rows, row_bytes), for the few input rows of a
 * decode step (the reference's fused mat-vecs _mv_q8_0 / _mv_q4_k / _mv_q5_k /
 * _mv_q2_k / _mv_q3_k / _mv_q6_k, kernels.py:482-676, and its row-decoding
 * _gguf_mm for the other types).  Every type of mb_gguf_dequant; each weight
 * is decoded bit-exactly, products and sums in f32.  x (n, cols) f32 and
 * y (n, rows) f32, x 16-byte aligned. */
int mb_gguf_matmul_t(const uint8_t *raw, int qtype, int64_t rows, int64_t row_bytes, int64_t cols, const float *x,
                     int64_t n, float *y, void *stream);

/* ---- activation rows in the wire formats --------------------------------------- */

/* Values per int8 scale for rows of width d: 64 when d is a multiple of 64,
 * else the whole row (moelan/protocol.py:96-97, 108). */
int mb_wire_group(int d);

/* moelan/protocol.py:99-114 encode_rows(a, wire, name) on the device, bit-exact:
 * a (n, d) f32 -> q (n, d) f16 (MB_WIRE_F16) or int8 (MB_WIRE_INT8) with scales
 * (n, d / mb_wire_group(d)) f32 = max|group| / 127 (1 for an all-zero group) and
 * q = clip(rint(a / scale), -127, 127). */
int mb_encode_rows(const float *a, int64_t n, int d, int wire, void *q, float *scales, void *stream);

/* moelan/protocol.py:117-123 decode_rows(arrays, name) on the device, bit-exact:
 * q (n, d) f16 or int8 (with its scales) -> out (n, d) f32. */
int mb_decode_rows(const void *q, const float *scales, int64_t n, int d, int wire, float *out, void *stream);

/* ---- router ------------------------------------------------------------------ */

/* Workspace bytes of mb_router_logits / mb_router_route. */
int64_t mb_router_workspace_bytes(int64_t T, int H, int E);

/* Router logits h @ router.T (moelan/model.py:597) in f32 (split over 256-
 * column slices, summed in slice order), plus, when row_exp != NULL, each
 * row's power-of-two exponent used by the mat-vecs. */
int mb_router_logits(const float *x, const float *router, int64_t T, int H, int E, float *logits,
                     int32_t *row_exp, void *workspace, int64_t workspace_bytes, void *stream);

/* Logits and route in two launches: moelan/model.py:597 then model.py:160
 * route(logits, top_k, normalize).  logits and row_exp may be NULL. */
int mb_router_route(const float *x, const float *router, int64_t T, int H, int E, int k, int normalize,
                    float *logits, int32_t *row_exp, int32_t *idx, float *w, void *workspace,
                    int64_t workspace_bytes, void *stream);

/* moelan/model.py:160 route(logits, top_k, normalize) with _top_k
 * (model.py:154-157): f32 softmax, k best experts (ties: lower id first),
 * weights renormalised when normalize != 0.  idx (T, k) i32, w (T, k) f32. */
int mb_router_topk(const float *logits, int64_t T, int E, int k, int normalize, int32_t *idx, float *w,
                   void *stream);

/* moelan/model.py:170-201 route_grouped(logits, cfg, bias): DeepSeek V2 / V3
 * routing on f32 logits (T, E).  Scores: softmax (sigmoid = 0) or sigmoid (1)
 * of the logits; choices: scores + bias (bias (E) f32, or NULL).  method 0
 * greedy, 1 group_limited_greedy (groups ranked by their best choice), 2
 * noaux_tc (by the sum of their two best); with method >= 1 and n_group > 1
 * only the topk_group best of n_group equal groups keep their choices, the
 * others' become 0.  idx (T, k): the k best choices (ties: lower id), w (T, k):
 * their scores, divided by their sum + 1e-20 when k > 1 and normalize (and
 * then multiplied by scaling for noaux_tc), else multiplied by scaling.
 * E <= 1024, k <= 32, n_group <= 32. */
int mb_router_grouped(const float *logits, const float *bias, int64_t T, int E, int k, int sigmoid, int method,
                      int n_group, int topk_group, int normalize, float scaling, int32_t *idx, float *w, void *stream);

/* moelan/model.py:204-223 route_sparsemixer(logits, eps): PhiMoE's top-2.
 * Pick j is the best expert not yet picked, weighted by its softmax over the
 * experts not yet picked whose logit l satisfies (best - l) / max(|l|, best)
 * <= 2 * eps.  idx (T, 2) i32, w (T, 2) f32, not renormalised.  2 <= E <= 1024. */
int mb_router_sparsemixer(const float *logits, int64_t T, int E, double eps, int32_t *idx, float *w, void *stream);

/* Each row's power-of-two exponent (for inputs that did not come through
 * mb_router_logits). */
int mb_row_exponents(const float *x, int64_t T, int H, int32_t *row_exp, void *stream);

/* moelan/model.py:226 group_by_expert(idx, w): stable counting sort of the
 * T*k picks by expert.  Outputs (all device):
 *   counts (E), offsets (E+1)        per expert, over all E experts
 *   sorted_rows (T*k), sorted_w      token and weight of each sorted pick
 *   inv (T*k)                        sorted position of pick t*k+j
 *   uexperts (E), uoffsets (E+1), n_unique (1): the compact form the
 *                                    reference returns (experts, offsets)
 * T*k <= 65536, E <= 1024.  Any output pointer except counts/offsets/
 * sorted_rows may be NULL. */
int mb_permute(const int32_t *idx, const float *w, int64_t T, int k, int E, int32_t *counts, int32_t *offsets,
               int32_t *sorted_rows, float *sorted_w, int32_t *inv, int32_t *uexperts, int32_t *uoffsets,
               int32_t *n_unique, void *stream);

/* The weighted combine out[r] (+)= sum_i pair_w[i] * y[pair_idx[i]] over
 * i in [row_ptr[r], row_ptr[r+1]) in that order (the scatter-adds of
 * moelan/experts.py:711,723,727 and kernels.py:778-782, 968).  When row_ptr
 * is NULL each row has k consecutive entries (i = r*k .. r*k+k-1).
 * accumulate != 0 adds into out, else overwrites.  y (P, H), out (T, H). */
int mb_unpermute_combine(const float *y, const int32_t *row_ptr, const int32_t *pair_idx, const float *pair_w,
                         int64_t T, int k, int H, int accumulate, float *out, void *stream);

/* ---- fused decode mat-vecs over packed experts -------------------------------- */

/* One expert's weights in the device tile layout: gate|up (2I, H) and down
 * (H, I), each a pointer to its tiles (16-byte aligned). */
typedef struct {
    const void *gu;
    const void *down;
} MbExpert;

/* Workspace bytes for mb_moe_decode with P = T*k picks. */
int64_t mb_moe_decode_workspace_bytes(int64_t P, int I);

/* One MoE layer's routed experts, for experts picked by at most max_rows
 * tokens (decode): moelan/kernels.py:942 moe_q4(x, items, H, I, gs, out)
 * (kernels.py:712-782), generalised to int8 experts (kernels.py:133-168) and
 * GGUF Q8_0 down projections.  For each expert e with 0 < counts[e] <=
 * max_rows, its picks offsets[e]..offsets[e+1] of the sorted order (rows of
 * x given by sorted_rows) are run through gate|up, SiLU(gate) * up and down:
 * y (P, H) f32 gets the unweighted expert output of each pick.  Pass row_exp
 * from mb_router_logits / mb_row_exponents.  fmt_gu / fmt_down: MB_FMT_*
 * (GGUF Q4_K gate|up as MB_FMT_Q4K_F32: moelan/kernels.py:499-527 _mv_q4_k).
 * Any H and I (multiples of gs and of 4); K above 2048 is taken in windows of
 * 2048 columns.
 * status: a device word the kernels OR MB_STATUS bits into, or NULL to use
 * a word inside the workspace. */
int mb_moe_decode(const MbExpert *table, int E, int H, int I, int gs, int fmt_gu, int fmt_down, const float *x,
                  const int32_t *row_exp, int64_t T, const int32_t *counts, const int32_t *offsets,
                  const int32_t *sorted_rows, int64_t P, int max_rows, float *y, void *workspace,
                  int64_t workspace_bytes, unsigned *status, void *stream);

/* Size of the scratch array built into the library for mb_moe_decode_noalloc. */
#define MB_NOALLOC_SCRATCH_BYTES (4 << 20)

/* mb_moe_decode for callers that cannot allocate device memory: those that
 * have no device allocator of their own (a binding that only forwards the
 * pointers it is given) or run where allocating is not allowed.  No
 * counterpart in the reference.  Same arguments and results as mb_moe_decode,
 * without the workspace: the scratch is a MB_NOALLOC_SCRATCH_BYTES array
 * inside the library (held on every GPU that loads the library until the
 * process exits), so mb_moe_decode_workspace_bytes(P, I) must fit in it
 * (about 1360 picks at I = 768); larger calls fail with MB_EINVAL.  The
 * call allocates nothing.  The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress); make that first call before any
 * stream capture.  The address is kept for the life of the process, so no
 * call may follow a reset of the device's context (cudaDeviceReset): the
 * kept address would then be stale.  All calls share the one array: calls
 * that overlap on the GPU (other streams, other host threads) race on it and
 * must be ordered by the caller. */
int mb_moe_decode_noalloc(const MbExpert *table, int E, int H, int I, int gs, int fmt_gu, int fmt_down,
                          const float *x, const int32_t *row_exp, int64_t T, const int32_t *counts,
                          const int32_t *offsets, const int32_t *sorted_rows, int64_t P, int max_rows, float *y,
                          unsigned *status, void *stream);

/* ---- prefill: grouped GEMMs on the tensor cores ---------------------------------- */

/* Workspace bytes for mb_moe_prefill with P picks (fmt_gu: the gate|up
 * format; MB_FMT_Q4K_F32 needs room for its precise gate|up products). */
int64_t mb_moe_prefill_workspace_bytes(int64_t P, int H, int I, int fmt_gu);

/* One MoE layer's routed experts for experts picked by at least min_rows
 * tokens (prefill), as grouped GEMMs (tcgen05, f16 operands, f32
 * accumulation): moelan/experts.py:148-151 and 216-219 (matmul_t with 8 or
 * more rows: widen the matrix to f32, x @ W.T), run per expert by
 * ExpertStore.compute (experts.py:707-727) as gate|up, SiLU(gate) * up,
 * down.  Same tables, routing, row_exp and y (P, H) as mb_moe_decode;
 * experts with fewer than min_rows picks are left to mb_moe_decode
 * (max_rows = min_rows - 1).  e_exp (E, 4) int32, per expert: the
 * power-of-two exponents that bring the largest possible weight of its
 * gate|up and of its down matrix into [2^13, 2^14) before rounding to f16,
 * then the activation exponent base a: a pick's SwiGLU activations are
 * scaled by 2^(a + 2 row_exp) before rounding to f16, and a must keep them
 * below 2^15 (a = -13 - ceil(log2(L1g * L1u)) with L1g, L1u the largest
 * row sums of |weight| of the gate and up halves does); the fourth entry is
 * unused.  Results agree with the f32 reference within 2e-3 of each output
 * row's largest magnitude.  With fmt_gu MB_FMT_Q4K_F32 (GGUF Q4_K: affine
 * weights whose activations can be heavy-tailed, where f16 operands alone
 * exceed that bar) the gate|up GEMM runs as three f16 products of the
 * weights' and tokens' f16 pieces (hi*hi + hi*lo + lo*hi) summed in f32.
 * Needs H % 128 == 0, I % 64 == 0, P <= 65536, x and workspace 16-byte
 * aligned. */
int mb_moe_prefill(const MbExpert *table, const int32_t *e_exp, int E, int H, int I, int gs, int fmt_gu,
                   int fmt_down, const float *x, const int32_t *row_exp, int64_t T, const int32_t *counts,
                   const int32_t *offsets, const int32_t *sorted_rows, int64_t P, int min_rows, float *y,
                   void *workspace, int64_t workspace_bytes, unsigned *status, void *stream);

/* ---- expert parallelism over the GPUs of one node (peer memory) ----------
 *
 * The reference's coordinator sends each worker one request per layer with
 * the rows routed to its experts and adds the results back
 * (moelan/coordinator.py:475-535); across the GPUs of one node (one process
 * per GPU) the rows move by stores into the other GPUs' memory instead.
 * Each rank allocates one arena with mb_peer_alloc, the ranks exchange the
 * handles (any host channel), and each maps the others' arenas with
 * mb_peer_open.  Ranks must not use an arena after its owner freed it. */
#define MB_PEER_HANDLE_BYTES 64

/* bytes of device memory, plus the handle (MB_PEER_HANDLE_BYTES) another
 * process of the node passes to mb_peer_open. */
int mb_peer_alloc(int64_t bytes, void **ptr, void *handle);
int mb_peer_open(const void *handle, void **ptr);
int mb_peer_close(void *ptr);   /* a mapping made by mb_peer_open */
int mb_peer_free(void *ptr);    /* an arena made by mb_peer_alloc */

/* One rank's dispatch of its own tokens to their experts' ranks (E experts,
 * expert e on rank e / (E/G)).  Inputs: x (T, H) f32 and row_exp (T,) (from
 * mb_router_route / mb_row_exponents), the picks idx (T, k) and, from
 * mb_permute of them, inv (T*k,) and offsets (E+1,); counts_all (G, E): every
 * rank's per-expert pick counts (row s = rank s's mb_permute counts).  The
 * receive rows of rank d are grouped by d's local expert, within an expert by
 * source rank, within a source in its mb_permute order; pick p of this rank
 * is stored there as the grouped GEMM's f16 operand row (scaled by
 * 2^row_exp, K order as mb_moe_prefill_rows reads it), with its exponent in
 * recv_exp and its return address (rank << 24 | p) in recv_ret.  recv_rows,
 * recv_exp, recv_ret: device arrays of G pointers (each rank's (cap, H) f16,
 * (cap,) and (cap,) int32, as mapped in this process).  Also writes this
 * rank's own receive plan: local_counts (E/G,) and local_offsets (E/G + 1,).
 * A pick that would land at or past cap sets MB_STATUS_BADARG in *status and
 * is skipped; cap = G*T*k always suffices.  Needs T*k < 2^24, H % 128 == 0.
 * The stores into other ranks' memory are complete when the launch is: a
 * stream-ordered collective after it (or any barrier that orders the ranks)
 * makes the rows safe to read on their ranks. */
int mb_ep_dispatch(const float *x, const int32_t *row_exp, int64_t T, int H, const int32_t *idx,
                   const int32_t *inv, int k, const int32_t *offsets, const int32_t *counts_all, int E, int G,
                   int rank, void *const *recv_rows, int32_t *const *recv_exp, int32_t *const *recv_ret,
                   int64_t cap, int32_t *local_counts, int32_t *local_offsets, unsigned *status, void *stream);

/* Workspace bytes for mb_moe_prefill_rows with P rows. */
int64_t mb_moe_prefill_rows_workspace_bytes(int64_t P, int I);

/* mb_moe_prefill over tokens already in the GEMM's f16 operand rows: xp
 * (P, H) as mb_ep_dispatch writes them, row_exp (P,) their exponents,
 * counts / offsets (E / E+1) the rows of each expert (rows past offsets[E]
 * are not read).  Output row p goes to y + p*H, or, when y_ret and y_peers
 * are given, to y_peers[y_ret[p] >> 24] + (y_ret[p] & 0xffffff) * H
 * (y_peers: a device array of n_peers row-buffer pointers, e.g. every rank's
 * result rows as mapped in this process, each of peer_rows rows), stored from
 * the GEMM epilogue; an address outside those buffers sets MB_STATUS_BADARG
 * in *status and its row is not stored.  Not for
 * fmt_gu MB_FMT_Q4K_F32 (MB_EUNSUPPORTED: its precise form needs the f32
 * rows).  P < 2^24. */
int mb_moe_prefill_rows(const MbExpert *table, const int32_t *e_exp, int E, int H, int I, int gs, int fmt_gu,
                        int fmt_down, const void *xp, const int32_t *row_exp, const int32_t *counts,
                        const int32_t *offsets, int64_t P, int min_rows, float *y, const int32_t *y_ret,
                        float *const *y_peers, int n_peers, int64_t peer_rows, void *workspace,
                        int64_t workspace_bytes, unsigned *status, void *stream);

/* Workspace bytes for mb_matmul_t with n input rows. */
int64_t mb_matmul_t_workspace_bytes(int64_t n);

/* x @ W.T for one packed matrix W (O, K) in the device tile layout (fmt
 * MB_FMT_*): moelan/kernels.py:1018 q4_matmul_t and kernels.py:1030
 * q8_matmul_t (GGUF Q8_0 rows too, as int8 tiles with f16 scales:
 * kernels.py:981 gguf_matmul_t).  x (n, K) f32, y (n, O) f32. */
int mb_matmul_t(const void *w_tiles, int fmt, int O, int K, const float *x, int64_t n, float *y, void *workspace,
                int64_t workspace_bytes, unsigned *status, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* MOELAN_B200_H */
