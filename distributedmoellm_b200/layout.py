"""The device tile layout of packed expert weights.

The reference keeps a matrix W (O rows, K columns) as moelan stores it
(moelan/experts.py:125-236): int4 ``raw`` (O, K/2) bytes, two
two's-complement nibbles per byte, low nibble = even column, plus ``s``
(O, K/gs) scales; int8 ``q`` (O, K) plus ``s``.  The decode kernels read a
re-arranged copy, made once when an expert is uploaded:

* rows are cut into tiles of 16; columns into quads of 128 (four groups of
  32).  A tile is a contiguous run of NQ = ceil(K/128) blocks, so one bulk
  copy moves a whole tile into shared memory;
* int4 block (1024 bytes of nibbles): [16 rows][4 lanes t][16 bytes], the 16
  bytes being word t (bytes 4t..4t+3, columns 8t..8t+7) of each of the quad's
  four groups.  Nibbles are stored offset by 8 (u = v + 8, the reference's
  XOR-0x88 "resident" form, experts.py:188-191);
* int8 block (2048 bytes): [2 halves][16 rows][4 lanes t][16 bytes], half h
  holding groups 2h and 2h+1, each as the 8 bytes of columns 8t..8t+7 in the
  order [c0 c4 c1 c5 c2 c6 c3 c7], offset by 128 (u = q + 128);
* each block is followed by its scales: [16 rows][4 groups] in f16 or f32
  (one per group of 32 columns; a group size of 64 or more repeats its scale);
* padding rows and columns hold zero weights and zero scales;
* an affine int4 block (GGUF Q4_K, value = (u - 8) * scale + bias per group
  of 32) is the int4 block followed by [16 rows][4 groups] f32 biases
  (1536 bytes);
* a gate|up matrix (2I rows) interleaves its halves: tile i holds gate rows
  8i..8i+7 and then up rows 8i..8i+7, so one tile yields SiLU(gate) * up.

These are the layouts the kernels in csrc/mb_decode.cu index; the lane
shapes follow the mma.sync m16n8k16 fragment layout.
"""

from __future__ import annotations

import numpy as np

FMT_Q4_F32, FMT_Q4_F16, FMT_Q8_F32, FMT_Q8_F16, FMT_Q4K_F32 = 1, 2, 3, 4, 5
TILE_ROWS, QUAD_COLS = 16, 128


def is_q8(fmt: int) -> bool:
    return fmt in (FMT_Q8_F32, FMT_Q8_F16)


def scale_is_f16(fmt: int) -> bool:
    return fmt in (FMT_Q4_F16, FMT_Q8_F16)


def block_bytes(fmt: int) -> int:
    if fmt == FMT_Q4K_F32:
        return 1024 + 64 * 4 + 64 * 4
    return (2048 if is_q8(fmt) else 1024) + 64 * (2 if scale_is_f16(fmt) else 4)


def fmt_of(kind: str, scales: np.ndarray) -> int:
    f16 = np.asarray(scales).dtype == np.float16
    if kind == "q4":
        return FMT_Q4_F16 if f16 else FMT_Q4_F32
    if kind == "q8":
        return FMT_Q8_F16 if f16 else FMT_Q8_F32
    raise ValueError(kind)


def padded_rows(O: int, gu_inter: int = 0) -> int:
    if gu_inter:
        return 2 * ((gu_inter + 7) // 8 * 8)
    return (O + TILE_ROWS - 1) // TILE_ROWS * TILE_ROWS


def tiles_nbytes(fmt: int, O: int, K: int, gu_inter: int = 0) -> int:
    nq = (K + QUAD_COLS - 1) // QUAD_COLS
    return padded_rows(O, gu_inter) // TILE_ROWS * nq * block_bytes(fmt)


def row_order(O: int, gu_inter: int = 0) -> np.ndarray:
    """Source row of each tile row (-1: padding)."""
    if gu_inter:
        I = gu_inter
        I8 = (I + 7) // 8 * 8
        j = np.arange(I8).reshape(-1, 8)
        gate = np.where(j < I, j, -1)
        up = np.where(j < I, I + j, -1)
        return np.concatenate([gate, up], axis=1).reshape(-1)
    Op = padded_rows(O)
    r = np.arange(Op)
    return np.where(r < O, r, -1)


def _group_scales(s: np.ndarray, order: np.ndarray, K: int, gs: int, dtype) -> np.ndarray:
    Kp = (K + QUAD_COLS - 1) // QUAD_COLS * QUAD_COLS
    G, Gr = Kp // 32, K // 32
    S = np.zeros((len(order), G), dtype)
    ok = order >= 0
    S[ok, :Gr] = np.asarray(s)[order[ok]][:, (np.arange(Gr) * 32) // gs].astype(dtype)
    return S


def _check(K: int, gs: int) -> None:
    if gs % 32 or K % gs:
        raise ValueError(f"the tile layout needs a group size that is a multiple of 32 and divides K "
                         f"(gs={gs}, K={K})")


def q4_tiles(raw: np.ndarray, s: np.ndarray, gs: int, offset: bool = False, gu_inter: int = 0) -> np.ndarray:
    """Tile bytes of a colibri int4 matrix.  ``offset``: ``raw`` already holds
    u = v + 8 (XOR-ed with 0x88).  ``gu_inter``: I, for a gate|up matrix."""
    raw = np.ascontiguousarray(raw, np.uint8)
    O, K = raw.shape[0], raw.shape[1] * 2
    _check(K, gs)
    sdt = np.float16 if np.asarray(s).dtype == np.float16 else np.float32
    order = row_order(O, gu_inter)
    Kp = (K + QUAD_COLS - 1) // QUAD_COLS * QUAD_COLS
    NQ, RT = Kp // QUAD_COLS, len(order) // TILE_ROWS
    U = np.full((len(order), Kp // 2), 0x88, np.uint8)
    ok = order >= 0
    U[ok, :K // 2] = raw[order[ok]] if offset else raw[order[ok]] ^ np.uint8(0x88)
    nib = U.reshape(RT, TILE_ROWS, NQ, 4, 4, 4).transpose(0, 2, 1, 4, 3, 5).reshape(RT, NQ, 1024)
    S = _group_scales(s, order, K, gs, sdt)
    sc = S.reshape(RT, TILE_ROWS, NQ, 4).transpose(0, 2, 1, 3)
    sc = np.ascontiguousarray(sc).view(np.uint8).reshape(RT, NQ, -1)
    return np.ascontiguousarray(np.concatenate([nib, sc], axis=2).reshape(-1))


_Q8_PERM = np.array([0, 4, 1, 5, 2, 6, 3, 7])


def q8_tiles(q: np.ndarray, s: np.ndarray, gs: int, gu_inter: int = 0) -> np.ndarray:
    """Tile bytes of a group-scaled int8 matrix (moelan GroupQuant)."""
    q = np.ascontiguousarray(q, np.int8)
    O, K = q.shape
    _check(K, gs)
    sdt = np.float16 if np.asarray(s).dtype == np.float16 else np.float32
    order = row_order(O, gu_inter)
    Kp = (K + QUAD_COLS - 1) // QUAD_COLS * QUAD_COLS
    NQ, RT = Kp // QUAD_COLS, len(order) // TILE_ROWS
    U = np.full((len(order), Kp), 0x80, np.uint8)
    ok = order >= 0
    U[ok, :K] = q[order[ok]].view(np.uint8) ^ np.uint8(0x80)
    v = U.reshape(RT, TILE_ROWS, NQ, 2, 2, 4, 8)[..., _Q8_PERM]   # (rt, row, q, half, gpos, t, 8)
    v = v.transpose(0, 2, 3, 1, 5, 4, 6).reshape(RT, NQ, 2048)     # (rt, q, half, row, t, gpos, 8)
    S = _group_scales(s, order, K, gs, sdt)
    sc = S.reshape(RT, TILE_ROWS, NQ, 4).transpose(0, 2, 1, 3)
    sc = np.ascontiguousarray(sc).view(np.uint8).reshape(RT, NQ, -1)
    return np.ascontiguousarray(np.concatenate([v, sc], axis=2).reshape(-1))


def q8_0_as_q8(raw: np.ndarray, cols: int):
    """GGUF Q8_0 rows (O, cols/32 * 34) -> (int8 values (O, cols), f16 scales
    (O, cols/32)): the same numbers as the Q8_0 block decoder
    (moelan/kernels.py:262-268) for finite scales."""
    raw = np.ascontiguousarray(raw, np.uint8)
    O = raw.shape[0]
    b = raw.reshape(O, cols // 32, 34)
    d = np.ascontiguousarray(b[:, :, :2]).view(np.float16).reshape(O, cols // 32)
    q = np.ascontiguousarray(b[:, :, 2:]).view(np.int8).reshape(O, cols)
    return q, d


def exponent_for(amax: float) -> int:
    """The power-of-two exponent e with amax * 2^e in [2^13, 2^14) (0 for
    zero or non-finite amax)."""
    if not (0.0 < amax < 3.0e38):
        return 0
    _, ex = np.frexp(np.float32(amax))
    return int(min(120, max(-120, 14 - int(ex))))


def weight_exponent(s, qmax: int) -> int:
    """The power-of-two exponent e that maps a matrix whose weights are at
    most qmax * max|s| in magnitude into [2^13, 2^14) (0 for an all-zero or
    non-finite bound): the tensor-core path multiplies the weights by 2^e
    before rounding them to f16, and the accumulators by 2^-e after."""
    amax = float(np.max(np.abs(np.asarray(s, np.float32)))) * qmax if np.size(s) else 0.0
    if not (0.0 < amax < 3.0e38):
        return 0
    _, ex = np.frexp(np.float32(amax))
    return int(min(120, max(-120, 14 - int(ex))))


def row_l1_q4(raw: np.ndarray, s, gs: int, offset: bool = False) -> np.ndarray:
    """Per row sum of |weight| of a colibri int4 matrix (float64)."""
    raw = np.asarray(raw, np.uint8)
    O, K = raw.shape[0], raw.shape[1] * 2
    lo, hi = (raw & 15).astype(np.int16), (raw >> 4).astype(np.int16)
    if offset:
        lo, hi = lo - 8, hi - 8
    else:
        lo, hi = np.where(lo >= 8, lo - 16, lo), np.where(hi >= 8, hi - 16, hi)
    g = (np.abs(lo) + np.abs(hi)).reshape(O, K // gs, gs // 2).sum(axis=2)
    return (g * np.asarray(s, np.float64)).sum(axis=1)


def row_l1_q8(q: np.ndarray, s, gs: int) -> np.ndarray:
    """Per row sum of |weight| of a group-scaled int8 matrix (float64)."""
    q = np.asarray(q, np.int8)
    O, K = q.shape
    g = np.abs(q.astype(np.int16)).reshape(O, K // gs, gs).sum(axis=2)
    return (g * np.asarray(s, np.float64)).sum(axis=1)


def act_exponent(gu_row_l1: np.ndarray, inter: int) -> int:
    """The activation exponent base a of an expert for the tensor-core path:
    with a token row's largest value below 2^(14 - row_exp), its SwiGLU
    activations satisfy |SiLU(g) u| <= |g| |u| < 2^(28 - 2 row_exp) * L1g * L1u
    (L1g, L1u: the largest row sums of |weight| of the gate and up halves), so
    scaling them by 2^(a + 2 row_exp) with a = -13 - ceil(log2(L1g * L1u))
    keeps them below 2^15, inside f16."""
    l1 = np.asarray(gu_row_l1, np.float64)
    b = float(l1[:inter].max(initial=0.0)) * float(l1[inter:].max(initial=0.0))
    if not (0.0 < b < 1e300):
        return 0
    return int(min(120, max(-120, -13 - int(np.ceil(np.log2(b))))))


def _f16_ref(bits: np.ndarray) -> np.ndarray:
    """f16 bits to f32 as moelan/kernels.py:244-255 decodes them (exponent 31
    -> +-inf whatever the payload)."""
    bits = np.asarray(bits, np.uint16)
    v = bits.view(np.float16).astype(np.float32)
    inf = ((bits >> 10) & 0x1F) == 31
    return np.where(inf, np.where(bits & 0x8000, -np.inf, np.inf), v).astype(np.float32)


def q4_k_as_affine(raw: np.ndarray, cols: int):
    """GGUF Q4_K rows (O, cols/256 * 144) -> (nibbles u (O, cols) uint8,
    scales (O, cols/32) f32, biases (O, cols/32) f32) with
    (u - 8) * scale + bias = d*sc*q - dmin*m (moelan/kernels.py:310-336):
    scale = f32(d) * sc, bias = 8 * scale - f32(dmin) * m, u = q."""
    raw = np.ascontiguousarray(raw, np.uint8)
    O, nb = raw.shape[0], cols // 256
    b = raw.reshape(O, nb, 144)
    d = _f16_ref(np.ascontiguousarray(b[:, :, 0:2]).view(np.uint16)[..., 0])
    dmin = _f16_ref(np.ascontiguousarray(b[:, :, 2:4]).view(np.uint16)[..., 0])
    sb = b[:, :, 4:16].astype(np.int32)
    sc = np.empty((O, nb, 8), np.int32)
    mn = np.empty((O, nb, 8), np.int32)
    sc[..., :4], mn[..., :4] = sb[..., 0:4] & 63, sb[..., 4:8] & 63
    sc[..., 4:] = (sb[..., 8:12] & 0xF) | ((sb[..., 0:4] >> 6) << 4)
    mn[..., 4:] = (sb[..., 8:12] >> 4) | ((sb[..., 4:8] >> 6) << 4)
    qs = b[:, :, 16:144].reshape(O, nb, 4, 32)
    u = np.stack([qs & 15, qs >> 4], axis=3).reshape(O, cols)      # chunk c: low -> 64c+i, high -> 64c+32+i
    scale = (d[:, :, None] * sc.astype(np.float32)).astype(np.float32)
    mins = (dmin[:, :, None] * mn.astype(np.float32)).astype(np.float32)
    bias = (np.float32(8.0) * scale - mins).astype(np.float32)
    return u.astype(np.uint8), scale.reshape(O, nb * 8), bias.reshape(O, nb * 8)


def q4k_tiles(raw: np.ndarray, cols: int, gu_inter: int = 0):
    """Tile bytes (FMT_Q4K_F32) of GGUF Q4_K rows; ``gu_inter``: I, for a
    gate|up matrix (2I rows: gate rows then up rows)."""
    u, sc, bias = q4_k_as_affine(raw, cols)
    packed = (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)
    base = q4_tiles(packed, sc, 32, True, gu_inter)
    order = row_order(raw.shape[0], gu_inter)
    Kp = (cols + QUAD_COLS - 1) // QUAD_COLS * QUAD_COLS
    NQ, RT = Kp // QUAD_COLS, len(order) // TILE_ROWS
    Bs = _group_scales(bias, order, cols, 32, np.float32)
    bt = np.ascontiguousarray(Bs.reshape(RT, TILE_ROWS, NQ, 4).transpose(0, 2, 1, 3)).view(np.uint8).reshape(RT, NQ, -1)
    return np.ascontiguousarray(np.concatenate([base.reshape(RT, NQ, -1), bt], axis=2).reshape(-1))


def q4k_weight_bound(raw: np.ndarray, cols: int):
    """(largest possible |weight|, per-row sum of |weight| (float64)) of GGUF Q4_K rows."""
    u, sc, bias = q4_k_as_affine(raw, cols)
    amax = float(np.max(8.0 * np.abs(sc.astype(np.float64)) + np.abs(bias.astype(np.float64)))) if sc.size else 0.0
    w = (u.reshape(u.shape[0], -1, 32).astype(np.float64) - 8.0) * sc[..., None] + bias[..., None]
    return amax, np.abs(w).sum(axis=(1, 2))


def q4_0_as_q4(raw: np.ndarray, cols: int):
    """GGUF Q4_0 rows (O, cols/32 * 18) -> (colibri-order offset nibbles (O,
    cols/2), f16 scales (O, cols/32)).  Q4_0 keeps a block's first 16 values
    in the low nibbles and the last 16 in the high ones (kernels.py:270-278);
    value = d * (nibble - 8), i.e. nibble = u in the offset form."""
    raw = np.ascontiguousarray(raw, np.uint8)
    O = raw.shape[0]
    b = raw.reshape(O, cols // 32, 18)
    d = np.ascontiguousarray(b[:, :, :2]).view(np.float16).reshape(O, cols // 32)
    qs = b[:, :, 2:]
    u = np.concatenate([qs & 15, qs >> 4], axis=2)                 # (O, nb, 32) in column order
    packed = (u[:, :, 0::2] | (u[:, :, 1::2] << 4)).astype(np.uint8)
    return np.ascontiguousarray(packed.reshape(O, cols // 2)), d
