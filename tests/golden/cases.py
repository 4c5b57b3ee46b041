"""Seeded inputs for the parity fixtures.

``make_golden.py`` feeds these to the reference (moelan, imported from its
source tree in the build container) and stores the reference's outputs in
``golden.npz``; the tests regenerate the same inputs from the same seeds and
compare.  numpy's PCG64 streams are deterministic, so only outputs (and small
inputs) are stored.
"""

from __future__ import annotations

import numpy as np

GGUF_BLOCK = {2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 10: (256, 84), 11: (256, 110),
              12: (256, 144), 13: (256, 176), 14: (256, 210)}
# offsets of the f16 scale fields of each block type, pinned to a small value
# in "well behaved" random blocks (the role of moelan/gguf.py:543-555)
GGUF_SCALE_FIELDS = {2: (0,), 3: (0, 2), 6: (0,), 7: (0, 2), 8: (0,), 10: (80, 82), 11: (108,), 12: (0, 2),
                     13: (0, 2), 14: (208,)}


def int4_quantize(w: np.ndarray, gs: int):
    """Symmetric int4 per group of ``gs`` inputs (values -8..7, f32 scale =
    group absmax / 7): the scheme of moelan/tiny.py:94-100."""
    O, K = w.shape
    g = w.reshape(O, K // gs, gs)
    s = (np.abs(g).max(2) / 7.0).astype(np.float32)
    s = np.where(s == 0, np.float32(1.0), s).astype(np.float32)
    v = np.clip(np.rint(g / s[:, :, None]), -8, 7).astype(np.int8).reshape(O, K)
    return v, s


def int4_pack(v: np.ndarray) -> np.ndarray:
    """Two's-complement nibbles, low nibble = even column (moelan/tiny.py:103-106)."""
    n = (v & 15).astype(np.uint8)
    return np.ascontiguousarray(n[:, 0::2] | (n[:, 1::2] << 4))


def int8_quantize(w: np.ndarray, gs: int):
    """int8 per group of ``gs``: scale = absmax / 127, rint, clip to +-127
    (moelan/experts.py:133-142)."""
    O, K = w.shape
    g = w.reshape(O, K // gs, gs)
    amax = np.abs(g).max(axis=2)
    s = np.where(amax == 0, 1.0, amax / 127.0).astype(np.float32)
    q = np.clip(np.rint(g / s[:, :, None]), -127, 127).astype(np.int8).reshape(O, K)
    return q, s


def gguf_random_rows(rows: int, cols: int, qtype: int, rng, scale: float = 0.01) -> np.ndarray:
    """Random but well-behaved blocks: random bytes with every f16 scale field
    set to ``scale`` (the role of moelan/gguf.py:547-555)."""
    block, size = GGUF_BLOCK[qtype]
    raw = rng.integers(0, 256, (rows, cols // block, size), dtype=np.uint8)
    half = np.frombuffer(np.float16(scale).tobytes(), np.uint8)
    for off in GGUF_SCALE_FIELDS[qtype]:
        raw[:, :, off:off + 2] = half
    return np.ascontiguousarray(raw.reshape(rows, cols // block * size))


def int4_expert(rng, H: int, I: int, gs: int, std: float = 0.02, f16_scales: bool = False):
    """One int4 SwiGLU expert from N(0, std) weights: gate|up (2I, H) and down
    (H, I), packed (raw, f32 scales)."""
    mats = [(rng.standard_normal((I, H)) * std).astype(np.float32),
            (rng.standard_normal((I, H)) * std).astype(np.float32),
            (rng.standard_normal((H, I)) * std).astype(np.float32)]
    q = [int4_quantize(m, gs) for m in mats]
    if f16_scales:
        q = [(v, s.astype(np.float16).astype(np.float32)) for v, s in q]
    gu_raw = np.concatenate([int4_pack(q[0][0]), int4_pack(q[1][0])], 0)
    gu_s = np.ascontiguousarray(np.concatenate([q[0][1], q[1][1]], 0))
    return gu_raw, gu_s, int4_pack(q[2][0]), np.ascontiguousarray(q[2][1])


def int8_expert(rng, H: int, I: int, gs: int, std: float = 0.02):
    mats = [(rng.standard_normal((2 * I, H)) * std).astype(np.float32),
            (rng.standard_normal((H, I)) * std).astype(np.float32)]
    (q1, s1), (q2, s2) = [int8_quantize(m, gs) for m in mats]
    return q1, s1, q2, s2


# ---- the fixture set -----------------------------------------------------------

ROUTER_CASES = [  # (name, T, E, k, normalize, seed)
    ("r64e128k8", 64, 128, 8, True, 11),
    ("r257e128k8", 257, 128, 8, True, 12),
    ("r33e16k2", 33, 16, 2, True, 13),
    ("r40e8k2", 40, 8, 2, True, 14),
    ("r20e60k6raw", 20, 60, 6, False, 15),
]


def router_logits(T, E, seed):
    rng = np.random.default_rng(seed)
    lg = rng.standard_normal((T, E)).astype(np.float32)
    # plant exact ties (equal logits -> equal probabilities -> lower id first)
    lg[1, 3] = lg[1, 5]
    lg[2, :] = 0.5
    return lg


Q4_DEQ = dict(O=64, K=256, gs=32, seed=21)
Q8_DEQ = dict(O=48, K=256, gs=32, seed=22)
GGUF_ROWS, GGUF_COLS = 5, 512
MATMUL_ROWS = (1, 3, 4, 17)          # the reference's own int4 matmul test rows
GGUF_MM_ROWS = (1, 2, 5)


def q4_deq_inputs():
    rng = np.random.default_rng(Q4_DEQ["seed"])
    raw = rng.integers(0, 256, (Q4_DEQ["O"], Q4_DEQ["K"] // 2), dtype=np.uint8)
    s = rng.random((Q4_DEQ["O"], Q4_DEQ["K"] // Q4_DEQ["gs"]), dtype=np.float32)
    return raw, s


def q8_deq_inputs():
    rng = np.random.default_rng(Q8_DEQ["seed"])
    q = rng.integers(-128, 128, (Q8_DEQ["O"], Q8_DEQ["K"]), dtype=np.int8)
    s = rng.random((Q8_DEQ["O"], Q8_DEQ["K"] // Q8_DEQ["gs"]), dtype=np.float32)
    return q, s


def gguf_deq_inputs(qtype):
    """Random bytes (any value, NaN/inf scales included) as the reference's
    block-decoder test uses (tests/test_gguf.py:25-33)."""
    rng = np.random.default_rng(100 + qtype)
    block, size = GGUF_BLOCK[qtype]
    return rng.integers(0, 256, (GGUF_ROWS, GGUF_COLS // block * size), dtype=np.uint8)


def gguf_mm_inputs(qtype, rows):
    rng = np.random.default_rng(200 + qtype * 10 + rows)
    raw = gguf_random_rows(GGUF_ROWS + 11, GGUF_COLS, qtype, rng)
    x = rng.standard_normal((rows, GGUF_COLS)).astype(np.float32)
    return raw, x


def q4_mm_inputs(rows):
    """The reference's int4 known-answer test (tests/test_moelan.py:245-258)."""
    rng = np.random.default_rng(rows)
    O, I, gs = 96, 128, 32
    v = rng.integers(-8, 8, (O, I))
    s = rng.random((O, I // gs)).astype(np.float32)
    nib = (v & 15).astype(np.uint8)
    raw = np.ascontiguousarray(nib[:, 0::2] | (nib[:, 1::2] << 4))
    W = (v.reshape(O, -1, gs) * s[:, :, None]).reshape(O, I).astype(np.float32)
    x = rng.standard_normal((rows, I)).astype(np.float32)
    return raw, s, W, x


# one MoE layer at the config-1 expert shape (H=256, I=512, 16 experts, top-2)
LAYER = dict(H=256, I=512, E=16, k=2, gs=32, T=32, seed=31)
LAYER_F16 = dict(H=256, I=256, E=8, k=2, gs=32, T=6, seed=32)   # f16 scales widened (config-2 scale type)
LAYER_Q8 = dict(H=256, I=512, E=8, k=2, gs=32, T=40, seed=33)    # int8 experts, big groups -> dequant+BLAS
LAYER_GGUF = dict(H=512, I=768, E=4, k=2, T=9, seed=34)          # Q4_K gate/up, Q8_0 down


def layer_inputs(cfg, kind="int4", f16_scales=False):
    rng = np.random.default_rng(cfg["seed"])
    H, I, E = cfg["H"], cfg["I"], cfg["E"]
    router = rng.standard_normal((E, H)).astype(np.float32)
    experts = {}
    for e in range(E):
        if kind == "int4":
            experts[e] = int4_expert(rng, H, I, cfg["gs"], f16_scales=f16_scales)
        elif kind == "int8":
            experts[e] = int8_expert(rng, H, I, cfg["gs"])
        else:
            experts[e] = (gguf_random_rows(I, H, 12, rng, 0.001), gguf_random_rows(I, H, 12, rng, 0.001),
                          gguf_random_rows(H, I, 8, rng, 0.001))
    x = rng.standard_normal((cfg["T"], H)).astype(np.float32)
    return x, router, experts


# ---- activation rows in the wire formats (moelan/protocol.py:96-123) ---------------

def wire_inputs():
    """Rows for encode_rows / decode_rows: the reference test's own case
    (tests/test_moelan.py:998-1009: N(0, 3) rows with one outlier channel x40),
    a width that is not a multiple of 64 (one scale per row), all-zero rows,
    and a row whose quotients fall exactly halfway (rint rounds half to even)."""
    rng = np.random.default_rng(6)
    a = rng.standard_normal((5, 2048)).astype(np.float32) * 3
    a[:, 7] *= 40
    b = rng.standard_normal((7, 96)).astype(np.float32)
    z = np.zeros((2, 8), np.float32)
    h = np.zeros((1, 64), np.float32)
    h[0, :8] = [127.0, 2.5, 3.5, -0.5, -1.5, 126.5, -126.5, 0.5]
    return {"wide": a, "narrow": b, "zeros": z, "halfway": h}


# ---- the other routers (moelan/model.py:170-223) -----------------------------------

# (name, T, E, k, scoring, method, n_group, topk_group, normalize, scaling, with bias, seed)
GROUPED_CASES = [
    ("v3", 64, 256, 8, "sigmoid", "noaux_tc", 8, 4, True, 2.5, True, 41),
    ("v3flat", 40, 64, 6, "sigmoid", "noaux_tc", 1, 1, True, 1.0, True, 42),
    ("v2lim", 48, 64, 6, "softmax", "group_limited_greedy", 8, 3, False, 16.0, False, 43),
    ("v2greedy", 33, 160, 6, "softmax", "greedy", 1, 1, False, 1.0, False, 44),
    ("k1", 20, 32, 1, "sigmoid", "noaux_tc", 4, 2, True, 2.0, True, 45),
]


def grouped_inputs(T, E, with_bias, seed):
    rng = np.random.default_rng(seed)
    lg = rng.standard_normal((T, E)).astype(np.float32)
    lg[1, 5] = lg[1, 9]                           # an exact tie between experts
    lg[3, :] = 0.25                               # a row of equal logits
    bias = (rng.standard_normal(E) * 0.05).astype(np.float32) if with_bias else None
    return lg, bias


def sparsemixer_inputs():
    """The reference's own case (tests/test_hf_reference.py:59-72): near-ties
    inside the 2 % band, negative maxima and exact zeros; plus a wider one."""
    rng = np.random.default_rng(0)
    base = rng.standard_normal((64, 16)).astype(np.float32)
    base[::3, 1:4] = base[::3, :1] * np.float32(1 - 0.01 * rng.random((22, 3)))
    base[1::4] = -np.abs(base[1::4])
    base[2::5, :5] = 0.0
    wide = np.random.default_rng(1).standard_normal((40, 48)).astype(np.float32)
    return {"hf": base, "wide": wide}
