"""Seeded synthetic experts and activations at the benchmark shapes.

The reference times its kernels on random experts of the model's shape
(moelan/experts.py:322-339 synthetic_expert: int4 nibbles uniform in a byte
with scales rand * 1e-3, int8 values uniform in -127..127 with scales
rand * 1e-4) and on random GGUF blocks with pinned f16 scales
(moelan/gguf.py:547-564).  These generators follow the same recipes with
numpy's PCG64, so the CPU baseline and the GPU see identical bytes.
"""

from __future__ import annotations

import numpy as np


def int4_expert(rng: np.random.Generator, H: int, I: int, gs: int, f16_scales: bool = True):
    """(gu_raw (2I, H/2) u8, gu_s (2I, H/gs), dn_raw (H, I/2), dn_s (H, I/gs))."""
    sdt = np.float16 if f16_scales else np.float32

    def mat(o, i):
        raw = np.frombuffer(rng.bytes(o * i // 2), np.uint8).reshape(o, i // 2)
        s = (rng.random((o, i // gs), dtype=np.float32) * 1e-3).astype(sdt)
        return raw, s

    gu_raw, gu_s = mat(2 * I, H)
    dn_raw, dn_s = mat(H, I)
    return gu_raw, gu_s, dn_raw, dn_s


def int8_expert(rng: np.random.Generator, H: int, I: int, gs: int):
    """(gu_q (2I, H) i8, gu_s (2I, H/gs) f32, dn_q (H, I), dn_s (H, I/gs))."""

    def mat(o, i):
        q = rng.integers(-127, 128, (o, i), dtype=np.int8)
        s = rng.random((o, i // gs), dtype=np.float32) * 1e-4
        return q, s

    gq, gs_ = mat(2 * I, H)
    dq, ds = mat(H, I)
    return gq, gs_, dq, ds


def gguf_rows(rng: np.random.Generator, rows: int, cols: int, qtype: int, scale: float = 0.001) -> np.ndarray:
    """Random blocks of a GGUF type with every f16 scale field set to ``scale``."""
    block, size = {8: (32, 34), 12: (256, 144), 2: (32, 18), 14: (256, 210)}[qtype]
    raw = np.frombuffer(rng.bytes(rows * (cols // block) * size), np.uint8).reshape(rows, cols // block, size).copy()
    half = np.frombuffer(np.float16(scale).tobytes(), np.uint8)
    fields = {8: (0,), 12: (0, 2), 2: (0,), 14: (208,)}[qtype]
    for off in fields:
        raw[:, :, off:off + 2] = half
    return raw.reshape(rows, cols // block * size)


def router(rng: np.random.Generator, E: int, H: int, std: float = 0.02) -> np.ndarray:
    return (rng.standard_normal((E, H), dtype=np.float32) * std).astype(np.float32)


def hidden(rng: np.random.Generator, T: int, H: int) -> np.ndarray:
    return rng.standard_normal((T, H), dtype=np.float32)
