"""moelan expert and matrix objects -> the device tile layout.

Accepts the reference's resident formats by their attributes (no import of
moelan is needed): ``Packed4`` (raw, s, gs, offset; moelan/experts.py:170-236),
``GroupQuant`` (q, s, gs; experts.py:125-167), ``gguf.QuantMatrix`` (raw,
qtype, shape; moelan/gguf.py:276-314) in Q8_0 or Q4_0, and ``gguf.Stacked``
(parts: gate, up; gguf.py:317-333) of those.  Dense formats (F32Matrix,
16-bit) have no packed form here: ``pack_expert`` returns None for them.
"""

from __future__ import annotations

import numpy as np

from . import layout


class Packed:
    """One expert in the tile layout: gate|up and down tiles plus the
    exponents of the tensor-core path."""

    def __init__(self, fmt_gu, fmt_down, gs, H, I, gu_tiles, dn_tiles, eexp):
        self.fmt_gu, self.fmt_down, self.gs, self.H, self.I = fmt_gu, fmt_down, gs, H, I
        self.gu_tiles, self.dn_tiles, self.eexp = gu_tiles, dn_tiles, eexp

    @property
    def signature(self):
        return (self.fmt_gu, self.fmt_down, self.gs, self.H, self.I)

    @property
    def nbytes(self):
        return self.gu_tiles.nbytes + self.dn_tiles.nbytes


def _as_group_matrix(m):
    """(kind, payload, scales, gs, offset): kind 'q4' (payload: colibri int4
    bytes) or 'q8' (payload: int8 values), or None when there is no packed form."""
    if hasattr(m, "raw") and hasattr(m, "s") and hasattr(m, "offset"):           # Packed4
        return "q4", np.asarray(m.raw, np.uint8), np.asarray(m.s), int(m.gs), bool(m.offset)
    if hasattr(m, "q") and hasattr(m, "s"):                                      # GroupQuant
        return "q8", np.asarray(m.q, np.int8), np.asarray(m.s), int(m.gs), False
    if hasattr(m, "raw") and hasattr(m, "qtype"):                                # gguf.QuantMatrix
        cols = int(m.shape[1])
        if m.qtype == 8:
            q, d = layout.q8_0_as_q8(m.raw, cols)
            return "q8", q, d, 32, False
        if m.qtype == 2:
            raw, d = layout.q4_0_as_q4(m.raw, cols)
            return "q4", raw, d, 32, True
        return None
    if hasattr(m, "parts"):                                                      # gguf.Stacked
        parts = [_as_group_matrix(p) for p in m.parts]
        if any(p is None for p in parts) or len({(p[0], p[2].dtype, p[3], p[4]) for p in parts}) != 1:
            return None
        k, _, s0, gs, off = parts[0]
        return (k, np.concatenate([p[1] for p in parts]), np.concatenate([p[2] for p in parts]).astype(s0.dtype),
                gs, off)
    return None


def pack_expert(expert, inter: int | None = None):
    """A moelan Expert (gu, down[, inter]) as a Packed, or None if a matrix
    has no packed form or the two matrices differ in kind / group size."""
    gu, dn = _as_group_matrix(expert.gu), _as_group_matrix(expert.down)
    if gu is None or dn is None or gu[0] != dn[0] or gu[3] != dn[3]:
        return None
    kind, gs = gu[0], gu[3]
    I = int(inter if inter is not None else expert.inter)
    H = dn[1].shape[0]
    try:
        if kind == "q4":
            if gu[4] != dn[4]:
                return None
            gt = layout.q4_tiles(gu[1], gu[2], gs, gu[4], gu_inter=I)
            dt = layout.q4_tiles(dn[1], dn[2], gs, dn[4])
            ex = (layout.weight_exponent(gu[2], 8), layout.weight_exponent(dn[2], 8),
                  layout.act_exponent(layout.row_l1_q4(gu[1], gu[2], gs, gu[4]), I))
        else:
            gt = layout.q8_tiles(gu[1], gu[2], gs, gu_inter=I)
            dt = layout.q8_tiles(dn[1], dn[2], gs)
            ex = (layout.weight_exponent(gu[2], 128), layout.weight_exponent(dn[2], 128),
                  layout.act_exponent(layout.row_l1_q8(gu[1], gu[2], gs), I))
    except ValueError:          # a group size the tile layout does not take
        return None
    return Packed(layout.fmt_of(kind, gu[2]), layout.fmt_of(kind, dn[2]), gs, H, I, gt, dt, ex)
