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
    """(kind, payload, scales, gs, offset[, biases]): kind 'q4' (payload:
    colibri int4 bytes), 'q8' (int8 values) or 'q4k' (GGUF Q4_K rows as they
    are: payload the raw blocks, scales the column count), or None when there
    is no packed form."""
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
        if m.qtype == 12:
            return "q4k", np.asarray(m.raw, np.uint8), cols, 32, False
        return None
    if hasattr(m, "parts"):                                                      # gguf.Stacked
        parts = [_as_group_matrix(p) for p in m.parts]
        if any(p is None for p in parts):
            return None
        kinds = {p[0] for p in parts}
        if len(kinds) != 1:
            return None
        if kinds == {"q4k"}:
            if len({p[2] for p in parts}) != 1:
                return None
            return "q4k", np.concatenate([p[1] for p in parts]), parts[0][2], 32, False
        if len({(p[2].dtype, p[3], p[4]) for p in parts}) != 1:
            return None
        k, _, s0, gs, off = parts[0]
        return (k, np.concatenate([p[1] for p in parts]), np.concatenate([p[2] for p in parts]).astype(s0.dtype),
                gs, off)
    return None


def _pack_matrix(mat, inter: int):
    """(fmt, tiles, weight exponent, per-row |w| sums or None) of one matrix;
    ``inter`` > 0 for a gate|up matrix."""
    kind, payload, s, gs, off = mat
    if kind == "q4":
        return (layout.fmt_of("q4", s), layout.q4_tiles(payload, s, gs, off, gu_inter=inter),
                layout.weight_exponent(s, 8), layout.row_l1_q4(payload, s, gs, off) if inter else None)
    if kind == "q8":
        return (layout.fmt_of("q8", s), layout.q8_tiles(payload, s, gs, gu_inter=inter),
                layout.weight_exponent(s, 128), layout.row_l1_q8(payload, s, gs) if inter else None)
    cols = s
    amax, l1 = layout.q4k_weight_bound(payload, cols)
    return layout.FMT_Q4K_F32, layout.q4k_tiles(payload, cols, gu_inter=inter), layout.exponent_for(amax), l1


def pack_expert(expert, inter: int | None = None):
    """A moelan Expert (gu, down[, inter]) as a Packed, or None if a matrix
    has no packed form or the two matrices' group sizes differ.  The two
    matrices may be of different kinds (GGUF experts: Q4_K gate|up, Q8_0 down)."""
    gu, dn = _as_group_matrix(expert.gu), _as_group_matrix(expert.down)
    if gu is None or dn is None or gu[3] != dn[3]:
        return None
    I = int(inter if inter is not None else expert.inter)
    H = dn[1].shape[0]
    try:
        fg, gt, eg, l1 = _pack_matrix(gu, I)
        fd, dt, ed, _ = _pack_matrix(dn, 0)
    except ValueError:          # a group size the tile layout does not take
        return None
    return Packed(fg, fd, gu[3], H, I, gt, dt, (eg, ed, layout.act_exponent(l1, I)))


def _dims(mat):
    """(rows, columns) of a matrix as _as_group_matrix gives it."""
    kind, payload, s = mat[0], mat[1], mat[2]
    if kind == "q4":
        return payload.shape[0], 2 * payload.shape[1]
    if kind == "q8":
        return payload.shape
    return payload.shape[0], int(s)


def _meta(mat, inter: int):
    """(fmt, weight exponent, per-row |w| sums or None) of one matrix, from its
    scales and bytes on the host; ``inter`` > 0 for a gate|up matrix."""
    kind, payload, s, gs, off = mat
    if kind == "q4":
        return (layout.fmt_of("q4", s), layout.weight_exponent(s, 8),
                layout.row_l1_q4(payload, s, gs, off) if inter else None)
    if kind == "q8":
        return (layout.fmt_of("q8", s), layout.weight_exponent(s, 128),
                layout.row_l1_q8(payload, s, gs) if inter else None)
    amax, l1 = layout.q4k_weight_bound(payload, s)
    return layout.FMT_Q4K_F32, layout.exponent_for(amax), l1


def _pack_on(mat, inter: int, out, dev) -> None:
    """Lay one matrix out into the device bytes ``out`` with the library's
    packers (mb_pack_q4 / mb_pack_q8 / mb_pack_q4k), from its bytes as stored."""
    import torch

    from . import device as D
    kind, payload, s, gs, off = mat

    def up(a, dt=None):
        return torch.from_numpy(np.ascontiguousarray(a if dt is None else a.astype(dt, copy=False))).to(dev)

    if kind == "q4":
        D.pack_q4(up(payload, np.uint8), up(s, np.float16 if s.dtype == np.float16 else np.float32), gs, off,
                  inter, out=out)
    elif kind == "q8":
        D.pack_q8(up(payload, np.int8), up(s, np.float16 if s.dtype == np.float16 else np.float32), gs, inter,
                  out=out)
    else:
        D.pack_q4k(up(payload, np.uint8), int(s), inter, out=out)


def pack_expert_on(expert, device, inter: int | None = None, max_bytes: int | None = None):
    """As :func:`pack_expert`, but the tiles are laid out on ``device`` by the
    library's packers from the matrices' bytes as moelan holds them, so only
    those bytes cross to the device and no host re-layout runs.  The Packed's
    ``gu_tiles`` / ``dn_tiles`` are views of one device buffer ``Packed.buf``
    (gate|up tiles, then the down tiles at a 256-byte boundary).  None where
    :func:`pack_expert` gives None, or when the buffer would exceed
    ``max_bytes`` (then nothing is allocated)."""
    import torch
    gu, dn = _as_group_matrix(expert.gu), _as_group_matrix(expert.down)
    if gu is None or dn is None or gu[3] != dn[3]:
        return None
    I = int(inter if inter is not None else expert.inter)
    try:
        (Og, Kg), (Od, Kd) = _dims(gu), _dims(dn)
        for K, gs in ((Kg, gu[3]), (Kd, dn[3])):
            layout._check(K, gs)
        fg, eg, l1 = _meta(gu, I)
        fd, ed, _ = _meta(dn, 0)
    except ValueError:          # a group size the tile layout does not take
        return None
    H = Od
    ng = layout.tiles_nbytes(fg, Og, Kg, gu_inter=I)
    nd = layout.tiles_nbytes(fd, Od, Kd)
    off = (ng + 255) // 256 * 256
    if max_bytes is not None and off + nd > max_bytes:
        return None
    dev = torch.device(device)
    buf = torch.empty(off + nd, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _pack_on(gu, I, buf[:ng], dev)
        _pack_on(dn, 0, buf[off:off + nd], dev)
    p = Packed(fg, fd, gu[3], H, I, buf[:ng], buf[off:off + nd], (eg, ed, layout.act_exponent(l1, I)))
    p.buf, p.dn_offset = buf, off
    return p
