"""Experts resident on one GPU, packed, in the device tile layout.

The reference keeps experts in host RAM in their packed formats
(moelan/experts.py:538-795, ExpertStore) and its GPU tier keeps a dequantised
fp16 copy (moelan/accel.py:75-109).  Here a layer's experts stay packed on
the device (2.65 MB per int4-g32-f16 Qwen3-30B expert instead of 9.4 MB of
fp16), one slot each in a single buffer, with a table of their addresses
(MbExpert entries) that the kernels index by expert id.
"""

from __future__ import annotations

import numpy as np
import torch

from . import layout

ALIGN = 256


def _up(a, dev) -> torch.Tensor:
    """A host array (or tensor) as a contiguous tensor on dev."""
    t = a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a))
    return t.to(dev).contiguous()


def _al(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


class LayerExperts:
    """One MoE layer's experts on a device.  ``ids``: the expert ids this
    device holds (all E by default; a slice under expert parallelism)."""

    def __init__(self, E: int, H: int, I: int, gs: int, fmt_gu: int, fmt_down: int, device, ids=None):
        self.E, self.H, self.I, self.gs = E, H, I, gs
        self.fmt_gu, self.fmt_down = fmt_gu, fmt_down
        self.device = torch.device(device)
        self.ids = list(range(E)) if ids is None else [int(i) for i in ids]
        self.gu_nbytes = layout.tiles_nbytes(fmt_gu, 2 * I, H, gu_inter=I)
        self.dn_nbytes = layout.tiles_nbytes(fmt_down, H, I)
        self.slot_bytes = _al(self.gu_nbytes) + _al(self.dn_nbytes)
        self.slot_of = {e: i for i, e in enumerate(self.ids)}
        self.buf = torch.zeros(max(1, len(self.ids)) * self.slot_bytes, dtype=torch.uint8, device=self.device)
        self._table_host = np.zeros((E, 2), np.int64)
        self.table = torch.zeros((E, 2), dtype=torch.int64, device=self.device)
        # per expert, the power-of-two exponents of the tensor-core path: the
        # gate|up and down weight exponents (layout.weight_exponent) and the
        # activation exponent base (layout.act_exponent); experts stored from
        # raw tiles without them keep the layer on the decode kernels
        self._eexp_host = np.zeros((E, 4), np.int32)
        self.eexp = torch.zeros((E, 4), dtype=torch.int32, device=self.device)
        self.missing_exp: set[int] = set()
        self.present: set[int] = set()

    # ---- placement
    def _slot(self, e: int):
        i = self.slot_of[e]
        base = i * self.slot_bytes
        return base, base + _al(self.gu_nbytes)

    def put_tiles(self, e: int, gu_tiles, dn_tiles, eexp=None) -> None:
        """Store expert ``e`` from tile bytes (numpy on the host, or uint8 tensors).
        ``eexp``: (gate|up weight exponent, down weight exponent, activation
        exponent base), needed by the tensor-core path."""
        if e not in self.slot_of:
            raise KeyError(f"expert {e} is not placed on this device")
        g0, d0 = self._slot(e)
        for off, t, n in ((g0, gu_tiles, self.gu_nbytes), (d0, dn_tiles, self.dn_nbytes)):
            src = torch.as_tensor(t) if isinstance(t, np.ndarray) else t
            if src.numel() != n:
                raise ValueError(f"tile bytes {src.numel()} != expected {n}")
            self.buf[off:off + n].copy_(src.reshape(-1), non_blocking=False)
        self._place(e, eexp)

    def _place(self, e: int, eexp) -> None:
        """Record expert e's slot addresses and exponents after its tiles are written."""
        g0, d0 = self._slot(e)
        base = self.buf.data_ptr()
        self._table_host[e] = (base + g0, base + d0)
        if eexp is None:
            self._eexp_host[e] = 0
            self.missing_exp.add(e)
        else:
            self._eexp_host[e, :3] = eexp
            self.missing_exp.discard(e)
        self.present.add(e)

    def _check_fmt(self, kind: str, s_gu, s_dn) -> None:
        if layout.fmt_of(kind, s_gu) != self.fmt_gu or layout.fmt_of(kind, s_dn) != self.fmt_down:
            raise ValueError(f"{kind} expert with {np.asarray(s_gu).dtype} / {np.asarray(s_dn).dtype} scales does "
                             f"not match this layer's formats {self.fmt_gu} / {self.fmt_down}")

    def put_int4(self, e: int, gu_raw, gu_s, dn_raw, dn_s, offset: bool = False) -> None:
        """Expert ``e`` from colibri int4 arrays (moelan Packed4: raw, s), laid
        out into its slot on the device (mb_pack_q4) from the bytes as they are."""
        from . import device as D
        if e not in self.slot_of:
            raise KeyError(f"expert {e} is not placed on this device")
        self._check_fmt("q4", gu_s, dn_s)
        g0, d0 = self._slot(e)
        dev = self.device
        with torch.cuda.device(dev):
            D.pack_q4(_up(gu_raw, dev), _up(gu_s, dev), self.gs, offset, self.I, out=self.buf[g0:g0 + self.gu_nbytes])
            D.pack_q4(_up(dn_raw, dev), _up(dn_s, dev), self.gs, offset, 0, out=self.buf[d0:d0 + self.dn_nbytes])
        self._place(e, (layout.weight_exponent(gu_s, 8), layout.weight_exponent(dn_s, 8),
                        layout.act_exponent(layout.row_l1_q4(gu_raw, gu_s, self.gs, offset), self.I)))

    def put_int8(self, e: int, gu_q, gu_s, dn_q, dn_s) -> None:
        """Expert ``e`` from group-scaled int8 arrays (moelan GroupQuant: q, s),
        laid out into its slot on the device (mb_pack_q8)."""
        from . import device as D
        if e not in self.slot_of:
            raise KeyError(f"expert {e} is not placed on this device")
        self._check_fmt("q8", gu_s, dn_s)
        g0, d0 = self._slot(e)
        dev = self.device
        with torch.cuda.device(dev):
            D.pack_q8(_up(gu_q, dev), _up(gu_s, dev), self.gs, self.I, out=self.buf[g0:g0 + self.gu_nbytes])
            D.pack_q8(_up(dn_q, dev), _up(dn_s, dev), self.gs, 0, out=self.buf[d0:d0 + self.dn_nbytes])
        self._place(e, (layout.weight_exponent(gu_s, 128), layout.weight_exponent(dn_s, 128),
                        layout.act_exponent(layout.row_l1_q8(gu_q, gu_s, self.gs), self.I)))

    def put_expert(self, e: int, expert) -> None:
        """Expert ``e`` from a moelan Expert object (any format packing.py
        takes: Packed4, GroupQuant, GGUF Q8_0 / Q4_0 / Q4_K and Stacked)."""
        from .packing import pack_expert
        p = pack_expert(expert, self.I)
        if p is None:
            raise ValueError(f"expert {e} has no packed form")
        if (p.fmt_gu, p.fmt_down, p.H, p.I) != (self.fmt_gu, self.fmt_down, self.H, self.I) or p.gs % 32:
            raise ValueError(f"expert {e} is {(p.fmt_gu, p.fmt_down, p.H, p.I)}, this layer "
                             f"{(self.fmt_gu, self.fmt_down, self.H, self.I)}")
        self.put_tiles(e, p.gu_tiles, p.dn_tiles, p.eexp)

    def publish(self) -> None:
        """Upload the address table after a batch of puts."""
        self.table.copy_(torch.from_numpy(self._table_host))
        self.eexp.copy_(torch.from_numpy(self._eexp_host))

    @property
    def nbytes(self) -> int:
        return self.buf.numel()
