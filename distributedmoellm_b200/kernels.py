"""moelan.kernels' expert entry points on the GPU, same signatures.

Mirrors moelan/kernels.py:930-1032: numpy arrays in, numpy arrays out (the
call copies its inputs to the current CUDA device, runs this library's
kernels and copies the result back), so ``install()`` can put them in place of
the reference's numba kernels behind ExpertStore, Packed4, GroupQuant and
gguf.QuantMatrix unchanged.  Dequantisation is bit-exact; the products match
the reference's f32 path within 1e-5 of each output row's largest magnitude.

Weight matrices are packed into the device tile layout on first use and kept
(keyed by the arrays' addresses, shapes and dtypes, holding a reference so
the address cannot be reused while cached): like the reference's resident
experts (kernels.py:942-947), they must not change while they are in use.

moelan calls these from several host threads at once (its worker's server
threads, the batcher thread, its BLAS pool): the caches are guarded by one
re-entrant lock, which is held across each call's device work and result
copy, so concurrent calls are serialised rather than interleaved.
"""

from __future__ import annotations

import ctypes
import threading
from collections import OrderedDict
from types import SimpleNamespace

import numpy as np
import torch

from . import device as D
from . import layout
from .accel import DevicePool
from .packing import pack_expert_on

_CACHE_MAX = 512
_lock = threading.RLock()                 # guards the caches below and each call's use of them
_mats: OrderedDict = OrderedDict()        # matrix key -> (device tiles or raw blocks, fmt, O, K, kept arrays)
_pool: dict = {}                          # device index -> (DevicePool of moe_q4 experts, their keys in use order)


def _dev():
    D.require_device()
    return torch.device("cuda", torch.cuda.current_device())


def _key(*arrays):
    return tuple((a.__array_interface__["data"][0], a.shape, a.dtype.str, a.strides) for a in arrays)


def _tiles(key, make, keep):
    """The cached device bytes for ``key`` (made by ``make(dev)`` on a miss: (fmt,
    O, K, device tensor)); call with _lock held."""
    dev = _dev()
    key = key + (dev.index,)
    hit = _mats.get(key)
    if hit is not None:
        _mats.move_to_end(key)
        return hit
    fmt, O, K, tiles = make(dev)
    ent = (tiles, fmt, O, K, keep)
    _mats[key] = ent
    while len(_mats) > _CACHE_MAX:
        _mats.popitem(last=False)
    return ent


def _matmul(key, make, keep, x):
    with _lock:
        t, fmt, O, K, _ = _tiles(key, make, keep)
        xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(t.device)
        return D.matmul_t(t, fmt, O, K, xd).cpu().numpy()


# ---- dequantisation (moelan/kernels.py:971-1003) ------------------------------------

def q4_dequant(raw, s, gs: int, offset: bool, out: np.ndarray) -> np.ndarray:
    dev = _dev()
    r = torch.from_numpy(np.ascontiguousarray(raw, np.uint8)).to(dev)
    sc = torch.from_numpy(np.ascontiguousarray(s)).to(dev)
    out[...] = D.q4_dequant(r, sc, gs, offset).cpu().numpy()
    return out


def q8_dequant(q, s, gs: int, out: np.ndarray) -> np.ndarray:
    dev = _dev()
    qq = torch.from_numpy(np.ascontiguousarray(q, np.int8)).to(dev)
    sc = torch.from_numpy(np.ascontiguousarray(s)).to(dev)
    out[...] = D.q8_dequant(qq, sc, gs).cpu().numpy()
    return out


def gguf_dequant(raw: np.ndarray, qtype: int, out: np.ndarray) -> np.ndarray:
    r = torch.from_numpy(np.ascontiguousarray(raw, np.uint8)).to(_dev())
    out[...] = D.gguf_dequant(r, int(qtype), out.shape[1]).cpu().numpy()
    return out


# ---- single matrices: x @ W.T (moelan/kernels.py:981-998, 1018-1032) ----------------
# A matrix's bytes go to the device as moelan holds them; the library's packers
# lay them out there (mb_pack_q4 / mb_pack_q8).

def _up(a, dtype, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype)).to(dev)


def _scales(s):
    """Scales as the packers take them: f16 stays f16, anything else f32."""
    return np.float16 if np.asarray(s).dtype == np.float16 else np.float32


def q4_matmul_t(x: np.ndarray, raw: np.ndarray, s: np.ndarray, gs: int, offset: bool) -> np.ndarray:
    """x @ W.T for colibri int4 bytes; ``offset`` means raw was XOR-ed with 0x88."""
    def make(dev):
        O, K = raw.shape[0], raw.shape[1] * 2
        layout._check(K, gs)
        return (layout.fmt_of("q4", s), O, K,
                D.pack_q4(_up(raw, np.uint8, dev), _up(s, _scales(s), dev), gs, bool(offset)))
    return _matmul(_key(raw, s) + (gs, bool(offset)), make, (raw, s), x)


def q8_matmul_t(x: np.ndarray, q: np.ndarray, s: np.ndarray, gs: int) -> np.ndarray:
    def make(dev):
        layout._check(q.shape[1], gs)
        return (layout.fmt_of("q8", s), q.shape[0], q.shape[1],
                D.pack_q8(_up(q, np.int8, dev), _up(s, _scales(s), dev), gs))
    return _matmul(_key(q, s) + (gs,), make, (q, s), x)


def gguf_matmul_t(x: np.ndarray, raw: np.ndarray, qtype: int, cols: int) -> np.ndarray:
    """x @ W.T for GGUF blocks of any type moelan reads (moelan/kernels.py:981-998):
    Q8_0 and Q4_0 as int8 / int4 tiles with their f16 block scales (the
    tensor-core mat-vec, mb_matmul_t), the other types straight from the
    blocks (mb_gguf_matmul_t)."""
    qtype = int(qtype)
    if qtype in (8, 2):
        if qtype == 8:
            def make(dev):
                q, d = layout.q8_0_as_q8(raw, cols)
                return (layout.FMT_Q8_F16, raw.shape[0], cols,
                        D.pack_q8(_up(q, np.int8, dev), _up(d, np.float16, dev), 32))
        else:
            def make(dev):
                r, d = layout.q4_0_as_q4(raw, cols)
                return (layout.FMT_Q4_F16, raw.shape[0], cols,
                        D.pack_q4(_up(r, np.uint8, dev), _up(d, np.float16, dev), 32, True))
        return _matmul(_key(raw) + (qtype, cols), make, (raw,), x)

    def make_raw(dev):
        return 0, raw.shape[0], cols, _up(raw, np.uint8, dev)
    with _lock:
        t, _, _, _, _ = _tiles(_key(raw) + (qtype, cols, "raw"), make_raw, (raw,))
        xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(t.device)
        return D.gguf_matmul_t(t, qtype, cols, xd).cpu().numpy()


# ---- the fused int4 layer call (moelan/kernels.py:930-968) ------------------------------

def q4_expert_ptrs(e) -> tuple[int, int, int, int, int] | None:
    """What :func:`moe_q4` needs of one int4 expert (addresses of its four
    arrays and the XOR for its nibbles), or None if it does not qualify; the
    same rule as the reference (kernels.py:930-939)."""
    gu, dn = e.gu, e.down
    for m in (gu, dn):
        if not (hasattr(m, "raw") and hasattr(m, "offset") and m.raw.flags.c_contiguous
                and m.s.flags.c_contiguous and m.raw.dtype == np.uint8 and m.s.dtype == np.float32):
            return None
    if gu.gs != dn.gs or gu.offset != dn.offset:
        return None
    addr = lambda a: a.__array_interface__["data"][0]   # noqa: E731
    return addr(gu.raw), addr(gu.s), addr(dn.raw), addr(dn.s), 0 if gu.offset else 0x88


def _from_address(addr: int, n: int, dtype) -> np.ndarray:
    ct = {np.uint8: ctypes.c_uint8, np.float32: ctypes.c_float}[dtype]
    return np.ctypeslib.as_array((ct * n).from_address(addr))


def moe_q4(x: np.ndarray, items, H: int, I: int, gs: int, out: np.ndarray) -> None:
    """Add ``sum_e w * expert_e(x[rows])`` into ``out`` for colibri int4
    experts in one call.  ``items``: (ptrs from :func:`q4_expert_ptrs`, rows,
    gate weights) per expert; the arrays behind the pointers must stay alive
    and unchanged (each expert is uploaded on first use and kept)."""
    with _lock:
        _moe_q4(x, items, H, I, gs, out)


def _moe_q4(x, items, H, I, gs, out):
    dev = _dev()
    if dev.index not in _pool:
        _pool[dev.index] = (DevicePool(dev), OrderedDict())
    pool, order = _pool[dev.index]
    keys = []
    for ptrs, _, _ in items:
        key = (ptrs if type(ptrs) is tuple else tuple(int(p) for p in ptrs), H, I, gs)
        if key not in pool.entries:
            g_raw = _from_address(ptrs[0], 2 * I * H // 2, np.uint8).reshape(2 * I, H // 2)
            g_s = _from_address(ptrs[1], 2 * I * (H // gs), np.float32).reshape(2 * I, H // gs)
            d_raw = _from_address(ptrs[2], H * I // 2, np.uint8).reshape(H, I // 2)
            d_s = _from_address(ptrs[3], H * (I // gs), np.float32).reshape(H, I // gs)
            off = int(ptrs[4]) == 0
            # the expert's bytes as moelan holds them, laid out on the device by the library's packer
            ex = SimpleNamespace(gu=SimpleNamespace(raw=g_raw, s=g_s, gs=gs, offset=off),
                                 down=SimpleNamespace(raw=d_raw, s=d_s, gs=gs, offset=off), inter=I)
            packed = pack_expert_on(ex, dev)
            if packed is None:
                layout._check(H, gs)
                layout._check(I, gs)
                raise ValueError(f"moe_q4: experts with H={H}, I={I}, gs={gs} have no tile layout")
            pool.put(key, packed)
        order[key] = None
        order.move_to_end(key)
        keys.append(key)
    while len(order) > max(_CACHE_MAX, len(keys)):      # never evict an expert this call uses
        pool.pop(order.popitem(last=False)[0])
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(dev)
    uniq, part, status = pool.compute(xd, keys, [r for _, r, _ in items], [w for _, _, w in items])
    res, st = pool.read_back(part, status)
    if st:
        raise RuntimeError(f"moe_q4: the GPU kernels reported status {st}")
    if len(uniq) and uniq[0] == 0 and uniq[-1] == len(uniq) - 1:   # rows 0..U-1 (sorted, unique): a slice
        out[:len(uniq)] += res
    else:
        out[uniq] += res
