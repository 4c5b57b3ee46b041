"""Device-level entry points: thin wrappers that pass torch CUDA tensors to
the C ABI (libmoelan_b200.so) on the current stream.  Every function raises
RuntimeError when the library reports an error; nothing here computes on the
CPU."""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, lib


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _cuda(*ts):
    for t in ts:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise RuntimeError("expected contiguous CUDA tensors")


_checked_devices: set = set()


def require_device() -> None:
    """Raise unless a CUDA device this library is built for (sm_100) is current."""
    if not torch.cuda.is_available():
        raise RuntimeError("distributedmoellm_b200 needs a CUDA device (sm_100a); none is available")
    dev = torch.cuda.current_device()
    if dev not in _checked_devices:
        check(lib().mb_device_check(), "mb_device_check")
        _checked_devices.add(dev)


# ---- the tile layout, made on the device ----------------------------------------------

def tiles_bytes(fmt: int, O: int, K: int, inter: int = 0) -> int:
    return int(lib().mb_tiles_bytes(int(fmt), O, K, inter))


def pack_q4(raw: torch.Tensor, s: torch.Tensor, gs: int, offset: bool, inter: int = 0, out: torch.Tensor | None = None):
    """Tiles of colibri int4 bytes raw (O, K/2) with scales s (O, K/gs) f16 or f32."""
    _cuda(raw, s, out)
    O, K = raw.shape[0], 2 * raw.shape[1]
    f16 = s.dtype == torch.float16
    n = tiles_bytes(2 if f16 else 1, O, K, inter)
    out = torch.empty(n, dtype=torch.uint8, device=raw.device) if out is None else out
    check(lib().mb_pack_q4(_p(raw), _p(s), int(f16), O, K, gs, 0 if offset else 0x88, inter, _p(out), _stream()),
          "mb_pack_q4")
    return out


def pack_q8(q: torch.Tensor, s: torch.Tensor, gs: int, inter: int = 0, out: torch.Tensor | None = None):
    """Tiles of group-scaled int8 q (O, K) with scales s (O, K/gs) f16 or f32."""
    _cuda(q, s, out)
    O, K = q.shape
    f16 = s.dtype == torch.float16
    n = tiles_bytes(4 if f16 else 3, O, K, inter)
    out = torch.empty(n, dtype=torch.uint8, device=q.device) if out is None else out
    check(lib().mb_pack_q8(_p(q), _p(s), int(f16), O, K, gs, inter, _p(out), _stream()), "mb_pack_q8")
    return out


def pack_q4k(raw: torch.Tensor, K: int, inter: int = 0, out: torch.Tensor | None = None):
    """Affine int4 tiles of GGUF Q4_K rows raw (O, K/256 * 144)."""
    _cuda(raw, out)
    O = raw.shape[0]
    n = tiles_bytes(5, O, K, inter)
    out = torch.empty(n, dtype=torch.uint8, device=raw.device) if out is None else out
    check(lib().mb_pack_q4k(_p(raw), O, K, inter, _p(out), _stream()), "mb_pack_q4k")
    return out


# ---- dequantisation ----------------------------------------------------------------

def q4_dequant(raw: torch.Tensor, s: torch.Tensor, gs: int, offset: bool, out: torch.Tensor | None = None):
    _cuda(raw, s)
    O, C = raw.shape
    out = torch.empty((O, 2 * C), dtype=torch.float32, device=raw.device) if out is None else out
    check(lib().mb_q4_dequant(_p(raw), _p(s), int(s.dtype == torch.float16), O, 2 * C, gs,
                              0 if offset else 0x88, _p(out), _stream()), "mb_q4_dequant")
    return out


def q8_dequant(q: torch.Tensor, s: torch.Tensor, gs: int, out: torch.Tensor | None = None):
    _cuda(q, s)
    O, K = q.shape
    out = torch.empty((O, K), dtype=torch.float32, device=q.device) if out is None else out
    check(lib().mb_q8_dequant(_p(q), _p(s), int(s.dtype == torch.float16), O, K, gs, _p(out), _stream()),
          "mb_q8_dequant")
    return out


def gguf_dequant(raw: torch.Tensor, qtype: int, cols: int, out: torch.Tensor | None = None):
    _cuda(raw)
    out = torch.empty((raw.shape[0], cols), dtype=torch.float32, device=raw.device) if out is None else out
    check(lib().mb_gguf_dequant(_p(raw), int(qtype), raw.shape[0], raw.shape[1], cols, _p(out), _stream()),
          "mb_gguf_dequant")
    return out


def gguf_matmul_t(raw: torch.Tensor, qtype: int, cols: int, x: torch.Tensor, y: torch.Tensor | None = None):
    """x @ W.T straight from the GGUF blocks of W (rows, row_bytes)."""
    _cuda(raw, x, y)
    n = x.shape[0]
    y = torch.empty((n, raw.shape[0]), dtype=torch.float32, device=x.device) if y is None else y
    check(lib().mb_gguf_matmul_t(_p(raw), int(qtype), raw.shape[0], raw.shape[1], cols, _p(x), n, _p(y),
                                 _stream()), "mb_gguf_matmul_t")
    return y


# ---- activation rows in the wire formats (moelan/protocol.py:96-123) -------------------

WIRE = {"f16": 1, "int8": 2}


def encode_rows(a: torch.Tensor, wire: str):
    """(q, scales) of f32 rows a (n, d) in wire format "f16" or "int8"
    (scales None for f16); "f32" returns a itself."""
    _cuda(a)
    if wire == "f32":
        return a, None
    n, d = a.shape
    if wire == "f16":
        q = torch.empty((n, d), dtype=torch.float16, device=a.device)
        sc = None
    else:
        q = torch.empty((n, d), dtype=torch.int8, device=a.device)
        sc = torch.empty((n, d // int(lib().mb_wire_group(d))), dtype=torch.float32, device=a.device)
    check(lib().mb_encode_rows(_p(a), n, d, WIRE[wire], _p(q), _p(sc), _stream()), "mb_encode_rows")
    return q, sc


def decode_rows(q: torch.Tensor, scales: torch.Tensor | None = None, out: torch.Tensor | None = None):
    """f32 rows from f16 rows, or from int8 rows and their scales."""
    _cuda(q, scales, out)
    if q.dtype == torch.float32:
        return q
    n, d = q.shape
    wire = WIRE["f16"] if q.dtype == torch.float16 else WIRE["int8"]
    out = torch.empty((n, d), dtype=torch.float32, device=q.device) if out is None else out
    check(lib().mb_decode_rows(_p(q), _p(scales), n, d, wire, _p(out), _stream()), "mb_decode_rows")
    return out


# ---- router -------------------------------------------------------------------------

def router_workspace_bytes(T: int, H: int, E: int) -> int:
    return int(lib().mb_router_workspace_bytes(T, H, E))


def _router_ws(T, H, E, ws, device):
    need = router_workspace_bytes(T, H, E)
    if ws is None:
        ws = torch.empty(need, dtype=torch.uint8, device=device)
    return ws


def router_logits(x: torch.Tensor, router: torch.Tensor, logits=None, row_exp=None, workspace=None):
    _cuda(x, router)
    T, H = x.shape
    E = router.shape[0]
    logits = torch.empty((T, E), dtype=torch.float32, device=x.device) if logits is None else logits
    ws = _router_ws(T, H, E, workspace, x.device)
    check(lib().mb_router_logits(_p(x), _p(router), T, H, E, _p(logits), _p(row_exp), _p(ws), ws.numel(),
                                 _stream()), "mb_router_logits")
    return logits


def router_route(x: torch.Tensor, router: torch.Tensor, k: int, normalize: bool, idx=None, w=None, logits=None,
                 row_exp=None, workspace=None):
    """Logits + top-k in two launches; returns (idx, w)."""
    _cuda(x, router)
    T, H = x.shape
    E = router.shape[0]
    idx = torch.empty((T, k), dtype=torch.int32, device=x.device) if idx is None else idx
    w = torch.empty((T, k), dtype=torch.float32, device=x.device) if w is None else w
    ws = _router_ws(T, H, E, workspace, x.device)
    check(lib().mb_router_route(_p(x), _p(router), T, H, E, k, int(bool(normalize)), _p(logits), _p(row_exp),
                                _p(idx), _p(w), _p(ws), ws.numel(), _stream()), "mb_router_route")
    return idx, w


def row_exponents(x: torch.Tensor, out=None):
    _cuda(x)
    out = torch.empty(x.shape[0], dtype=torch.int32, device=x.device) if out is None else out
    check(lib().mb_row_exponents(_p(x), x.shape[0], x.shape[1], _p(out), _stream()), "mb_row_exponents")
    return out


def router_topk(logits: torch.Tensor, k: int, normalize: bool, idx=None, w=None):
    _cuda(logits)
    T, E = logits.shape
    idx = torch.empty((T, k), dtype=torch.int32, device=logits.device) if idx is None else idx
    w = torch.empty((T, k), dtype=torch.float32, device=logits.device) if w is None else w
    check(lib().mb_router_topk(_p(logits), T, E, k, int(bool(normalize)), _p(idx), _p(w), _stream()),
          "mb_router_topk")
    return idx, w


GROUPED_METHODS = {"greedy": 0, "group_limited_greedy": 1, "noaux_tc": 2}


def router_grouped(logits: torch.Tensor, k: int, scoring: str = "softmax", method: str = "greedy", n_group: int = 1,
                   topk_group: int = 1, normalize: bool = True, scaling: float = 1.0, bias: torch.Tensor | None = None,
                   idx=None, w=None):
    """DeepSeek V2 / V3 routing (moelan/model.py:170-201); returns (idx, w)."""
    _cuda(logits, bias)
    T, E = logits.shape
    idx = torch.empty((T, k), dtype=torch.int32, device=logits.device) if idx is None else idx
    w = torch.empty((T, k), dtype=torch.float32, device=logits.device) if w is None else w
    check(lib().mb_router_grouped(_p(logits), _p(bias), T, E, k, int(scoring == "sigmoid"), GROUPED_METHODS[method],
                                  int(n_group), int(topk_group), int(bool(normalize)), float(scaling), _p(idx), _p(w),
                                  _stream()), "mb_router_grouped")
    return idx, w


def router_sparsemixer(logits: torch.Tensor, eps: float, idx=None, w=None):
    """PhiMoE's top-2 (moelan/model.py:204-223); returns (idx, w)."""
    _cuda(logits)
    T, E = logits.shape
    idx = torch.empty((T, 2), dtype=torch.int32, device=logits.device) if idx is None else idx
    w = torch.empty((T, 2), dtype=torch.float32, device=logits.device) if w is None else w
    check(lib().mb_router_sparsemixer(_p(logits), T, E, float(eps), _p(idx), _p(w), _stream()),
          "mb_router_sparsemixer")
    return idx, w


class Routing:
    """Device buffers of one permutation of T*k picks over E experts."""

    def __init__(self, T: int, k: int, E: int, device):
        P = T * k
        i32 = dict(dtype=torch.int32, device=device)
        self.T, self.k, self.E, self.P = T, k, E, P
        self.counts = torch.empty(E, **i32)
        self.offsets = torch.empty(E + 1, **i32)
        self.sorted_rows = torch.empty(max(P, 1), **i32)
        self.sorted_w = torch.empty(max(P, 1), dtype=torch.float32, device=device)
        self.inv = torch.empty(max(P, 1), **i32)
        self.uexperts = torch.empty(E, **i32)
        self.uoffsets = torch.empty(E + 1, **i32)
        self.n_unique = torch.empty(1, **i32)

    @classmethod
    def from_plan(cls, counts: torch.Tensor, offsets: torch.Tensor, sorted_rows: torch.Tensor) -> "Routing":
        """A grouping made elsewhere (expert parallelism: rows received from
        other ranks): per-expert counts (E,), offsets (E+1,) and the row of
        each grouped pick (P,), all int32 on the device."""
        r = cls.__new__(cls)
        r.E, r.P, r.T, r.k = counts.numel(), sorted_rows.numel(), sorted_rows.numel(), 1
        r.counts, r.offsets, r.sorted_rows = counts.contiguous(), offsets.contiguous(), sorted_rows.contiguous()
        r.sorted_w = r.inv = r.uexperts = r.uoffsets = r.n_unique = None
        return r


def permute(idx: torch.Tensor, w: torch.Tensor | None, E: int, r: Routing | None = None) -> Routing:
    _cuda(idx, w)
    T, k = idx.shape
    r = Routing(T, k, E, idx.device) if r is None else r
    check(lib().mb_permute(_p(idx), _p(w), T, k, E, _p(r.counts), _p(r.offsets), _p(r.sorted_rows),
                           _p(r.sorted_w), _p(r.inv), _p(r.uexperts), _p(r.uoffsets), _p(r.n_unique),
                           _stream()), "mb_permute")
    return r


def combine(y: torch.Tensor, pair_idx: torch.Tensor, pair_w: torch.Tensor, T: int, k: int,
            out: torch.Tensor | None = None, accumulate: bool = False, row_ptr: torch.Tensor | None = None):
    """out[r] (+)= sum of pair_w[i] * y[pair_idx[i]] over row r's entries."""
    _cuda(y, pair_idx, pair_w, row_ptr)
    H = y.shape[1]
    out = torch.empty((T, H), dtype=torch.float32, device=y.device) if out is None else out
    check(lib().mb_unpermute_combine(_p(y), _p(row_ptr), _p(pair_idx), _p(pair_w), T, k, H, int(accumulate),
                                     _p(out), _stream()), "mb_unpermute_combine")
    return out


# ---- fused decode -------------------------------------------------------------------

def decode_workspace_bytes(P: int, I: int) -> int:
    return int(lib().mb_moe_decode_workspace_bytes(P, I))


def moe_decode(table: torch.Tensor, E: int, H: int, I: int, gs: int, fmt_gu: int, fmt_down: int, x: torch.Tensor,
               row_exp: torch.Tensor, r: Routing, y: torch.Tensor, workspace: torch.Tensor, max_rows: int = 0,
               status: torch.Tensor | None = None):
    _cuda(table, x, row_exp, y, workspace, status)
    check(lib().mb_moe_decode(_p(table), E, H, I, gs, fmt_gu, fmt_down, _p(x), _p(row_exp), x.shape[0],
                              _p(r.counts), _p(r.offsets), _p(r.sorted_rows), r.P, int(max_rows), _p(y),
                              _p(workspace), workspace.numel() * workspace.element_size(), _p(status), _stream()),
          "mb_moe_decode")
    return y


def prefill_workspace_bytes(P: int, H: int, I: int, fmt_gu: int = 0) -> int:
    return int(lib().mb_moe_prefill_workspace_bytes(P, H, I, int(fmt_gu)))


def moe_prefill(table: torch.Tensor, e_exp: torch.Tensor, E: int, H: int, I: int, gs: int, fmt_gu: int,
                fmt_down: int, x: torch.Tensor, row_exp: torch.Tensor, r: Routing, y: torch.Tensor,
                workspace: torch.Tensor, min_rows: int = 1, status: torch.Tensor | None = None):
    """Experts with at least ``min_rows`` picks as grouped GEMMs (f16 tensor cores, f32 accumulation)."""
    _cuda(table, e_exp, x, row_exp, y, workspace, status)
    check(lib().mb_moe_prefill(_p(table), _p(e_exp), E, H, I, gs, fmt_gu, fmt_down, _p(x), _p(row_exp), x.shape[0],
                               _p(r.counts), _p(r.offsets), _p(r.sorted_rows), r.P, int(min_rows), _p(y),
                               _p(workspace), workspace.numel() * workspace.element_size(), _p(status), _stream()),
          "mb_moe_prefill")
    return y


def matmul_t(w_tiles: torch.Tensor, fmt: int, O: int, K: int, x: torch.Tensor, y: torch.Tensor | None = None,
             workspace: torch.Tensor | None = None, status: torch.Tensor | None = None):
    """x @ W.T for one matrix in the tile layout."""
    _cuda(w_tiles, x, y, workspace, status)
    n = x.shape[0]
    y = torch.empty((n, O), dtype=torch.float32, device=x.device) if y is None else y
    if workspace is None:
        workspace = torch.empty(int(lib().mb_matmul_t_workspace_bytes(n)), dtype=torch.uint8, device=x.device)
    check(lib().mb_matmul_t(_p(w_tiles), fmt, O, K, _p(x), n, _p(y), _p(workspace), workspace.numel(), _p(status),
                            _stream()), "mb_matmul_t")
    return y


__all__ = [n for n in dir() if not n.startswith("_")] + ["_lib"]


# ---- expert parallelism through peer memory ---------------------------------------------

PEER_HANDLE_BYTES = 64


def peer_alloc(nbytes: int) -> tuple[int, bytes]:
    """nbytes of device memory on the current device that other processes of
    the node can map: (address, handle for peer_open)."""
    ptr = ctypes.c_void_p()
    h = ctypes.create_string_buffer(PEER_HANDLE_BYTES)
    check(lib().mb_peer_alloc(int(nbytes), ctypes.byref(ptr), h), "mb_peer_alloc")
    return int(ptr.value), h.raw


def peer_open(handle: bytes) -> int:
    """This process's address of another process's peer_alloc memory."""
    if len(handle) != PEER_HANDLE_BYTES:
        raise ValueError(f"a peer handle has {PEER_HANDLE_BYTES} bytes, got {len(handle)}")
    ptr = ctypes.c_void_p()
    check(lib().mb_peer_open(ctypes.c_char_p(bytes(handle)), ctypes.byref(ptr)), "mb_peer_open")
    return int(ptr.value)


def peer_close(ptr: int) -> None:
    check(lib().mb_peer_close(ctypes.c_void_p(ptr)), "mb_peer_close")


def peer_free(ptr: int) -> None:
    check(lib().mb_peer_free(ctypes.c_void_p(ptr)), "mb_peer_free")


def ep_dispatch(x: torch.Tensor, row_exp: torch.Tensor, idx: torch.Tensor, r: Routing, counts_all: torch.Tensor,
                rank: int, recv_rows: torch.Tensor, recv_exp: torch.Tensor, recv_ret: torch.Tensor, cap: int,
                local_counts: torch.Tensor, local_offsets: torch.Tensor, status: torch.Tensor):
    """This rank's picks (idx (T, k), permuted into ``r``) stored into their
    experts' ranks' receive rows; recv_*: int64 device tensors of G
    addresses; counts_all (G, E) every rank's counts."""
    _cuda(x, row_exp, idx, counts_all, recv_rows, recv_exp, recv_ret, local_counts, local_offsets, status)
    T, k = idx.shape
    G, E = counts_all.shape
    check(lib().mb_ep_dispatch(_p(x), _p(row_exp), T, x.shape[1], _p(idx), _p(r.inv), k, _p(r.offsets),
                               _p(counts_all), E, G, int(rank), _p(recv_rows), _p(recv_exp), _p(recv_ret), int(cap),
                               _p(local_counts), _p(local_offsets), _p(status), _stream()), "mb_ep_dispatch")


def prefill_rows_workspace_bytes(P: int, I: int) -> int:
    return int(lib().mb_moe_prefill_rows_workspace_bytes(P, I))


def moe_prefill_rows(experts, xp: int, row_exp: int, counts: torch.Tensor, offsets: torch.Tensor, P: int,
                     workspace: torch.Tensor, y: torch.Tensor | None = None, y_ret: int | None = None,
                     y_peers: torch.Tensor | None = None, peer_rows: int = 0, status: torch.Tensor | None = None,
                     min_rows: int = 1):
    """The grouped GEMMs of ``experts`` (a LayerExperts) over P f16 operand
    rows at address ``xp`` (exponents at ``row_exp``), grouped by counts /
    offsets; output rows into y, or to the return addresses at ``y_ret``
    over the row buffers (``peer_rows`` rows each) listed in ``y_peers``
    (int64 device tensor)."""
    ex = experts
    _cuda(counts, offsets, workspace, y, y_peers, status)
    n_peers = 0 if y_peers is None else y_peers.numel()
    check(lib().mb_moe_prefill_rows(_p(ex.table), _p(ex.eexp), ex.E, ex.H, ex.I, ex.gs, ex.fmt_gu, ex.fmt_down,
                                    ctypes.c_void_p(xp), ctypes.c_void_p(row_exp), _p(counts), _p(offsets), int(P),
                                    int(min_rows), _p(y), None if y_ret is None else ctypes.c_void_p(y_ret),
                                    _p(y_peers), n_peers, int(peer_rows), _p(workspace),
                                    workspace.numel() * workspace.element_size(), _p(status), _stream()),
          "mb_moe_prefill_rows")
