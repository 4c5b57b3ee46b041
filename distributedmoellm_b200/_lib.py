"""ctypes binding of libmoelan_b200.so (the C ABI declared in
include/moelan_b200.h).  There is no fallback: if the library is missing or
the device is not an sm_100 part, calls raise RuntimeError."""

from __future__ import annotations

import ctypes
import threading

from . import _build

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_u8 = ctypes.c_uint8

# name -> (restype, argtypes); the order follows include/moelan_b200.h
SIGNATURES = {
    "mb_last_error": (ctypes.c_char_p, []),
    "mb_version": (_int, []),
    "mb_device_check": (_int, []),
    "mb_tiles_bytes": (_i64, [_int, _int, _int, _int]),
    "mb_pack_q4": (_int, [_vp, _vp, _int, _int, _int, _int, _u8, _int, _vp, _vp]),
    "mb_pack_q8": (_int, [_vp, _vp, _int, _int, _int, _int, _int, _vp, _vp]),
    "mb_pack_q4k": (_int, [_vp, _int, _int, _int, _vp, _vp]),
    "mb_q4_dequant": (_int, [_vp, _vp, _int, _i64, _i64, _int, _u8, _vp, _vp]),
    "mb_q8_dequant": (_int, [_vp, _vp, _int, _i64, _i64, _int, _vp, _vp]),
    "mb_gguf_dequant": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp]),
    "mb_gguf_matmul_t": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _i64, _vp, _vp]),
    "mb_wire_group": (_int, [_int]),
    "mb_encode_rows": (_int, [_vp, _i64, _int, _int, _vp, _vp, _vp]),
    "mb_decode_rows": (_int, [_vp, _vp, _i64, _int, _int, _vp, _vp]),
    "mb_router_workspace_bytes": (_i64, [_i64, _int, _int]),
    "mb_router_logits": (_int, [_vp, _vp, _i64, _int, _int, _vp, _vp, _vp, _i64, _vp]),
    "mb_router_route": (_int, [_vp, _vp, _i64, _int, _int, _int, _int, _vp, _vp, _vp, _vp, _vp, _i64, _vp]),
    "mb_router_topk": (_int, [_vp, _i64, _int, _int, _int, _vp, _vp, _vp]),
    "mb_router_grouped": (_int, [_vp, _vp, _i64, _int, _int, _int, _int, _int, _int, _int, ctypes.c_float, _vp, _vp,
                                 _vp]),
    "mb_router_sparsemixer": (_int, [_vp, _i64, _int, ctypes.c_double, _vp, _vp, _vp]),
    "mb_row_exponents": (_int, [_vp, _i64, _int, _vp, _vp]),
    "mb_permute": (_int, [_vp, _vp, _i64, _int, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "mb_unpermute_combine": (_int, [_vp, _vp, _vp, _vp, _i64, _int, _int, _int, _vp, _vp]),
    "mb_moe_decode_workspace_bytes": (_i64, [_i64, _int]),
    "mb_moe_decode": (_int, [_vp, _int, _int, _int, _int, _int, _int, _vp, _vp, _i64, _vp, _vp, _vp, _i64, _int,
                             _vp, _vp, _i64, _vp, _vp]),
    "mb_moe_decode_noalloc": (_int, [_vp, _int, _int, _int, _int, _int, _int, _vp, _vp, _i64, _vp, _vp, _vp, _i64,
                                     _int, _vp, _vp, _vp]),
    "mb_moe_prefill_workspace_bytes": (_i64, [_i64, _int, _int, _int]),
    "mb_moe_prefill": (_int, [_vp, _vp, _int, _int, _int, _int, _int, _int, _vp, _vp, _i64, _vp, _vp, _vp, _i64,
                              _int, _vp, _vp, _i64, _vp, _vp]),
    "mb_peer_alloc": (_int, [_i64, ctypes.POINTER(_vp), _vp]),
    "mb_peer_open": (_int, [_vp, ctypes.POINTER(_vp)]),
    "mb_peer_close": (_int, [_vp]),
    "mb_peer_free": (_int, [_vp]),
    "mb_ep_dispatch": (_int, [_vp, _vp, _i64, _int, _vp, _vp, _int, _vp, _vp, _int, _int, _int, _vp, _vp, _vp,
                              _i64, _vp, _vp, _vp, _vp]),
    "mb_moe_prefill_rows_workspace_bytes": (_i64, [_i64, _int]),
    "mb_moe_prefill_rows": (_int, [_vp, _vp, _int, _int, _int, _int, _int, _int, _vp, _vp, _vp, _vp, _i64, _int,
                                   _vp, _vp, _vp, _int, _i64, _vp, _i64, _vp, _vp]),
    "mb_matmul_t_workspace_bytes": (_i64, [_i64]),
    "mb_matmul_t": (_int, [_vp, _int, _int, _int, _vp, _i64, _vp, _vp, _i64, _vp, _vp]),
}

_lock = threading.Lock()
_L = None


def lib():
    """The loaded library (built on first use if the build tree is writable)."""
    global _L
    if _L is None:
        with _lock:
            if _L is None:
                path = _build.LIB
                if not path.exists():
                    _build.build()
                L = ctypes.CDLL(str(path))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _L = L
    return _L


def last_error() -> str:
    return (lib().mb_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed (code {rc}): {last_error()}")
