"""The C ABI library: it builds, loads without a GPU, exports every entry
point include/moelan_b200.h declares, and rejects bad arguments before
touching a device."""

import ctypes
import re
from pathlib import Path

import pytest

from distributedmoellm_b200 import _build, _lib

ROOT = Path(__file__).resolve().parents[1]


def declared():
    text = (ROOT / "include" / "moelan_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def L():
    _build.build()
    return _lib.lib()


def test_every_declared_symbol_is_exported(L):
    names = declared()
    assert len(names) >= 14
    for n in names:
        assert hasattr(L, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_version_and_error_string(L):
    assert L.mb_version() == 1
    assert isinstance(_lib.last_error(), str)


def test_bad_arguments_are_rejected_on_the_host(L):
    assert L.mb_q4_dequant(None, None, 0, 4, 64, 32, 0, None, None) == 1
    assert "null pointer" in _lib.last_error()
    buf = ctypes.create_string_buffer(64)
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert L.mb_q4_dequant(p, p, 0, 4, 60, 32, 0, p, None) == 1        # cols not a multiple of gs
    assert L.mb_router_topk(p, 4, 2000, 2, 1, p, p, None) == 1          # E too large
    assert L.mb_permute(p, p, 70000, 1, 8, p, p, p, p, p, p, p, p, None) == 1
    assert L.mb_moe_decode(p, 8, 256, 512, 16, 2, 2, p, p, 1, p, p, p, 2, 0, p, p, 1 << 20, None, None) == 1
    assert "group size" in _lib.last_error()
    # expert-parallel dispatch and the pre-gathered GEMM: shapes checked before any device work
    assert L.mb_ep_dispatch(p, p, 4, 256, p, p, 2, p, p, 8, 3, 0, p, p, p, 64, p, p, p, None) == 1   # 8 % 3
    assert L.mb_ep_dispatch(p, p, 4, 200, p, p, 2, p, p, 8, 2, 0, p, p, p, 64, p, p, p, None) == 1   # H % 128
    assert L.mb_ep_dispatch(p, p, 4, 256, p, p, 2, p, p, 8, 2, 2, p, p, p, 64, p, p, p, None) == 1   # rank
    assert L.mb_ep_dispatch(p, p, 1 << 23, 256, p, p, 2, p, p, 8, 2, 0, p, p, p, 64, p, p, p, None) == 1
    assert L.mb_moe_prefill_rows(p, p, 8, 256, 256, 32, 2, 2, p, p, p, p, 1 << 24, 1, p, None, None, 0, 0, p,
                                 1 << 30, None, None) == 1
    assert L.mb_moe_prefill_rows(p, p, 8, 256, 256, 32, 2, 2, p, p, p, p, 64, 1, None, p, p, 0, 64, p,
                                 1 << 30, None, None) == 1                                   # no result buffers
    assert L.mb_moe_prefill_rows(p, p, 8, 256, 256, 32, 5, 2, p, p, p, p, 64, 1, p, None, None, 0, 0, p,
                                 1 << 30, None, None) == 3                                   # Q4_K gate|up
    assert L.mb_peer_open(None, None) == 1


def test_workspace_sizes(L):
    assert L.mb_moe_decode_workspace_bytes(512, 768) >= 512 * 768 * 4 + 512 * 4
    assert L.mb_matmul_t_workspace_bytes(17) >= 17 * 4
    assert L.mb_moe_prefill_rows_workspace_bytes(4096, 768) >= 4096 * 768 * 2
