"""mb_moe_decode_noalloc: the decode for callers that cannot allocate device
memory (a binding that only forwards the pointers it was given, or code
running where allocation is not allowed).  It must give what mb_moe_decode
gives with a caller workspace, call after call, although its scratch is one
array inside the library that every call reuses.  This file is collected last
so a run that stops at the first failure has run every other test first."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-5   # the f32-path bar of the other parity tests: max|diff| / max|ref| per row


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_decode_matches_workspace_decode_twice():
    from distributedmoellm_b200 import _build
    _build.build()
    from distributedmoellm_b200 import _lib
    from distributedmoellm_b200 import device as D
    from distributedmoellm_b200 import layout as L
    from distributedmoellm_b200 import synthetic as S
    from distributedmoellm_b200.store import LayerExperts
    D.require_device()
    lib = _lib.lib()

    E, H, I, gs, k = 16, 512, 256, 32, 2
    rng = np.random.default_rng(42)
    ex = LayerExperts(E, H, I, gs, L.FMT_Q4_F16, L.FMT_Q4_F16, "cuda")
    for e in range(E):
        ex.put_int4(e, *S.int4_expert(rng, H, I, gs, f16_scales=True))
    ex.publish()
    router = torch.from_numpy(S.router(rng, E, H)).cuda()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    for call, T in enumerate((8, 33)):             # two calls in a row, different sizes and inputs
        x = torch.from_numpy(S.hidden(rng, T, H)).cuda()
        rexp = torch.empty(T, dtype=torch.int32, device="cuda")
        idx, w = D.router_route(x, router, k, True, row_exp=rexp)
        r = D.permute(idx, w, E)
        P = T * k
        want = torch.empty((P, H), dtype=torch.float32, device="cuda")
        ws = torch.empty(D.decode_workspace_bytes(P, I), dtype=torch.uint8, device="cuda")
        D.moe_decode(ex.table, E, H, I, gs, ex.fmt_gu, ex.fmt_down, x, rexp, r, want, ws)
        got = torch.full((P, H), float("nan"), dtype=torch.float32, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        rc = lib.mb_moe_decode_noalloc(_p(ex.table), E, H, I, gs, ex.fmt_gu, ex.fmt_down, _p(x), _p(rexp), T,
                                       _p(r.counts), _p(r.offsets), _p(r.sorted_rows), P, 0, _p(got), _p(status),
                                       stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        g, wnt = got.cpu().numpy().astype(np.float64), want.cpu().numpy().astype(np.float64)
        err = np.abs(g - wnt).max(axis=1) / np.maximum(np.abs(wnt).max(axis=1), 1e-30)
        assert np.isfinite(g).all() and err.max() <= TOL, (call, err.max())


def test_noalloc_decode_rejects_calls_beyond_its_scratch():
    from distributedmoellm_b200 import _build
    _build.build()
    from distributedmoellm_b200 import _lib
    lib = _lib.lib()
    buf = ctypes.create_string_buffer(256)
    p = ctypes.cast(buf, ctypes.c_void_p)
    P, I = 100000, 768                              # far more than MB_NOALLOC_SCRATCH_BYTES holds
    rc = lib.mb_moe_decode_noalloc(p, 8, 2048, I, 32, 2, 2, p, p, P // 8, p, p, p, P, 0, p, None, None)
    assert rc == 1 and "scratch" in _lib.last_error()
