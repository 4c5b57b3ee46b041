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


def _layer(kind, E, H, I, gs, rng):
    from distributedmoellm_b200 import layout as L
    from distributedmoellm_b200 import synthetic as S
    from distributedmoellm_b200.store import LayerExperts
    if kind == "q4":
        ex = LayerExperts(E, H, I, gs, L.FMT_Q4_F16, L.FMT_Q4_F16, "cuda")
        parts = [S.int4_expert(rng, H, I, gs, f16_scales=True) for _ in range(E)]
        desc = {e: (("q4", g, gs_.astype(np.float32), gs, False), ("q4", d, ds.astype(np.float32), gs, False))
                for e, (g, gs_, d, ds) in enumerate(parts)}
        for e, pt in enumerate(parts):
            ex.put_int4(e, *pt)
    else:
        ex = LayerExperts(E, H, I, gs, L.FMT_Q8_F32, L.FMT_Q8_F32, "cuda")
        parts = [S.int8_expert(rng, H, I, gs) for _ in range(E)]
        desc = {e: (("q8", g, gs_, gs), ("q8", d, ds, gs)) for e, (g, gs_, d, ds) in enumerate(parts)}
        for e, pt in enumerate(parts):
            ex.put_int8(e, *pt)
    ex.publish()
    return ex, desc


def _row_err(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return (np.abs(got - want).max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)).max()


def test_noalloc_decode_matches_workspace_decode_call_after_call():
    from distributedmoellm_b200 import _build
    _build.build()
    import oracle as O
    from distributedmoellm_b200 import _lib
    from distributedmoellm_b200 import device as D
    from distributedmoellm_b200 import synthetic as S
    D.require_device()
    lib = _lib.lib()

    E, H, gs, k = 16, 512, 32, 2
    rng = np.random.default_rng(42)
    layers = {"q4": _layer("q4", E, H, 256, gs, rng), "q8": _layer("q8", E, H, 128, gs, rng)}
    router = torch.from_numpy(S.router(rng, E, H)).cuda()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    # calls in a row on the one shared array: different sizes and inputs, then a much smaller call in
    # another format and intermediate size after a call that left larger activation maxima behind
    for call, (kind, T, scale) in enumerate((("q4", 8, 1.0), ("q4", 33, 30.0), ("q8", 3, 0.01))):
        ex, desc = layers[kind]
        I = ex.I
        xh = (S.hidden(rng, T, H) * scale).astype(np.float32)
        x = torch.from_numpy(xh).cuda()
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
        g = got.cpu().numpy()
        assert np.isfinite(g).all()
        assert _row_err(g, want.cpu().numpy()) <= TOL, call
        # and on its own against the CPU oracle: each pick's unweighted expert output
        counts, rows = r.counts.cpu().numpy(), r.sorted_rows.cpu().numpy()
        pick_e = np.repeat(np.arange(E), counts)
        ref = np.stack([O.expert_forward(xh[rows[p]:rows[p] + 1], desc[pick_e[p]][0], desc[pick_e[p]][1], I)[0]
                        for p in range(P)])
        assert _row_err(g, ref) <= TOL, call


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
