"""GPU parity of the grouped-GEMM expert path (tcgen05 tensor cores, f16
operands with power-of-two range scaling, f32 accumulation) against the CPU
oracle's f32 path.

Bar: 2e-3 of each output row's largest magnitude, max|got - want| /
max|want| per row (f16 rounds each weight, token and activation once; the
reference multiplies in f32)."""

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

TOL_TC = 2e-3


@pytest.fixture(scope="module")
def D():
    from distributedmoellm_b200 import _build
    _build.build()
    from distributedmoellm_b200 import device
    device.require_device()
    return device


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def row_err(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float((np.abs(got - want).max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)).max())


def _experts(rng, kind, E, H, I, gs):
    """Device store + oracle descriptions of E random experts."""
    from distributedmoellm_b200 import layout as L
    from distributedmoellm_b200 import synthetic as S
    from distributedmoellm_b200.store import LayerExperts
    desc, parts = {}, {}
    for e in range(E):
        if kind in ("q4", "q4h"):
            gr, gsc, dr, dsc = S.int4_expert(rng, H, I, gs, f16_scales=(kind == "q4h"))
            parts[e] = (gr, gsc, dr, dsc)
            desc[e] = (("q4", gr, gsc.astype(np.float32), gs, False), ("q4", dr, dsc.astype(np.float32), gs, False))
        else:
            gq, gsc, dq, dsc = S.int8_expert(rng, H, I, gs)
            if kind == "q8h":
                gsc, dsc = gsc.astype(np.float16), dsc.astype(np.float16)
            parts[e] = (gq, gsc, dq, dsc)
            desc[e] = (("q8", gq, gsc.astype(np.float32), gs), ("q8", dq, dsc.astype(np.float32), gs))
    s0 = parts[0][1]
    fmt = L.fmt_of("q4" if kind.startswith("q4") else "q8", s0)
    ex = LayerExperts(E, H, I, gs, fmt, fmt, "cuda")
    for e, p in parts.items():
        if kind.startswith("q4"):
            ex.put_int4(e, *p, offset=False)
        else:
            ex.put_int8(e, *p)
    ex.publish()
    return ex, desc


def _run(D, ex, desc, counts, min_rows, seed):
    """Picks with the given per-expert counts (k = 1), through mb_moe_prefill."""
    rng = np.random.default_rng(seed)
    E, H, I = ex.E, ex.H, ex.I
    idx = np.repeat(np.arange(E, dtype=np.int32), counts)
    rng.shuffle(idx)
    T = len(idx)
    x = rng.standard_normal((T, H), dtype=np.float32)
    r = D.permute(cu(idx[:, None]), cu(np.ones((T, 1), np.float32)), E)
    y = torch.full((T, H), float("nan"), dtype=torch.float32, device="cuda")
    ws = torch.empty(D.prefill_workspace_bytes(T, H, I, ex.fmt_gu), dtype=torch.uint8, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    xd = cu(x)
    D.moe_prefill(ex.table, ex.eexp, E, H, I, ex.gs, ex.fmt_gu, ex.fmt_down, xd, D.row_exponents(xd), r, y, ws,
                  min_rows=min_rows, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    got = y.cpu().numpy()
    off = r.offsets.cpu().numpy()
    rows = r.sorted_rows.cpu().numpy()
    assert np.array_equal(r.counts.cpu().numpy(), np.asarray(counts))
    for e in range(E):
        seg = slice(off[e], off[e + 1])
        if counts[e] < min_rows:
            assert np.isnan(got[seg]).all(), f"expert {e} below min_rows was written"
            continue
        want = O.expert_forward(x[rows[seg]], desc[e][0], desc[e][1], I)
        assert np.isfinite(got[seg]).all()
        err = row_err(got[seg], want)
        assert err < TOL_TC, f"expert {e} ({counts[e]} rows): {err}"


@pytest.mark.parametrize("kind", ["q4", "q4h", "q8", "q8h"])
def test_prefill_ragged_counts(D, kind):
    """Counts 0, 1, 16, 17, 64, 192 (one full pass), 250 (two passes)."""
    ex, desc = _experts(np.random.default_rng(41), kind, 8, 256, 256, 32)
    _run(D, ex, desc, [250, 17, 1, 0, 192, 16, 64, 33], 1, 7)


def test_prefill_min_rows_leaves_small_experts(D):
    ex, desc = _experts(np.random.default_rng(42), "q4h", 6, 256, 192, 32)
    _run(D, ex, desc, [40, 31, 32, 5, 0, 100], 32, 8)


@pytest.mark.parametrize("H,I,gs", [(512, 320, 32), (384, 448, 64), (256, 128, 128)])
def test_prefill_shapes(D, H, I, gs):
    """Odd K-chunk counts (I = 320, 448), group sizes 64 and 128."""
    ex, desc = _experts(np.random.default_rng(H + I), "q4h", 3, H, I, gs)
    _run(D, ex, desc, [70, 9, 130], 1, 9)


def test_prefill_int8_group64(D):
    ex, desc = _experts(np.random.default_rng(43), "q8", 3, 512, 256, 64)
    _run(D, ex, desc, [300, 48, 2], 1, 10)


def test_prefill_bad_shape_raises(D):
    ex, _ = _experts(np.random.default_rng(44), "q4h", 2, 256, 96, 32)   # I % 64 != 0
    r = D.permute(cu(np.zeros((4, 1), np.int32)), None, 2)
    y = torch.empty((4, 256), dtype=torch.float32, device="cuda")
    ws = torch.empty(D.prefill_workspace_bytes(4, 256, 96), dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError, match="mb_moe_prefill"):
        xd = torch.zeros((4, 256), device="cuda")
        D.moe_prefill(ex.table, ex.eexp, 2, 256, 96, 32, ex.fmt_gu, ex.fmt_down, xd, D.row_exponents(xd), r, y, ws)


@pytest.fixture(scope="module")
def qwen_q8(D):
    """Int8 group-32 experts with f32 scales in the Qwen3-30B-A3B layer shape."""
    from distributedmoellm_b200 import synthetic as S
    from distributedmoellm_b200.layer import MoELayer
    rng = np.random.default_rng(3)
    H, I, E, k, gs = 2048, 768, 128, 8, 32
    ex, desc = _experts(rng, "q8", E, H, I, gs)
    router = S.router(rng, E, H)
    return MoELayer(cu(router), ex, k, True), desc, router, dict(H=H, I=I, E=E, k=k)


@pytest.mark.parametrize("T", [512, 2048, 4096])
def test_qwen_shape_prefill_layer_matches_oracle(qwen_q8, T):
    layer, desc, router, cfg = qwen_q8
    assert layer.uses_gemm(T)
    from distributedmoellm_b200 import synthetic as S
    x = S.hidden(np.random.default_rng(200 + T), T, cfg["H"])
    out = layer(cu(x)).cpu().numpy()
    b = layer.buffers(T)
    idx, w = b.idx.cpu().numpy(), b.w.cpu().numpy()
    ex, off, rows, wts = O.group_by_expert(idx, w)
    groups = [(ex[i], rows[off[i]:off[i + 1]], wts[off[i]:off[i + 1]]) for i in range(len(ex))]
    want = O.store_compute(x, groups, desc, cfg["I"])
    assert row_err(out, want) < TOL_TC
    assert layer.status(T) == 0


@pytest.fixture(scope="module")
def qwen_q4(D):
    """The north_star prefill layer: int4 group-32 experts with f16 scales in
    the Qwen3-30B-A3B layer shape (the benchmark's own recipe)."""
    from distributedmoellm_b200 import synthetic as S
    from distributedmoellm_b200.layer import MoELayer
    rng = np.random.default_rng(5)
    H, I, E, k, gs = 2048, 768, 128, 8, 32
    ex, desc = _experts(rng, "q4h", E, H, I, gs)
    router = S.router(rng, E, H)
    return MoELayer(cu(router), ex, k, True), desc, router, dict(H=H, I=I, E=E, k=k)


@pytest.mark.parametrize("T", [2048, 4096])
def test_qwen_shape_int4_prefill_layer_matches_oracle(qwen_q4, T):
    layer, desc, router, cfg = qwen_q4
    assert layer.uses_gemm(T)
    from distributedmoellm_b200 import synthetic as S
    x = S.hidden(np.random.default_rng(300 + T), T, cfg["H"])
    out = layer(cu(x)).cpu().numpy()
    b = layer.buffers(T)
    idx, w = b.idx.cpu().numpy(), b.w.cpu().numpy()
    ex, off, rows, wts = O.group_by_expert(idx, w)
    groups = [(ex[i], rows[off[i]:off[i + 1]], wts[off[i]:off[i + 1]]) for i in range(len(ex))]
    want = O.store_compute(x, groups, desc, cfg["I"])
    assert row_err(out, want) < TOL_TC
    assert layer.status(T) == 0


def _heavy_tailed(rng, T, H):
    """N(0, 1) token rows, with some rows far from it: a single large outlier
    per row, Student-t rows (df 1.5), and whole rows scaled by 1e-3 and 1e3."""
    x = rng.standard_normal((T, H), dtype=np.float32)
    n = max(1, T // 16)
    for r in range(0, n):
        x[r, rng.integers(0, H)] = np.float32(rng.choice([-1, 1]) * 300.0)
    x[n:2 * n] = rng.standard_t(1.5, (n, H)).astype(np.float32)
    x[2 * n:3 * n] *= np.float32(1e-3)
    x[3 * n:4 * n] *= np.float32(1e3)
    return x


@pytest.mark.parametrize("kind", ["q4h", "q8"])
def test_prefill_quantised_gaussian_weights_heavy_tailed_tokens(D, kind):
    """Weights quantised from N(0, 0.02) (int4: symmetric, scale absmax / 7,
    moelan/tiny.py:94-100, scales through f16; int8: GroupQuant.quantize,
    moelan/experts.py:134-142) instead of the uniform-nibble benchmark recipe,
    and heavy-tailed token rows: the activation exponent bound of the
    tensor-core path keeps the 2e-3 bar outside the synthetic recipe."""
    import cases as C
    from distributedmoellm_b200 import layout as L
    from distributedmoellm_b200 import synthetic as S
    from distributedmoellm_b200.layer import MoELayer
    from distributedmoellm_b200.store import LayerExperts
    rng = np.random.default_rng(61 if kind == "q4h" else 62)
    H, I, E, k, gs, T = 2048, 768, 16, 2, 32, 1024
    fmt = L.FMT_Q4_F16 if kind == "q4h" else L.FMT_Q8_F32
    ex = LayerExperts(E, H, I, gs, fmt, fmt, "cuda")
    desc = {}
    for e in range(E):
        if kind == "q4h":
            gr, gsc, dr, dsc = C.int4_expert(rng, H, I, gs, f16_scales=True)
            ex.put_int4(e, gr, gsc.astype(np.float16), dr, dsc.astype(np.float16))
            desc[e] = (("q4", gr, gsc, gs, False), ("q4", dr, dsc, gs, False))
        else:
            gq, gsc, dq, dsc = C.int8_expert(rng, H, I, gs)
            ex.put_int8(e, gq, gsc, dq, dsc)
            desc[e] = (("q8", gq, gsc, gs), ("q8", dq, dsc, gs))
    ex.publish()
    layer = MoELayer(cu(S.router(rng, E, H)), ex, k, True)
    assert layer.uses_gemm(T)
    x = _heavy_tailed(rng, T, H)
    out = layer(cu(x)).cpu().numpy()
    b = layer.buffers(T)
    idx, w = b.idx.cpu().numpy(), b.w.cpu().numpy()
    e_, off, rows, wts = O.group_by_expert(idx, w)
    groups = [(e_[i], rows[off[i]:off[i + 1]], wts[off[i]:off[i + 1]]) for i in range(len(e_))]
    want = O.store_compute(x, groups, desc, I)
    assert np.isfinite(out).all()
    assert row_err(out, want) < TOL_TC
    assert layer.status(T) == 0


def test_prefill_repeats_bit_identical(qwen_q8):
    """The grouped GEMMs are deterministic: repeated layer calls (two passes
    per expert at 4096 tokens) give bit-identical outputs and a clean status."""
    layer, desc, router, cfg = qwen_q8
    from distributedmoellm_b200 import synthetic as S
    x = cu(S.hidden(np.random.default_rng(77), 4096, cfg["H"]))
    first = layer(x).clone()
    for _ in range(6):
        assert torch.equal(layer(x), first)
    assert layer.status(4096) == 0


def _gguf_layer(rng, E, H, I, k):
    """Mixtral-style GGUF experts: gate and up Q4_K (Stacked), down Q8_0."""
    import types
    from distributedmoellm_b200 import layout as L
    from distributedmoellm_b200 import synthetic as S
    from distributedmoellm_b200.layer import MoELayer
    from distributedmoellm_b200.store import LayerExperts
    NS = types.SimpleNamespace
    ex = LayerExperts(E, H, I, 32, L.FMT_Q4K_F32, L.FMT_Q8_F16, "cuda")
    desc = {}
    for e in range(E):
        g, u = S.gguf_rows(rng, I, H, 12), S.gguf_rows(rng, I, H, 12)
        d = S.gguf_rows(rng, H, I, 8)
        ex.put_expert(e, NS(gu=NS(parts=(NS(raw=g, qtype=12, shape=(I, H)), NS(raw=u, qtype=12, shape=(I, H)))),
                            down=NS(raw=d, qtype=8, shape=(H, I)), inter=I))
        desc[e] = ([("gguf", g, 12, H), ("gguf", u, 12, H)], ("gguf", d, 8, I))
    ex.publish()
    router = S.router(rng, E, H)
    return MoELayer(cu(router), ex, k, True), desc


def _check_gguf_layer(layer, desc, x, I):
    """The layer against the oracle: 1e-5 per row when only the decode
    kernels ran (f32-exact products), 2e-3 when the grouped GEMM did."""
    out = layer(cu(x)).cpu().numpy()
    b = layer.buffers(x.shape[0])
    idx, w = b.idx.cpu().numpy(), b.w.cpu().numpy()
    ex, off, rows, wts = O.group_by_expert(idx, w)
    groups = [(ex[i], rows[off[i]:off[i + 1]], wts[off[i]:off[i + 1]]) for i in range(len(ex))]
    want = O.store_compute(x, groups, desc, I)
    tol = TOL_TC if layer.uses_gemm(x.shape[0]) else 1e-5
    assert row_err(out, want) < tol, (layer.kernel_plan(x.shape[0]), row_err(out, want))
    assert layer.status(x.shape[0]) == 0


def test_gguf_q4_k_layer_matches_oracle(D):
    """Q4_K gate|up + Q8_0 down: the affine int4 decode kernel at 1 and 12
    tokens (1e-5), the grouped GEMM at 300 (2e-3)."""
    rng = np.random.default_rng(12)
    layer, desc = _gguf_layer(rng, 4, 512, 256, 2)
    for T in (1, 12, 300):
        assert layer.uses_gemm(T) == (T == 300)
        _check_gguf_layer(layer, desc, rng.standard_normal((T, 512), dtype=np.float32), 256)


@pytest.mark.parametrize("T", [1, 16, 512])
def test_gguf_mixtral_shape_matches_oracle(D, T):
    """Config 4: d_model 4096, 8 experts top-2, intermediate 14336, Q4_K gate/up, Q8_0 down:
    the decode kernels in K windows (gate|up K = 4096, down K = 14336) at 1 and 16
    tokens, the grouped GEMM at 512."""
    global _MIXTRAL
    if "_MIXTRAL" not in globals():
        _MIXTRAL = _gguf_layer(np.random.default_rng(4), 8, 4096, 14336, 2)
    layer, desc = _MIXTRAL
    _check_gguf_layer(layer, desc, np.random.default_rng(40 + T).standard_normal((T, 4096), dtype=np.float32), 14336)
