"""GPU parity of every kernel on the routed-expert path against the
reference's own outputs (golden.npz) and the CPU oracle.

Bars: dequantisation and router indices / grouping bit-exact; f32-path
outputs within 1e-5 of the reference measured per output row as
max|got - want| / max|want| (the reference itself runs with fastmath and
cancels u*x*s against 8*s*sum(x), so element-wise relative error is not a
meaningful bar near zero)."""

import numpy as np
import pytest
import torch

import cases as C
import oracle as O

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5


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


def same_bits(got, want):
    fin = np.isfinite(want)
    return (np.array_equal(np.isnan(got), np.isnan(want)) and np.array_equal(np.isinf(got), np.isinf(want))
            and np.array_equal(got.view(np.uint32)[fin], want.view(np.uint32)[fin]))


# ---- dequantisation ------------------------------------------------------------------

@pytest.mark.parametrize("off", [0, 1])
@pytest.mark.parametrize("f16", [False, True])
def test_q4_dequant(D, golden, off, f16):
    raw, s = C.q4_deq_inputs()
    r = raw ^ 0x88 if off else raw
    if f16:
        s = s.astype(np.float16)
        want = O.q4_dequant(r, s.astype(np.float32), 32, bool(off))
    else:
        want = golden[f"q4_deq_off{off}"]
    got = D.q4_dequant(cu(r), cu(s), 32, bool(off)).cpu().numpy()
    assert same_bits(got, want)


def test_q8_dequant(D, golden):
    q, s = C.q8_deq_inputs()
    assert same_bits(D.q8_dequant(cu(q), cu(s), 32).cpu().numpy(), golden["q8_deq"])


@pytest.mark.parametrize("qt", sorted(C.GGUF_BLOCK))
def test_gguf_dequant_all_types(D, golden, qt):
    raw = C.gguf_deq_inputs(qt)
    got = D.gguf_dequant(cu(raw), qt, C.GGUF_COLS).cpu().numpy()
    assert same_bits(got, golden[f"gguf_deq_{qt}"])


def test_gguf_dequant_large(D):
    rng = np.random.default_rng(3)
    for qt in (12, 8, 14):
        raw = C.gguf_random_rows(300, 4096, qt, rng)
        got = D.gguf_dequant(cu(raw), qt, 4096).cpu().numpy()
        assert same_bits(got, O.gguf_dequant(raw, qt, 4096))


# ---- router, permute, combine --------------------------------------------------------

def test_router_known_answer(D, golden):
    idx, w = D.router_topk(cu(golden["router_known_logits"]), 2, True)
    assert idx.cpu().numpy().tolist() == [[1, 3], [0, 3]]
    np.testing.assert_allclose(w.cpu().numpy(), golden["router_known_w"], rtol=1e-6)


@pytest.mark.parametrize("case", C.ROUTER_CASES, ids=[c[0] for c in C.ROUTER_CASES])
def test_router_topk_matches_reference(D, golden, case):
    name, T, E, k, norm, seed = case
    lg = C.router_logits(T, E, seed)
    idx, w = D.router_topk(cu(lg), k, norm)
    idx, w = idx.cpu().numpy(), w.cpu().numpy()
    ties = set(O.near_ties(lg, k).tolist())
    rows = [t for t in range(T) if t not in ties]
    assert len(ties) <= max(1, T // 50)
    assert np.array_equal(idx[rows], golden[f"{name}_idx"][rows])
    np.testing.assert_allclose(w[rows], golden[f"{name}_w"][rows], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("T,H,E,k", [(1, 2048, 128, 8), (37, 2048, 128, 8), (64, 256, 16, 2), (300, 4096, 8, 2),
                                     (5, 200, 60, 6), (600, 2048, 128, 8), (777, 1000, 60, 6), (2048, 2048, 128, 8)])
def test_router_logits_and_route(D, T, H, E, k):
    rng = np.random.default_rng(T + H)
    x = rng.standard_normal((T, H)).astype(np.float32)
    r = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    want = x.astype(np.float64) @ r.T.astype(np.float64)
    lg = D.router_logits(cu(x), cu(r)).cpu().numpy()
    assert np.abs(lg - want).max() <= 2e-6 * np.abs(want).max()
    logits = torch.empty((T, E), dtype=torch.float32, device="cuda")
    rexp = torch.empty(T, dtype=torch.int32, device="cuda")
    idx, w = D.router_route(cu(x), cu(r), k, True, logits=logits, row_exp=rexp)
    lg2 = logits.cpu().numpy()
    assert np.array_equal(lg2, lg)                        # the same slice-ordered sums
    ridx, rw = O.route(lg2, k, True)
    keep = [t for t in range(T) if t not in set(O.near_ties(lg2, k).tolist())]
    assert np.array_equal(idx.cpu().numpy()[keep], ridx[keep])
    np.testing.assert_allclose(w.cpu().numpy()[keep], rw[keep], rtol=2e-6, atol=1e-7)
    amax = np.abs(x).max(axis=1)
    assert np.array_equal(rexp.cpu().numpy(), 14 - np.frexp(amax)[1])


@pytest.mark.parametrize("case", C.ROUTER_CASES, ids=[c[0] for c in C.ROUTER_CASES])
def test_permute_matches_group_by_expert(D, golden, case):
    name, T, E, k, norm, seed = case
    idx, w = golden[f"{name}_idx"], golden[f"{name}_w"]
    r = D.permute(cu(idx), cu(w), E)
    torch.cuda.synchronize()
    n = int(r.n_unique.item())
    assert np.array_equal(r.uexperts[:n].cpu().numpy(), golden[f"{name}_experts"])
    assert np.array_equal(r.uoffsets[:n + 1].cpu().numpy(), golden[f"{name}_offsets"])
    assert np.array_equal(r.sorted_rows[:T * k].cpu().numpy(), golden[f"{name}_rows"])
    assert np.array_equal(r.sorted_w[:T * k].cpu().numpy(), golden[f"{name}_weights"])
    inv = r.inv[:T * k].cpu().numpy()
    assert np.array_equal(np.sort(inv), np.arange(T * k))
    counts = np.bincount(idx.reshape(-1), minlength=E)
    assert np.array_equal(r.counts.cpu().numpy(), counts)


def test_permute_large_and_skewed(D):
    rng = np.random.default_rng(7)
    T, k, E = 4096, 8, 128
    idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    idx[:1000, 0] = 5                      # a hot expert
    idx[:1000, 1:] = np.arange(1, k)[None, :] + 10
    w = rng.random((T, k), dtype=np.float32)
    r = D.permute(cu(idx), cu(w), E)
    ex, off, rows, wts = O.group_by_expert(idx, w)
    torch.cuda.synchronize()
    assert np.array_equal(r.sorted_rows.cpu().numpy(), rows)
    assert np.array_equal(r.sorted_w.cpu().numpy(), wts)
    assert int(r.n_unique.item()) == len(ex)


@pytest.mark.parametrize("T,k,E", [(1, 1, 1), (2047, 1, 7), (2048, 1, 3), (2049, 1, 5), (750, 8, 64),
                                   (3000, 6, 60), (8192, 8, 1024), (65536, 1, 2)])
def test_permute_sizes(D, T, k, E):
    """One CTA up to 2048 picks, then one more per 2048 up to a cluster of 8:
    the chunk edges, the largest E (shared memory) and the largest P."""
    rng = np.random.default_rng(T + E)
    idx = rng.integers(0, E, (T, k)).astype(np.int32)
    if E >= k:
        idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    w = rng.random((T, k), dtype=np.float32)
    r = D.permute(cu(idx), cu(w), E)
    ex, off, rows, wts = O.group_by_expert(idx, w)
    torch.cuda.synchronize()
    n = int(r.n_unique.item())
    assert n == len(ex)
    assert np.array_equal(r.uexperts[:n].cpu().numpy(), ex)
    assert np.array_equal(r.uoffsets[:n + 1].cpu().numpy(), off)
    assert np.array_equal(r.sorted_rows.cpu().numpy()[:T * k], rows)
    assert np.array_equal(r.sorted_w.cpu().numpy()[:T * k], wts)
    counts = np.bincount(idx.reshape(-1), minlength=E)
    assert np.array_equal(r.counts.cpu().numpy(), counts)
    assert np.array_equal(r.offsets.cpu().numpy(), np.concatenate([[0], np.cumsum(counts)]))
    inv = r.inv[:T * k].cpu().numpy()
    assert np.array_equal(r.sorted_rows.cpu().numpy()[inv], np.repeat(np.arange(T), k))


def test_combine(D):
    rng = np.random.default_rng(1)
    T, k, H = 37, 3, 256
    y = rng.standard_normal((T * k, H)).astype(np.float32)
    inv = rng.permutation(T * k).astype(np.int32)
    w = rng.random(T * k).astype(np.float32)
    want = np.zeros((T, H), np.float32)
    for t in range(T):
        for j in range(k):
            want[t] += w[t * k + j] * y[inv[t * k + j]]
    got = D.combine(cu(y), cu(inv), cu(w), T, k).cpu().numpy()
    assert row_err(got, want) < 1e-6
    base = rng.standard_normal((T, H)).astype(np.float32)
    out = cu(base)
    D.combine(cu(y), cu(inv), cu(w), T, k, out=out, accumulate=True)
    assert row_err(out.cpu().numpy(), want + base) < 1e-6


# ---- single-matrix products from packed bytes ----------------------------------------

@pytest.mark.parametrize("rows", C.MATMUL_ROWS)
def test_q4_matmul_known_answer(D, golden, rows):
    from distributedmoellm_b200 import layout as L
    raw, s, W, x = C.q4_mm_inputs(rows)
    tiles = cu(L.q4_tiles(raw, s, 32, False))
    got = D.matmul_t(tiles, L.FMT_Q4_F32, 96, 128, cu(x)).cpu().numpy()
    np.testing.assert_allclose(got, x @ W.T, atol=1e-3)
    assert row_err(got, golden[f"q4_mm_{rows}"]) < TOL_F32


@pytest.mark.parametrize("n", [1, 5, 9, 40])
def test_q8_matmul(D, n):
    from distributedmoellm_b200 import layout as L
    rng = np.random.default_rng(n)
    q = rng.integers(-127, 128, (200, 768), dtype=np.int8)
    s = (rng.random((200, 24), dtype=np.float32) * 1e-3)
    x = rng.standard_normal((n, 768)).astype(np.float32)
    got = D.matmul_t(cu(L.q8_tiles(q, s, 32)), L.FMT_Q8_F32, 200, 768, cu(x)).cpu().numpy()
    assert row_err(got, O.q8_matmul_t(x, q, s, 32)) < TOL_F32


@pytest.mark.parametrize("rows", C.GGUF_MM_ROWS)
def test_gguf_q8_0_and_q4_0_matmul(D, golden, rows):
    from distributedmoellm_b200 import layout as L
    raw, x = C.gguf_mm_inputs(8, rows)
    q, d = L.q8_0_as_q8(raw, C.GGUF_COLS)
    got = D.matmul_t(cu(L.q8_tiles(q, d, 32)), L.FMT_Q8_F16, raw.shape[0], C.GGUF_COLS, cu(x)).cpu().numpy()
    assert row_err(got, golden[f"gguf_mm_8_{rows}"]) < TOL_F32
    raw, x = C.gguf_mm_inputs(2, rows)
    u, d = L.q4_0_as_q4(raw, C.GGUF_COLS)
    got = D.matmul_t(cu(L.q4_tiles(u, d, 32, True)), L.FMT_Q4_F16, raw.shape[0], C.GGUF_COLS, cu(x)).cpu().numpy()
    assert row_err(got, golden[f"gguf_mm_2_{rows}"]) < TOL_F32


@pytest.mark.parametrize("K", [2176, 4096, 14336])
@pytest.mark.parametrize("n", [1, 6])
def test_matmul_wide_k_windows(D, K, n):
    """K above 2048 runs in windows of 2048 columns: int4 (f16 scales),
    int8 (f32 scales) and the affine int4 form of GGUF Q4_K."""
    from distributedmoellm_b200 import layout as L
    rng = np.random.default_rng(K + n)
    O_ = 72
    x = rng.standard_normal((n, K)).astype(np.float32)
    raw = rng.integers(0, 256, (O_, K // 2), dtype=np.uint8)
    s = (rng.random((O_, K // 32), dtype=np.float32) * 1e-2).astype(np.float16)
    got = D.matmul_t(cu(L.q4_tiles(raw, s, 32, False)), L.FMT_Q4_F16, O_, K, cu(x)).cpu().numpy()
    assert row_err(got, O.q4_matmul_t(x, raw, s.astype(np.float32), 32, False)) < TOL_F32
    q = rng.integers(-127, 128, (O_, K), dtype=np.int8)
    s8 = rng.random((O_, K // 64), dtype=np.float32) * 1e-3
    got = D.matmul_t(cu(L.q8_tiles(q, s8, 64)), L.FMT_Q8_F32, O_, K, cu(x)).cpu().numpy()
    assert row_err(got, O.q8_matmul_t(x, q, s8, 64)) < TOL_F32
    if K % 256 == 0:
        g = C.gguf_random_rows(O_, K, 12, rng, 0.01)
        got = D.matmul_t(cu(L.q4k_tiles(g, K)), L.FMT_Q4K_F32, O_, K, cu(x)).cpu().numpy()
        w = O.gguf_dequant(g, 12, K).astype(np.float64)
        assert row_err(got, x.astype(np.float64) @ w.T) < TOL_F32


@pytest.mark.parametrize("T", [1, 5, 40])
def test_wide_layer_decode_matches_oracle(D, T):
    """A layer whose gate|up (K = H = 3072) and down (K = I = 2560) both run in
    two K windows, the second one narrow (8 and 4 of 16 quads), through the
    decode kernels only: 1, 5 and 40 tokens (chunks of up to 8 picks, several
    segments per chunk)."""
    from distributedmoellm_b200 import synthetic as S
    rng = np.random.default_rng(90 + T)
    cfg = dict(H=3072, I=2560, E=8, k=2, gs=32)
    experts = {e: C.int4_expert(rng, cfg["H"], cfg["I"], 32, f16_scales=True) for e in range(cfg["E"])}
    router = rng.standard_normal((cfg["E"], cfg["H"])).astype(np.float32)
    layer = _layer(cfg, "q4", experts, router, f16=True)
    layer.gemm_min_rows = 0
    x = S.hidden(rng, T, cfg["H"])
    out = layer(cu(x)).cpu().numpy()
    b = layer.buffers(T)
    idx, w = b.idx.cpu().numpy(), b.w.cpu().numpy()
    e_, off, rows, wts = O.group_by_expert(idx, w)
    groups = [(e_[i], rows[off[i]:off[i + 1]], wts[off[i]:off[i + 1]]) for i in range(len(e_))]
    desc = {e: (("q4", g, gs_, 32, False), ("q4", d, ds, 32, False)) for e, (g, gs_, d, ds) in experts.items()}
    want = O.store_compute(x, groups, desc, cfg["I"])
    assert row_err(out, want) < TOL_F32
    assert layer.status(T) == 0


@pytest.mark.parametrize("qt", sorted(C.GGUF_BLOCK))
@pytest.mark.parametrize("rows", C.GGUF_MM_ROWS)
def test_gguf_matmul_all_types(D, golden, qt, rows):
    """mb_gguf_matmul_t straight from the blocks, every type, against the
    reference's fused mat-vecs (its own bar: rtol = atol = 1e-4,
    tests/test_gguf.py:34-39) and against the oracle's f32 product of the
    bit-exact dequantised weights (1e-5 per row)."""
    raw, x = C.gguf_mm_inputs(qt, rows)
    got = D.gguf_matmul_t(cu(raw), qt, C.GGUF_COLS, cu(x)).cpu().numpy()
    np.testing.assert_allclose(got, golden[f"gguf_mm_{qt}_{rows}"], rtol=1e-4, atol=1e-4)
    w = O.gguf_dequant(raw, qt, C.GGUF_COLS).astype(np.float64)
    assert row_err(got, x.astype(np.float64) @ w.T) < TOL_F32


@pytest.mark.parametrize("qt", [12, 8, 14])
def test_gguf_matmul_wide(D, qt):
    """Mixtral-wide rows (K = 14336) and more input rows than one pass takes."""
    rng = np.random.default_rng(qt)
    raw = C.gguf_random_rows(40, 14336, qt, rng, 0.001)
    x = rng.standard_normal((11, 14336)).astype(np.float32)
    got = D.gguf_matmul_t(cu(raw), qt, 14336, cu(x)).cpu().numpy()
    w = O.gguf_dequant(raw, qt, 14336).astype(np.float64)
    assert row_err(got, x.astype(np.float64) @ w.T) < TOL_F32


# ---- one MoE layer ------------------------------------------------------------------

def _layer(cfg, kind, experts, router, f16=False):
    from distributedmoellm_b200 import layout as L
    from distributedmoellm_b200.layer import MoELayer
    from distributedmoellm_b200.store import LayerExperts
    H, I, E = cfg["H"], cfg["I"], cfg["E"]
    if kind == "q4":
        s0 = experts[0][1].astype(np.float16) if f16 else experts[0][1]
        fmt = L.fmt_of("q4", s0)
    else:
        fmt = L.FMT_Q8_F32
    ex = LayerExperts(E, H, I, cfg["gs"], fmt, fmt, "cuda")
    for e, parts in experts.items():
        if kind == "q4":
            gr, gsc, dr, dsc = parts
            if f16:
                gsc, dsc = gsc.astype(np.float16), dsc.astype(np.float16)
            ex.put_int4(e, gr, gsc, dr, dsc, offset=False)
        else:
            ex.put_int8(e, *parts)
    ex.publish()
    return MoELayer(cu(router), ex, cfg["k"], True, gemm_min_rows=0)   # the f32 decode path (1e-5 bar)


def test_layer_int4_matches_reference(D, golden):
    x, router, experts = C.layer_inputs(C.LAYER, "int4")
    layer = _layer(C.LAYER, "q4", experts, router)
    out = layer(cu(x)).cpu().numpy()
    b = layer.buffers(x.shape[0])
    ties = set(O.near_ties(golden["layer_q4_logits"], 2).tolist())
    rows = [t for t in range(x.shape[0]) if t not in ties]
    assert np.array_equal(b.idx.cpu().numpy()[rows], golden["layer_q4_idx"][rows])
    assert row_err(out[rows], golden["layer_q4_out"][rows]) < TOL_F32
    assert layer.status(x.shape[0]) == 0


def test_layer_int4_f16_scales_matches_reference(D, golden):
    x, router, experts = C.layer_inputs(C.LAYER_F16, "int4", f16_scales=True)
    layer = _layer(C.LAYER_F16, "q4", experts, router, f16=True)
    out = layer(cu(x)).cpu().numpy()
    assert np.array_equal(layer.buffers(x.shape[0]).idx.cpu().numpy(), golden["layer_q4h_idx"])
    assert row_err(out, golden["layer_q4h_out"]) < TOL_F32


def test_layer_int8_matches_reference(D, golden):
    x, router, experts = C.layer_inputs(C.LAYER_Q8, "int8")
    layer = _layer(C.LAYER_Q8, "q8", experts, router)
    out = layer(cu(x)).cpu().numpy()
    assert np.array_equal(layer.buffers(x.shape[0]).idx.cpu().numpy(), golden["layer_q8_idx"])
    assert row_err(out, golden["layer_q8_out"]) < TOL_F32


@pytest.fixture(scope="module")
def qwen_layer(D):
    """Config 2: Qwen3-30B-A3B MoE layer shape, int4 g32 with f16 scales."""
    from distributedmoellm_b200 import synthetic as S
    rng = np.random.default_rng(0)
    H, I, E, k, gs = 2048, 768, 128, 8, 32
    experts = {e: S.int4_expert(rng, H, I, gs, f16_scales=True) for e in range(E)}
    router = S.router(rng, E, H)
    cfg = dict(H=H, I=I, E=E, k=k, gs=gs)
    layer = _layer(cfg, "q4", experts, router, f16=True)
    desc = {e: (("q4", gr, gsc.astype(np.float32), gs, False), ("q4", dr, dsc.astype(np.float32), gs, False))
            for e, (gr, gsc, dr, dsc) in experts.items()}
    return layer, desc, router, cfg


@pytest.mark.parametrize("T", [1, 8, 32, 64])
def test_qwen_shape_decode_matches_oracle(qwen_layer, T):
    layer, desc, router, cfg = qwen_layer
    from distributedmoellm_b200 import synthetic as S
    x = S.hidden(np.random.default_rng(100 + T), T, cfg["H"])
    out = layer(cu(x)).cpu().numpy()
    b = layer.buffers(T)
    idx, w = b.idx.cpu().numpy(), b.w.cpu().numpy()
    ex, off, rows, wts = O.group_by_expert(idx, w)
    groups = [(ex[i], rows[off[i]:off[i + 1]], wts[off[i]:off[i + 1]]) for i in range(len(ex))]
    want = O.store_compute(x, groups, desc, cfg["I"])
    assert row_err(out, want) < TOL_F32
    # and the router against the oracle's on the GPU's own logits
    ridx, rw = O.route(b.logits.cpu().numpy(), cfg["k"], True)
    ties = set(O.near_ties(b.logits.cpu().numpy(), cfg["k"]).tolist())
    keep = [t for t in range(T) if t not in ties]
    assert np.array_equal(idx[keep], ridx[keep])
    assert layer.status(T) == 0


def test_layer_graph_replay_matches_eager(qwen_layer):
    layer, desc, router, cfg = qwen_layer
    from distributedmoellm_b200 import synthetic as S
    x = cu(S.hidden(np.random.default_rng(5), 16, cfg["H"]))
    eager = layer(x).clone()
    g = layer.capture(x)
    x2 = cu(S.hidden(np.random.default_rng(6), 16, cfg["H"]))
    want2 = layer(x2).clone()
    x.copy_(x2)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(layer.buffers(16).out, want2)
    x.copy_(cu(S.hidden(np.random.default_rng(5), 16, cfg["H"])))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(layer.buffers(16).out, eager)


def test_bad_format_raises(D):
    from distributedmoellm_b200 import _lib
    t = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    x = torch.zeros((2, 128), dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError, match="weight format"):
        D.matmul_t(t, 99, 16, 128, x)
    assert "weight format" in _lib.last_error()


# ---- activation rows in the wire formats ---------------------------------------------

@pytest.mark.parametrize("name", ["wide", "narrow", "zeros", "halfway"])
@pytest.mark.parametrize("wire", ["f16", "int8"])
def test_wire_rows_bit_exact(D, golden, name, wire):
    """mb_encode_rows / mb_decode_rows against the reference's encode_rows /
    decode_rows (moelan/protocol.py:99-123), bit for bit."""
    a = C.wire_inputs()[name]
    q, s = D.encode_rows(cu(a), wire)
    qh = q.cpu().numpy()
    assert np.array_equal(qh.view(np.uint8), golden[f"wire_{name}_{wire}_q"].view(np.uint8))
    if wire == "int8":
        assert np.array_equal(s.cpu().numpy().view(np.uint32), golden[f"wire_{name}_{wire}_s"].view(np.uint32))
    dec = D.decode_rows(q, s).cpu().numpy()
    assert np.array_equal(dec.view(np.uint32), golden[f"wire_{name}_{wire}_dec"].view(np.uint32))


def test_wire_rows_large_round_trip(D):
    """A decode-step-sized batch (64 x 2048) and a prefill-sized one (2048 x
    2048): device bytes equal the restatement's; the reference test's size and
    error bounds hold (f16 1e-3, int8 6e-3 of each row's largest magnitude)."""
    rng = np.random.default_rng(8)
    for n in (64, 2048):
        a = (rng.standard_normal((n, 2048)) * 3).astype(np.float32)
        a[:, 7] *= 40
        for wire, tol in (("f16", 1e-3), ("int8", 6e-3)):
            q, s = D.encode_rows(cu(a), wire)
            wq, ws = O.encode_rows(a, wire)
            assert np.array_equal(q.cpu().numpy().view(np.uint8), wq.view(np.uint8))
            dec = D.decode_rows(q, s).cpu().numpy()
            err = np.abs(dec - a)[:, 64:].max(1) / np.abs(a[:, 64:]).max(1)
            assert err.max() <= tol


# ---- the other routers ----------------------------------------------------------------

def _near_ties(v: np.ndarray, n: int, ulps: int = 4) -> np.ndarray:
    """Rows whose n + 1 largest values hold two distinct ones within ulps f32
    ulps: ranking them can differ through the last bit of an exponential."""
    s = -np.sort(-v.astype(np.float32), axis=1)[:, :n + 1]
    gap = s[:, :-1] - s[:, 1:]
    return ((gap <= ulps * np.spacing(np.abs(s[:, :-1]))) & (gap != 0)).any(axis=1)


@pytest.mark.parametrize("case", C.GROUPED_CASES, ids=[c[0] for c in C.GROUPED_CASES])
def test_grouped_router_matches_reference(D, golden, case):
    """mb_router_grouped against moelan's route_grouped: indices bit-exact
    (rows with a near-tie among the deciding choices or group scores aside:
    none in these cases is expected, and they are counted), weights within
    2e-6 relative (the device's exp and sum order differ from numpy's in the
    last bits)."""
    name, T, E, k, scoring, method, ng, tg, norm, scale, with_bias, seed = case
    lg, bias = C.grouped_inputs(T, E, with_bias, seed)
    idx, w = D.router_grouped(cu(lg), k, scoring, method, ng, tg, norm, scale, None if bias is None else cu(bias))
    idx, w = idx.cpu().numpy(), w.cpu().numpy()
    _, _, choice = O.route_grouped(lg, k, scoring, method, ng, tg, norm, scale, bias)
    skip = _near_ties(choice, k)
    if method != "greedy" and ng > 1:
        sc = 1.0 / (1.0 + np.exp(-lg)) if scoring == "sigmoid" else O.softmax(lg)
        ch = (sc + bias[None, :]) if bias is not None else sc
        g = ch.reshape(T, ng, E // ng)
        gs = -np.sort(-g, axis=-1)[..., :2].sum(-1) if method == "noaux_tc" else g.max(-1)
        skip |= _near_ties(gs, tg)
    assert skip.sum() <= 2
    want_i, want_w = golden[f"grouped_{name}_idx"], golden[f"grouped_{name}_w"]
    assert np.array_equal(idx[~skip], want_i[~skip])
    np.testing.assert_allclose(w[~skip], want_w[~skip], rtol=2e-6, atol=1e-12)


@pytest.mark.parametrize("name", ["hf", "wide"])
@pytest.mark.parametrize("eps", [0.01, 0.1])
def test_sparsemixer_matches_reference(D, golden, name, eps):
    """mb_router_sparsemixer against moelan's route_sparsemixer on the
    reference's own near-tie / negative / zero case: picks bit-exact (they
    come from the logits alone), weights within 2e-6 relative."""
    lg = C.sparsemixer_inputs()[name]
    idx, w = D.router_sparsemixer(cu(lg), eps)
    assert np.array_equal(idx.cpu().numpy(), golden[f"sparse_{name}_{eps}_idx"])
    np.testing.assert_allclose(w.cpu().numpy(), golden[f"sparse_{name}_{eps}_w"], rtol=2e-6, atol=1e-12)
    assert (golden[f"sparse_{name}_{eps}_w"] < 0.999).any()


def test_grouped_router_large_batch(D):
    """DeepSeek-V3 routing (256 experts, 8 groups, keep 4, top-8) at prefill
    size against the numpy restatement."""
    rng = np.random.default_rng(99)
    T, E = 4096, 256
    lg = rng.standard_normal((T, E)).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.05).astype(np.float32)
    idx, w = D.router_grouped(cu(lg), 8, "sigmoid", "noaux_tc", 8, 4, True, 2.5, cu(bias))
    want_i, want_w, choice = O.route_grouped(lg, 8, "sigmoid", "noaux_tc", 8, 4, True, 2.5, bias)
    ok = ~_near_ties(choice, 8)
    assert ok.mean() > 0.99
    assert np.array_equal(idx.cpu().numpy()[ok], want_i[ok])
    np.testing.assert_allclose(w.cpu().numpy()[ok], want_w[ok], rtol=2e-6, atol=1e-12)


# ---- the tile layout made on the device -------------------------------------------------

@pytest.mark.parametrize("O,K,gs,inter", [(96, 256, 32, 0), (33, 384, 64, 0), (2 * 52, 512, 32, 52),
                                          (1536, 2048, 32, 768), (2048, 768, 32, 0)])
@pytest.mark.parametrize("f16", [False, True])
def test_pack_matches_host_layout(D, O, K, gs, inter, f16):
    """mb_pack_q4 / mb_pack_q8 write byte for byte what layout.q4_tiles /
    q8_tiles write, both nibble forms, plain and gate|up matrices, ragged rows."""
    from distributedmoellm_b200 import layout as L
    rng = np.random.default_rng(O + K)
    raw = rng.integers(0, 256, (O, K // 2), dtype=np.uint8)
    s = rng.random((O, K // gs), dtype=np.float32)
    if f16:
        s = s.astype(np.float16)
    for offset in (False, True):
        got = D.pack_q4(cu(raw), cu(s), gs, offset, inter).cpu().numpy()
        assert np.array_equal(got, L.q4_tiles(raw, s, gs, offset, gu_inter=inter))
    q = rng.integers(-127, 128, (O, K), dtype=np.int8)
    got = D.pack_q8(cu(q), cu(s), gs, inter).cpu().numpy()
    assert np.array_equal(got, L.q8_tiles(q, s, gs, gu_inter=inter))


@pytest.mark.parametrize("O,K,inter", [(40, 512, 0), (2 * 56, 1024, 56), (4096, 256, 0)])
def test_pack_q4k_matches_host_layout(D, O, K, inter):
    """mb_pack_q4k against layout.q4k_tiles on random Q4_K rows: every packed
    scale / min code, f16 d and dmin finite (normal and subnormal; an infinite
    d makes NaN biases, whose bit pattern differs between numpy and CUDA)."""
    from distributedmoellm_b200 import layout as L
    rng = np.random.default_rng(O)
    raw = rng.integers(0, 256, (O, K // 256, 144), dtype=np.uint8)
    dd = (rng.standard_normal((O, K // 256, 2)) * 0.01).astype(np.float16)
    dd[::7, :, 0] = np.float16(3e-6)                      # subnormal d
    raw[:, :, 0:4] = dd.view(np.uint8).reshape(O, K // 256, 4)
    raw = raw.reshape(O, K // 256 * 144)
    got = D.pack_q4k(cu(raw), K, inter).cpu().numpy()
    want = L.q4k_tiles(raw, K, gu_inter=inter)
    assert np.array_equal(got, want)
