"""The CPU oracle against the reference's own outputs (golden.npz, made by
tests/golden/make_golden.py from moelan itself).  Nothing here needs a GPU."""

import numpy as np
import pytest

import cases as C
import oracle as O


def test_router_known_answer(golden):
    # tests/test_moelan.py:64-71 of the reference
    idx, w = O.route(golden["router_known_logits"], 2, True)
    assert idx.tolist() == [[1, 3], [0, 3]]
    assert np.array_equal(idx, golden["router_known_idx"])
    np.testing.assert_allclose(w, golden["router_known_w"], rtol=1e-6)
    ex, off, rows, wts = O.group_by_expert(idx, w)
    assert ex.tolist() == [0, 1, 3] and rows[off[2]:off[3]].tolist() == [0, 1]


@pytest.mark.parametrize("case", C.ROUTER_CASES, ids=[c[0] for c in C.ROUTER_CASES])
def test_router_and_grouping(golden, case):
    name, T, E, k, norm, seed = case
    idx, w = O.route(C.router_logits(T, E, seed), k, norm)
    assert np.array_equal(idx, golden[f"{name}_idx"])
    np.testing.assert_allclose(w, golden[f"{name}_w"], rtol=1e-6, atol=1e-7)
    for got, key in zip(O.group_by_expert(idx, golden[f"{name}_w"]), ("experts", "offsets", "rows", "weights")):
        assert np.array_equal(got, golden[f"{name}_{key}"]), key


@pytest.mark.parametrize("off", [0, 1])
def test_q4_dequant_bit_exact(golden, off):
    raw, s = C.q4_deq_inputs()
    r = np.bitwise_xor(raw, 0x88) if off else raw
    assert np.array_equal(O.q4_dequant(r, s, C.Q4_DEQ["gs"], bool(off)), golden[f"q4_deq_off{off}"])


def test_q8_dequant_bit_exact(golden):
    q, s = C.q8_deq_inputs()
    assert np.array_equal(O.q8_dequant(q, s, C.Q8_DEQ["gs"]), golden["q8_deq"])


@pytest.mark.parametrize("qt", sorted(C.GGUF_BLOCK), ids=[O.QTYPES[q][0] for q in sorted(C.GGUF_BLOCK)])
def test_gguf_dequant_bit_exact(golden, qt):
    got = O.gguf_dequant(C.gguf_deq_inputs(qt), qt, C.GGUF_COLS)
    want = golden[f"gguf_deq_{qt}"]
    # bit-exact including the non-finite pattern (the reference maps f16 exponent 31 to inf)
    assert np.array_equal(got.view(np.uint32)[np.isfinite(want)], want.view(np.uint32)[np.isfinite(want)])
    assert np.array_equal(np.isnan(got), np.isnan(want)) and np.array_equal(np.isinf(got), np.isinf(want))


@pytest.mark.parametrize("qt", sorted(C.GGUF_BLOCK), ids=[O.QTYPES[q][0] for q in sorted(C.GGUF_BLOCK)])
@pytest.mark.parametrize("rows", C.GGUF_MM_ROWS)
def test_gguf_matmul(golden, qt, rows):
    raw, x = C.gguf_mm_inputs(qt, rows)
    np.testing.assert_allclose(O.gguf_matmul_t(x, raw, qt, C.GGUF_COLS), golden[f"gguf_mm_{qt}_{rows}"],
                               rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("rows", C.MATMUL_ROWS)
def test_q4_matmul_known_answer(golden, rows):
    raw, s, W, x = C.q4_mm_inputs(rows)
    np.testing.assert_allclose(O.q4_matmul_t(x, raw, s, 32, False), x @ W.T, atol=1e-3)
    _close_rows(O.q4_matmul_t(x, raw, s, 32, False), golden[f"q4_mm_{rows}"], 1e-5)
    _close_rows(O.q4_matmul_t(x, raw ^ 0x88, s, 32, True), golden[f"q4_mm_res_{rows}"], 1e-5)
    if rows == 1:
        assert np.array_equal(O.q4_dequant(raw, s, 32, False), golden["q4_mm_dequant"])


def _q4_desc(experts, resident_every=0):
    out = {}
    for e, (gr, gsc, dr, dsc) in experts.items():
        res = bool(resident_every and e % resident_every == 1)
        if res:
            gr, dr = gr ^ 0x88, dr ^ 0x88
        out[e] = (("q4", gr, gsc, 32, res), ("q4", dr, dsc, 32, res))
    return out


def _close_rows(got, want, tol):
    """max |got - want| over each row, relative to max |want| of that row."""
    err = np.abs(got - want).max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)
    assert err.max() <= tol, err.max()


def test_layer_int4(golden):
    x, router, experts = C.layer_inputs(C.LAYER, "int4")
    out, idx, w = O.moe_layer(x, router, _q4_desc(experts, 3), C.LAYER["k"], True, C.LAYER["I"])
    assert np.array_equal(idx, golden["layer_q4_idx"])
    _close_rows(out, golden["layer_q4_out"], 1e-5)


def test_layer_int4_f16_scales(golden):
    x, router, experts = C.layer_inputs(C.LAYER_F16, "int4", f16_scales=True)
    out, idx, _ = O.moe_layer(x, router, _q4_desc(experts), 2, True, C.LAYER_F16["I"])
    assert np.array_equal(idx, golden["layer_q4h_idx"])
    _close_rows(out, golden["layer_q4h_out"], 1e-5)


def test_layer_int8(golden):
    x, router, experts = C.layer_inputs(C.LAYER_Q8, "int8")
    desc = {e: (("q8", q1, s1, 32), ("q8", q2, s2, 32)) for e, (q1, s1, q2, s2) in experts.items()}
    out, idx, _ = O.moe_layer(x, router, desc, 2, True, C.LAYER_Q8["I"])
    assert np.array_equal(idx, golden["layer_q8_idx"])
    _close_rows(out, golden["layer_q8_out"], 1e-5)


def test_layer_gguf(golden):
    cfg = C.LAYER_GGUF
    x, router, experts = C.layer_inputs(cfg, "gguf")
    desc = {e: ([("gguf", gr, 12, cfg["H"]), ("gguf", ur, 12, cfg["H"])], ("gguf", dr, 8, cfg["I"]))
            for e, (gr, ur, dr) in experts.items()}
    out, idx, _ = O.moe_layer(x, router, desc, 2, True, cfg["I"])
    assert np.array_equal(idx, golden["layer_gguf_idx"])
    _close_rows(out, golden["layer_gguf_out"], 1e-5)


def test_moe_q4_mixed_raw_and_resident(golden):
    x, _, experts = C.layer_inputs(C.LAYER_F16, "int4")
    d = _q4_desc(experts)
    a, b = d[3], d[6]
    wv = np.array([0.25, 0.75], np.float32)
    keep = [np.ascontiguousarray(v) for v in (a[0][1], a[0][2], a[1][1], a[1][2],
                                               b[0][1] ^ 0x88, b[0][2], b[1][1] ^ 0x88, b[1][2])]
    items = [((O._addr(keep[0]), O._addr(keep[1]), O._addr(keep[2]), O._addr(keep[3]), 0x88), np.array([0, 1]), wv),
             ((O._addr(keep[4]), O._addr(keep[5]), O._addr(keep[6]), O._addr(keep[7]), 0), np.array([1]), wv[:1])]
    out = np.zeros((2, C.LAYER_F16["H"]), np.float32)
    O.moe_q4(x[:2], items, C.LAYER_F16["H"], C.LAYER_F16["I"], 32, out)
    _close_rows(out, golden["moe_q4_mixed_out"], 1e-5)


@pytest.mark.parametrize("name", ["wide", "narrow", "zeros", "halfway"])
@pytest.mark.parametrize("wire", ["f16", "int8"])
def test_wire_rows_bit_exact(golden, name, wire):
    """The wire-format restatement against the reference's encode_rows /
    decode_rows (moelan/protocol.py:99-123): every byte and every decoded value."""
    a = C.wire_inputs()[name]
    q, s = O.encode_rows(a, wire)
    assert q.dtype == golden[f"wire_{name}_{wire}_q"].dtype
    assert np.array_equal(q.view(np.uint8), golden[f"wire_{name}_{wire}_q"].view(np.uint8))
    if wire == "int8":
        assert np.array_equal(s.view(np.uint32), golden[f"wire_{name}_{wire}_s"].view(np.uint32))
    dec = O.decode_rows(q, s)
    assert np.array_equal(dec.view(np.uint32), golden[f"wire_{name}_{wire}_dec"].view(np.uint32))


@pytest.mark.parametrize("case", C.GROUPED_CASES, ids=[c[0] for c in C.GROUPED_CASES])
def test_grouped_router_bit_exact(golden, case):
    """DeepSeek grouped routing restated in numpy against moelan's route_grouped."""
    name, T, E, k, scoring, method, ng, tg, norm, scale, with_bias, seed = case
    lg, bias = C.grouped_inputs(T, E, with_bias, seed)
    idx, w, _ = O.route_grouped(lg, k, scoring, method, ng, tg, norm, scale, bias)
    assert np.array_equal(idx, golden[f"grouped_{name}_idx"])
    assert np.array_equal(w.view(np.uint32), golden[f"grouped_{name}_w"].view(np.uint32))


@pytest.mark.parametrize("name", ["hf", "wide"])
@pytest.mark.parametrize("eps", [0.01, 0.1])
def test_sparsemixer_bit_exact(golden, name, eps):
    lg = C.sparsemixer_inputs()[name]
    idx, w = O.route_sparsemixer(lg, eps)
    assert np.array_equal(idx, golden[f"sparse_{name}_{eps}_idx"])
    assert np.array_equal(w.view(np.uint32), golden[f"sparse_{name}_{eps}_w"].view(np.uint32))
