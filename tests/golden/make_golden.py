"""Generate ``golden.npz``: outputs of the reference (moelan) on the seeded
inputs of ``cases.py``.

Run in the build container, where the reference's source tree is mounted:

    python tests/golden/make_golden.py /path/to/reference

It imports moelan from that tree with numba on and MOELAN_INT8_ACT=0 (the
exact float kernels), and checks the reference's GGUF block decoders against
gguf-py while it is at it, as the reference's own test does.  The GPU box
never runs this script; the tests only read ``golden.npz``.
"""

from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba-golden-"))
    os.environ["MOELAN_INT8_ACT"] = "0"
    sys.path.insert(0, ref_root)
    sys.path.insert(0, str(HERE))
    import numpy as np
    import cases as C
    from moelan import kernels, model
    from moelan.experts import Expert, ExpertStore, GroupQuant, Packed4
    from moelan.gguf import QuantMatrix, Stacked, dequantize

    assert kernels.ENABLED and not kernels.INT8_ACT
    g = {}

    # router: the reference's known answer (tests/test_moelan.py:64-71) and random cases
    lg = np.array([[0.0, 3.0, 1.0, 2.0], [5.0, 0.0, 0.0, 4.0]], np.float32)
    idx, w = model.route(lg, 2, True)
    g["router_known_logits"], g["router_known_idx"], g["router_known_w"] = lg, idx, w
    for name, T, E, k, norm, seed in C.ROUTER_CASES:
        lg = C.router_logits(T, E, seed)
        idx, w = model.route(lg, k, norm)
        ex, off, rows, wts = model.group_by_expert(idx, w)
        g[f"{name}_idx"], g[f"{name}_w"] = idx, w
        g[f"{name}_experts"], g[f"{name}_offsets"], g[f"{name}_rows"], g[f"{name}_weights"] = ex, off, rows, wts

    # int4 / int8 dequantisation
    raw, s = C.q4_deq_inputs()
    gs = C.Q4_DEQ["gs"]
    for off in (False, True):
        r = np.bitwise_xor(raw, 0x88) if off else raw
        out = np.empty((raw.shape[0], 2 * raw.shape[1]), np.float32)
        g[f"q4_deq_off{int(off)}"] = kernels.q4_dequant(r, s, gs, off, out).copy()
    q, s8 = C.q8_deq_inputs()
    out = np.empty(q.shape, np.float32)
    g["q8_deq"] = kernels.q8_dequant(q, s8, C.Q8_DEQ["gs"], out).copy()

    # GGUF block decoders (and gguf-py, as tests/test_gguf.py:25-33 checks)
    import gguf as gpy
    for qt in sorted(C.GGUF_BLOCK):
        raw = C.gguf_deq_inputs(qt)
        got = dequantize(raw, qt, C.GGUF_COLS)
        want = gpy.quants.dequantize(raw.copy(), gpy.GGMLQuantizationType(qt)).astype(np.float32).reshape(
            raw.shape[0], C.GGUF_COLS)
        ok = np.isfinite(want)
        assert np.array_equal(np.isfinite(got), ok) and np.array_equal(got[ok], want[ok]), qt
        g[f"gguf_deq_{qt}"] = got
        for rows in C.GGUF_MM_ROWS:
            raw2, x = C.gguf_mm_inputs(qt, rows)
            g[f"gguf_mm_{qt}_{rows}"] = kernels.gguf_matmul_t(x, raw2, qt, C.GGUF_COLS)

    # int4 matmul known answer (tests/test_moelan.py:245-258)
    for rows in C.MATMUL_ROWS:
        raw, s, W, x = C.q4_mm_inputs(rows)
        p = Packed4(raw, s, 32, (96, 128))
        g[f"q4_mm_{rows}"] = p.matmul_t(x)
        g[f"q4_mm_res_{rows}"] = p.resident().matmul_t(x)
        if rows == 1:
            g["q4_mm_dequant"] = p.dequant()

    class MemSource:
        zero_copy = False

        def __init__(self, ex):
            self.ex = ex

        def has(self, key):
            return key[1] in self.ex

        def load(self, key):
            return self.ex[key[1]]

    def run_layer(name, cfg, experts_obj, fmt, x, router):
        logits = x @ router.T
        idx, w = model.route(logits, cfg["k"], True)
        ex, off, rows, wts = model.group_by_expert(idx, w)
        groups = [(ex[i], rows[off[i]:off[i + 1]], wts[off[i]:off[i + 1]]) for i in range(len(ex))]
        store = ExpertStore([MemSource(experts_obj)], fmt=fmt)
        out = store.compute(0, x, groups)
        g[f"{name}_logits"], g[f"{name}_idx"], g[f"{name}_w"], g[f"{name}_out"] = logits, idx, w, out

    def q4_experts(experts, cfg, resident_every=0):
        H, I, gsz = cfg["H"], cfg["I"], cfg["gs"]
        obj = {}
        for e, (gr, gsc, dr, dsc) in experts.items():
            ex = Expert(Packed4(gr, gsc, gsz, (2 * I, H)), Packed4(dr, dsc, gsz, (H, I)), I)
            if resident_every and e % resident_every == 1:
                ex = Expert(ex.gu.resident(), ex.down.resident(), I)
            obj[e] = ex
        return obj

    x, router, experts = C.layer_inputs(C.LAYER, "int4")
    run_layer("layer_q4", C.LAYER, q4_experts(experts, C.LAYER, resident_every=3), "int4", x, router)
    x, router, experts = C.layer_inputs(C.LAYER_F16, "int4", f16_scales=True)
    run_layer("layer_q4h", C.LAYER_F16, q4_experts(experts, C.LAYER_F16), "int4", x, router)

    x, router, experts = C.layer_inputs(C.LAYER_Q8, "int8")
    H, I, gsz = C.LAYER_Q8["H"], C.LAYER_Q8["I"], C.LAYER_Q8["gs"]
    obj = {e: Expert(GroupQuant(q1, s1, gsz), GroupQuant(q2, s2, gsz), I) for e, (q1, s1, q2, s2) in experts.items()}
    run_layer("layer_q8", C.LAYER_Q8, obj, "int8", x, router)

    x, router, experts = C.layer_inputs(C.LAYER_GGUF, "gguf")
    H, I = C.LAYER_GGUF["H"], C.LAYER_GGUF["I"]
    obj = {e: Expert(Stacked(QuantMatrix(gr, 12, H), QuantMatrix(ur, 12, H)), QuantMatrix(dr, 8, I), I)
           for e, (gr, ur, dr) in experts.items()}
    run_layer("layer_gguf", C.LAYER_GGUF, obj, "native", x, router)

    # one fused moe_q4 call mixing raw and resident experts (tests/test_fused.py:57-74)
    x, router, experts = C.layer_inputs(C.LAYER_F16, "int4")
    obj = q4_experts(experts, C.LAYER_F16)
    a, b = obj[3], obj[6]
    b = Expert(b.gu.resident(), b.down.resident(), b.inter)
    wv = np.array([0.25, 0.75], np.float32)
    items = [(kernels.q4_expert_ptrs(a), np.array([0, 1]), wv), (kernels.q4_expert_ptrs(b), np.array([1]), wv[:1])]
    out = np.zeros((2, C.LAYER_F16["H"]), np.float32)
    kernels.moe_q4(x[:2], items, C.LAYER_F16["H"], C.LAYER_F16["I"], 32, out)
    g["moe_q4_mixed_out"] = out

    # activation rows in the wire formats (moelan/protocol.py:99-123)
    from moelan.protocol import decode_rows, encode_rows
    for name, a in C.wire_inputs().items():
        for wire in ("f16", "int8"):
            enc = encode_rows(a, wire, "x")
            g[f"wire_{name}_{wire}_q"] = enc["x"]
            if wire == "int8":
                g[f"wire_{name}_{wire}_s"] = enc["x_scale"]
            g[f"wire_{name}_{wire}_dec"] = decode_rows(enc, "x")

    # the other routers: DeepSeek grouped routing and PhiMoE's sparsemixer (moelan/model.py:170-223)
    import types
    for name, T, E, k, scoring, method, ng, tg, norm, scale, with_bias, seed in C.GROUPED_CASES:
        lg, bias = C.grouped_inputs(T, E, with_bias, seed)
        cfg = types.SimpleNamespace(scoring_func=scoring, topk_method=method, n_group=ng, topk_group=tg, top_k=k,
                                    norm_topk_prob=norm, routed_scaling_factor=scale)
        idx, w = model.route_grouped(lg, cfg, bias)
        g[f"grouped_{name}_idx"], g[f"grouped_{name}_w"] = idx, w
    for name, lg in C.sparsemixer_inputs().items():
        for eps in (0.01, 0.1):
            idx, w = model.route_sparsemixer(lg, eps)
            g[f"sparse_{name}_{eps}_idx"], g[f"sparse_{name}_{eps}_w"] = idx, w

    np.savez_compressed(HERE / "golden.npz", **g)
    print("wrote", HERE / "golden.npz", sum(v.nbytes for v in g.values()), "bytes (uncompressed)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python make_golden.py <moelan project root>")
    main(sys.argv[1])
