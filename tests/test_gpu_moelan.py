"""moelan itself with this library installed behind it (install()), on the GPU.

The reference is installed under baseline/_ref (pip install --target, no
dependencies: its stack is in the image), which travels with the repository
snapshot; these tests skip when it is absent.  They run moelan's own code
paths with the patched entry points:

* config 1 end to end: moelan's MoEModel on the tiny 4-layer model, greedy
  tokens identical to the reference's own run and logits within 1e-4
  (tests/golden/config1.npz, made by tests/golden/make_config1_golden.py),
  once through the patched kernels module and once with every expert on this
  library's GPU tier (MoEModel(gpu="cuda"), moelan/experts.py:755-795);
* ExpertStore.compute (moelan/experts.py:641-753) over groups of 1-3 rows
  (the fused moe_q4 call), 4-7 rows (per-expert mat-vecs) and 8 or more rows
  (dequantisation + BLAS), against the unpatched reference at 1e-5 per row;
* gguf.QuantMatrix.matmul_t (moelan/gguf.py:287-289) for K-quant matrices,
  which moelan sends to kernels.gguf_matmul_t below eight input rows.
"""

import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"

pytestmark = pytest.mark.gpu

TOL = 1e-5


def row_err(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float((np.abs(got - want).max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)).max())


@pytest.fixture(scope="module")
def moelan():
    if not (REF / "moelan").is_dir():
        pytest.skip("the reference is not installed under baseline/_ref")
    os.environ.setdefault("MOELAN_INT8_ACT", "0")
    os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba_"))
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import moelan as m
    import moelan.experts  # noqa: F401
    import moelan.gguf  # noqa: F401
    import moelan.model  # noqa: F401
    from distributedmoellm_b200 import _build, device
    _build.build()
    device.require_device()
    return m


@pytest.fixture
def installed(moelan):
    import distributedmoellm_b200 as mb
    saved = mb.install(moelan)
    yield moelan
    mb.uninstall(saved)


@pytest.fixture(scope="module")
def c1_golden():
    with np.load(ROOT / "tests" / "golden" / "config1.npz") as f:
        return {k: f[k] for k in f.files}


def _check_c1(toks, logits, golden):
    assert toks.tolist() == golden["tokens"].tolist()
    g = golden["logits"]
    assert np.abs(logits - g).max() <= 1e-4 * max(1.0, float(np.abs(g).max()))


def test_config1_generate_through_the_patched_kernels(installed, tmp_path, c1_golden):
    import config1 as C1
    from moelan.model import MoEModel
    model = MoEModel(C1.write_model(tmp_path))
    toks, logits = C1.greedy(model)
    _check_c1(toks, logits, c1_golden)


def test_config1_generate_with_every_expert_on_the_gpu_tier(installed, tmp_path, c1_golden):
    import config1 as C1
    from distributedmoellm_b200.accel import GpuTier
    from moelan.model import MoEModel
    model = MoEModel(C1.write_model(tmp_path), gpu="cuda", gpu_budget=1 << 30, gpu_mode="max")
    tier = model.backend.store.gpu
    assert isinstance(tier, GpuTier) and len(tier.experts) == C1.LAYERS * C1.EXPERTS
    toks, logits = C1.greedy(model)
    _check_c1(toks, logits, c1_golden)
    assert tier.calls > 0


def test_expert_store_compute_matches_the_reference(moelan, tmp_path):
    import config1 as C1
    import distributedmoellm_b200 as mb
    from moelan.model import MoEModel
    store = MoEModel(C1.write_model(tmp_path)).backend.store
    rng = np.random.default_rng(5)
    T = 40
    x = rng.standard_normal((T, C1.HIDDEN)).astype(np.float32)
    sizes = [1, 2, 3, 4, 5, 7, 8, 12, 1, 3, 6, 9, 2, 1, 4, 10]   # fused, per-expert and BLAS paths
    groups = [(e, np.sort(rng.choice(T, size=n, replace=False)), rng.random(n).astype(np.float32))
              for e, n in enumerate(sizes)]
    for layer in (0, 3):
        want = store.compute(layer, x, groups)
        saved = mb.install(moelan)
        try:
            got = store.compute(layer, x, groups)
        finally:
            mb.uninstall(saved)
        assert row_err(got, want) < TOL


@pytest.mark.parametrize("qtype", [12, 13, 14, 10, 11, 8])
def test_quant_matrix_matmul_t_for_k_quants(moelan, qtype):
    import cases as C
    import distributedmoellm_b200 as mb
    from moelan.gguf import QuantMatrix
    rng = np.random.default_rng(qtype)
    cols = 1024
    m = QuantMatrix(C.gguf_random_rows(64, cols, qtype, rng, 0.01), qtype, cols)
    for n in (1, 3, 7):
        x = rng.standard_normal((n, cols)).astype(np.float32)
        want = m.matmul_t(x)
        saved = mb.install(moelan)
        try:
            got = m.matmul_t(x)
        finally:
            mb.uninstall(saved)
        assert row_err(got, want) < TOL


@pytest.mark.parametrize("fmt", ["int4", "int8", "gguf:Q4_K,Q4_K,Q6_K"])
def test_bench_expert_runs_through_the_patched_kernels(installed, fmt):
    """moelan's node benchmark (moelan/experts.py:342-382) with install()
    active times this library: int4 through the patched moe_q4, int8 through
    q8_matmul_t, GGUF K-quants through gguf_matmul_t; and moelan.accel's
    bench_gpu is this library's (moelan/accel.py:400-411 keys)."""
    from moelan import accel
    from moelan.experts import bench_expert, synthetic_expert
    import distributedmoellm_b200.kernels as K
    calls = {"n": 0}
    for name in ("moe_q4", "q8_matmul_t", "gguf_matmul_t"):
        fn = getattr(installed.kernels, name)

        def counted(*a, _fn=fn, **k):
            calls["n"] += 1
            return _fn(*a, **k)
        setattr(installed.kernels, name, counted)
    try:
        ms = bench_expert(512, 256, fmt, gs=32, reps=8)
    finally:
        for name in ("moe_q4", "q8_matmul_t", "gguf_matmul_t"):
            setattr(installed.kernels, name, getattr(K, name))
    assert 0.0 < ms < 1000.0 and calls["n"] > 0
    if fmt == "int4":
        b = accel.bench_gpu("cuda", 1 << 28, 512, 256, "int4", 32)
        assert set(b) == {"gpu_ms", "gpu_experts", "gpu_name"} and b["gpu_experts"] > 0
    e = synthetic_expert(512, 256, fmt, 32)
    x = np.random.default_rng(3).standard_normal((2, 512)).astype(np.float32)
    assert np.isfinite(e(x)).all()
