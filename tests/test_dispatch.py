"""The layer's choice of kernels (layer.kernel_plan / run_experts), on CPU
with the device entry points replaced by recorders: every expert on the
decode mat-vecs below GEMM_MIN_ROWS (12) picks per expert on average, every expert
as a grouped GEMM from there on, for every weight format and size (affine
int4, K > 2048 included), never a split between the two."""

import sys
import types
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from distributedmoellm_b200 import layer as Lyr  # noqa: E402
from distributedmoellm_b200 import layout as L  # noqa: E402


def _experts(E=128, H=2048, I=768, fmt=L.FMT_Q4_F16):
    return types.SimpleNamespace(E=E, H=H, I=I, gs=32, fmt_gu=fmt, fmt_down=fmt, table=None, eexp=None,
                                 missing_exp=False)


def _run(monkeypatch, ex, P, picks=None, m=Lyr.GEMM_MIN_ROWS):
    calls = []
    monkeypatch.setattr(Lyr.D, "moe_decode", lambda *a, **k: calls.append(("decode", k.get("max_rows"))))
    monkeypatch.setattr(Lyr.D, "moe_prefill", lambda *a, **k: calls.append(("gemm", k.get("min_rows"))))
    monkeypatch.setattr(Lyr.D, "decode_workspace_bytes", lambda *a: 0)
    monkeypatch.setattr(Lyr.D, "prefill_workspace_bytes", lambda *a: 0)
    routing = types.SimpleNamespace(P=P)
    Lyr.run_experts(ex, None, None, routing, None, lambda name, n: None, None, m, picks=picks)
    return calls


@pytest.mark.parametrize("T,want", [
    (1, [("decode", 0)]),
    (64, [("decode", 0)]),       # 512 picks over 128 experts: 4 per expert
    (128, [("decode", 0)]),      # 1024 picks: 8 per expert
    (191, [("decode", 0)]),
    (192, [("gemm", 1)]),        # 1536 picks: 12 per expert
    (2048, [("gemm", 1)]),
])
def test_kernel_choice_by_batch(monkeypatch, T, want):
    assert _run(monkeypatch, _experts(), T * 8) == want


def test_affine_and_wide_experts_follow_the_batch(monkeypatch):
    # GGUF Q4_K (affine int4) and K > 2048 run on the decode kernels at decode sizes too
    assert _run(monkeypatch, _experts(fmt=L.FMT_Q4K_F32), 1) == [("decode", 0)]
    assert _run(monkeypatch, _experts(E=8, H=4096, I=14336, fmt=L.FMT_Q8_F16), 2) == [("decode", 0)]
    assert _run(monkeypatch, _experts(E=8, H=4096, I=14336, fmt=L.FMT_Q4K_F32), 1024) == [("gemm", 1)]


def test_expert_parallel_slice_decides_by_its_own_picks(monkeypatch):
    # a rank's 16 experts out of 128 see all ranks' picks in the routing; the choice follows its share
    ex = _experts(E=16)
    assert _run(monkeypatch, ex, 4096, picks=512) == [("gemm", 1)]    # 8 ranks x 64 tokens: 32 per expert
    assert _run(monkeypatch, ex, 4096, picks=191) == [("decode", 0)]  # below 12 per expert on average


def test_shapes_the_gemm_cannot_take_stay_on_decode(monkeypatch):
    assert _run(monkeypatch, _experts(H=1000), 65536) == [("decode", 0)]   # H % 128
    assert _run(monkeypatch, _experts(I=96), 65536) == [("decode", 0)]     # I % 64
    assert _run(monkeypatch, _experts(), 4096, m=0) == [("decode", 0)]     # gemm_min_rows=0


def test_experts_without_exponents_stay_on_the_decode_kernels(monkeypatch):
    # experts stored from raw tiles without the tensor-core exponents never reach the grouped GEMM
    ex = _experts(fmt=L.FMT_Q4K_F32)
    ex.missing_exp = {3}
    assert _run(monkeypatch, ex, 1) == [("decode", 0)]
    assert _run(monkeypatch, ex, 65536) == [("decode", 0)]


def test_largest_permutation_reaches_the_gemm(monkeypatch):
    # mb_permute takes up to 65536 picks (T=8192, k=8) and so does the grouped GEMM
    assert _run(monkeypatch, _experts(fmt=L.FMT_Q4K_F32), 65536) == [("gemm", 1)]
    assert _run(monkeypatch, _experts(), 65537) == [("decode", 0)]
