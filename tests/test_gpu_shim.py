"""GPU tests of the drop-in (distributedmoellm_b200.kernels / accel): the
same calls moelan makes, on duck-typed stand-ins for its matrix objects
(Packed4, GroupQuant, gguf.QuantMatrix), checked against the CPU oracle.
Bars: dequantisation bit-exact; f32 mat-vec paths 1e-5 of each row's max."""

import types

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
NS = types.SimpleNamespace
TOL = 1e-5


@pytest.fixture(scope="module")
def K():
    from distributedmoellm_b200 import _build
    _build.build()
    from distributedmoellm_b200 import device, kernels
    device.require_device()
    return kernels


def row_err(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float((np.abs(got - want).max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)).max())


def packed4(raw, s, gs, offset=False):
    return NS(raw=np.ascontiguousarray(raw), s=np.ascontiguousarray(s), gs=gs, offset=offset,
              shape=(raw.shape[0], raw.shape[1] * 2))


class StandInExpert:
    """moelan's Expert as the tier sees it: gu, down, inter, and e(x) (the CPU forward)."""

    def __init__(self, gu, down, inter, desc):
        self.gu, self.down, self.inter, self.desc = gu, down, inter, desc

    def __call__(self, x):
        return O.expert_forward(x, *self.desc, self.inter)


def int4_expert(rng, H, I, gs=32, f16=False):
    from distributedmoellm_b200 import synthetic as S
    gr, gsc, dr, dsc = S.int4_expert(rng, H, I, gs, f16_scales=f16)
    desc = (("q4", gr, gsc.astype(np.float32), gs, False), ("q4", dr, dsc.astype(np.float32), gs, False))
    return StandInExpert(packed4(gr, gsc, gs), packed4(dr, dsc, gs), I, desc), desc


def test_dequant_entry_points_bit_exact(K):
    from distributedmoellm_b200 import synthetic as S
    rng = np.random.default_rng(0)
    gr, gsc, _, _ = S.int4_expert(rng, 256, 128, 32, f16_scales=False)
    out = np.empty((256, 256), np.float32)
    assert K.q4_dequant(gr, gsc, 32, False, out) is out
    assert np.array_equal(out.view(np.uint32), O.q4_dequant(gr, gsc, 32, False).view(np.uint32))
    q, s, _, _ = S.int8_expert(rng, 128, 128, 32)
    out8 = np.empty(q.shape, np.float32)
    K.q8_dequant(q, s, 32, out8)
    assert np.array_equal(out8, O.q8_dequant(q, s, 32))
    raw = S.gguf_rows(rng, 16, 512, 12)
    og = np.empty((16, 512), np.float32)
    K.gguf_dequant(raw, 12, og)
    assert np.array_equal(og, O.gguf_dequant(raw, 12, 512))


@pytest.mark.parametrize("n", [1, 3, 9])
def test_matmul_entry_points(K, n):
    from distributedmoellm_b200 import synthetic as S
    rng = np.random.default_rng(n)
    x = rng.standard_normal((n, 512), dtype=np.float32)
    gr, gsc, _, _ = S.int4_expert(rng, 512, 128, 32, f16_scales=False)
    assert row_err(K.q4_matmul_t(x, gr, gsc, 32, False), O.q4_matmul_t(x, gr, gsc, 32, False)) < TOL
    assert row_err(K.q4_matmul_t(x, gr, gsc, 32, False), O.q4_matmul_t(x, gr, gsc, 32, False)) < TOL   # cached
    q, s, _, _ = S.int8_expert(rng, 512, 128, 32)
    assert row_err(K.q8_matmul_t(x, q, s, 32), O.q8_matmul_t(x, q, s, 32)) < TOL
    for qt in (8, 2):
        raw = S.gguf_rows(rng, 96, 512, qt)
        assert row_err(K.gguf_matmul_t(x, raw, qt, 512), O.gguf_matmul_t(x, raw, qt, 512)) < TOL


@pytest.mark.parametrize("qt", [2, 3, 6, 7, 8, 10, 11, 12, 13, 14])
def test_gguf_matmul_t_takes_every_type(K, qt):
    """install() puts this in place of moelan.kernels.gguf_matmul_t, which
    moelan's QuantMatrix.matmul_t calls for every GGUF matrix with fewer than
    eight input rows (moelan/gguf.py:287-289): no type moelan reads may fail."""
    import cases as C
    rng = np.random.default_rng(100 + qt)
    raw = C.gguf_random_rows(48, 512, qt, rng, 0.01)
    for n in (1, 5):
        x = rng.standard_normal((n, 512), dtype=np.float32)
        w = O.gguf_dequant(raw, qt, 512).astype(np.float64)
        assert row_err(K.gguf_matmul_t(x, raw, qt, 512), x.astype(np.float64) @ w.T) < TOL
    # a Mixtral-wide Q8_0 down projection (K = 14336) as well
    if qt == 8:
        raw = C.gguf_random_rows(64, 14336, 8, rng, 0.001)
        x = rng.standard_normal((1, 14336), dtype=np.float32)
        w = O.gguf_dequant(raw, 8, 14336).astype(np.float64)
        assert row_err(K.gguf_matmul_t(x, raw, 8, 14336), x.astype(np.float64) @ w.T) < TOL


def test_moe_q4_matches_the_reference_kernel(K):
    rng = np.random.default_rng(7)
    H, I, gs, T = 512, 256, 32, 12
    experts = [int4_expert(rng, H, I, gs) for _ in range(5)]
    x = rng.standard_normal((T, H), dtype=np.float32)
    items = []
    for j, (e, desc) in enumerate(experts):
        rows = np.sort(rng.choice(T, size=2 + j, replace=False)).astype(np.int64)
        w = rng.random(len(rows), dtype=np.float32)
        ptrs = K.q4_expert_ptrs(e)
        assert ptrs is not None and ptrs[4] == 0x88
        items.append((ptrs, rows, w))
    out = rng.standard_normal((T, H), dtype=np.float32)
    want = out.copy()
    O.moe_q4(x, items, H, I, gs, want)
    for _ in range(2):              # the second call reuses the uploaded experts
        got = out.copy()
        K.moe_q4(x, items, H, I, gs, got)
        assert row_err(got, want) < TOL


def test_gpu_tier_launch_collect_and_stats():
    from distributedmoellm_b200.accel import GpuTier, bench_gpu
    rng = np.random.default_rng(11)
    H, I = 256, 256
    tier = GpuTier("cuda", 64 << 20)
    experts = {e: int4_expert(rng, H, I, f16=(e % 2 == 1)) for e in range(4)}
    for e, (ex, _) in experts.items():
        assert tier.add((3, e), ex)
    assert (3, 1) in tier and (4, 1) not in tier
    dense = NS(gu=NS(w=np.zeros((2 * I, H), np.float32)), down=NS(w=np.zeros((H, I), np.float32)), inter=I)
    assert not tier.add((3, 9), dense)
    x = rng.standard_normal((20, H), dtype=np.float32)
    groups = [(e, np.sort(rng.choice(20, size=3 + e, replace=False)), rng.random(3 + e, dtype=np.float32))
              for e in range(4)] + [(7, np.array([0, 1]), np.ones(2, np.float32))]
    handle, rest = tier.launch_held(3, x, groups)
    assert [g[0] for g in rest] == [7]
    # collect adds into out: seed it with values of the outputs' own size (1e-4), so that the
    # comparison is not swamped by the rounding of a large offset
    base = (rng.standard_normal((20, H), dtype=np.float32) * 1e-4).astype(np.float32)
    out = base.copy()
    tier.collect(handle, out)
    want = base.astype(np.float64)
    for e, rows, w in groups[:4]:
        want[rows] += O.expert_forward(x[rows], *experts[e][1], I) * w[:, None]
    assert row_err(out, want) < TOL
    st = tier.stats()
    assert set(st) == {"device", "experts", "used_bytes", "budget_bytes", "share", "gpu_ms_per_expert",
                       "cpu_ms_per_expert", "calls", "busy_s"}
    assert st["experts"] == 4 and st["calls"] == 1 and st["used_bytes"] == tier.used > 0
    tier.release()
    assert tier.used == 0 and not tier.experts
    share = tier.calibrate(experts[0][0], lambda xx: O.expert_forward(xx, *experts[0][1], I), H)
    assert 0.0 < share < 1.0 and tier.used == 0
    b = bench_gpu("cuda", 1 << 30, H, I, "int4", 32, make_expert=lambda h, i, f, g: int4_expert(rng, h, i, g)[0])
    assert b["gpu_experts"] > 0 and b["gpu_ms"] > 0


def _gguf_expert(rng, H, I, qt_gu, qt_dn):
    from distributedmoellm_b200 import synthetic as S
    g = NS(raw=S.gguf_rows(rng, I, H, qt_gu), qtype=qt_gu, shape=(I, H))
    u = NS(raw=S.gguf_rows(rng, I, H, qt_gu), qtype=qt_gu, shape=(I, H))
    d = NS(raw=S.gguf_rows(rng, H, I, qt_dn), qtype=qt_dn, shape=(H, I))
    return NS(gu=NS(parts=(g, u)), down=d, inter=I)


def test_experts_laid_out_on_the_device_match_the_host_layout(K):
    """packing.pack_expert_on (the GPU tier's and moe_q4's upload: moelan's
    bytes to the device, laid out there by mb_pack_*) gives the bytes and
    exponents of the host layout (packing.pack_expert) for every packed form."""
    import torch

    from distributedmoellm_b200 import synthetic as S
    from distributedmoellm_b200.packing import pack_expert, pack_expert_on
    rng = np.random.default_rng(23)
    H, I = 256, 384
    cases = [int4_expert(rng, H, I, 32)[0], int4_expert(rng, H, I, 64, f16=True)[0]]
    gr, gsc, dr, dsc = S.int4_expert(rng, H, I, 32, f16_scales=False)
    cases.append(NS(gu=packed4(gr ^ 0x88, gsc, 32, offset=True), down=packed4(dr ^ 0x88, dsc, 32, offset=True),
                    inter=I))
    gq, gs8, dq, ds8 = S.int8_expert(rng, H, I, 64)
    cases.append(NS(gu=NS(q=gq, s=gs8, gs=64), down=NS(q=dq, s=ds8, gs=64), inter=I))
    cases += [_gguf_expert(rng, 512, 512, 12, 8), _gguf_expert(rng, 512, 512, 2, 2), _gguf_expert(rng, 256, 256, 8, 8)]
    for i, ex in enumerate(cases):
        want = pack_expert(ex)
        got = pack_expert_on(ex, "cuda")
        assert want is not None and got is not None, i
        assert got.signature == want.signature and tuple(got.eexp) == tuple(want.eexp), i
        torch.cuda.synchronize()
        assert np.array_equal(got.gu_tiles.cpu().numpy(), want.gu_tiles), i
        assert np.array_equal(got.dn_tiles.cpu().numpy(), want.dn_tiles), i
        assert got.buf.numel() == got.dn_offset + want.dn_tiles.nbytes and got.dn_offset % 256 == 0
        assert pack_expert_on(ex, "cuda", max_bytes=got.buf.numel() - 1) is None
    dense = NS(gu=NS(w=np.zeros((2 * I, H), np.float32)), down=NS(w=np.zeros((H, I), np.float32)), inter=I)
    assert pack_expert_on(dense, "cuda") is None
