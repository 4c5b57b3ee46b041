"""The drop-in on CPU: packing of moelan's matrix objects into the tile
layout, and install() patching (it must refuse, patching nothing, without an
sm_100 device; with the device check bypassed it replaces exactly the
reference's expert entry points and uninstall() restores them)."""

import os
import sys
import types
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from distributedmoellm_b200 import layout as L  # noqa: E402
from distributedmoellm_b200 import synthetic as S  # noqa: E402
from distributedmoellm_b200.packing import pack_expert  # noqa: E402

NS = types.SimpleNamespace


def packed4(raw, s, gs, offset=False):
    return NS(raw=raw, s=s, gs=gs, offset=offset, shape=(raw.shape[0], raw.shape[1] * 2))


def test_pack_int4_expert_matches_the_tile_layout():
    rng = np.random.default_rng(0)
    gr, gsc, dr, dsc = S.int4_expert(rng, 256, 128, 32, f16_scales=False)
    p = pack_expert(NS(gu=packed4(gr, gsc, 32), down=packed4(dr, dsc, 32), inter=128))
    assert (p.fmt_gu, p.gs, p.H, p.I) == (L.FMT_Q4_F32, 32, 256, 128)
    assert np.array_equal(p.gu_tiles, L.q4_tiles(gr, gsc, 32, False, gu_inter=128))
    assert np.array_equal(p.dn_tiles, L.q4_tiles(dr, dsc, 32, False))
    assert p.eexp[0] == L.weight_exponent(gsc, 8)


def test_pack_int8_and_gguf_and_stacked():
    rng = np.random.default_rng(1)
    gq, gs_, dq, ds = S.int8_expert(rng, 256, 128, 32)
    p = pack_expert(NS(gu=NS(q=gq, s=gs_, gs=32), down=NS(q=dq, s=ds, gs=32), inter=128))
    assert p.fmt_gu == L.FMT_Q8_F32 and np.array_equal(p.dn_tiles, L.q8_tiles(dq, ds, 32))
    g = NS(raw=S.gguf_rows(rng, 128, 256, 8), qtype=8, shape=(128, 256))
    u = NS(raw=S.gguf_rows(rng, 128, 256, 8), qtype=8, shape=(128, 256))
    d = NS(raw=S.gguf_rows(rng, 256, 128, 8), qtype=8, shape=(256, 128))
    p = pack_expert(NS(gu=NS(parts=(g, u)), down=d, inter=128))
    q, sc = L.q8_0_as_q8(np.concatenate([g.raw, u.raw]), 256)
    assert p.fmt_gu == L.FMT_Q8_F16 and np.array_equal(p.gu_tiles, L.q8_tiles(q, sc, 32, gu_inter=128))
    q40 = NS(raw=S.gguf_rows(rng, 256, 128, 2), qtype=2, shape=(256, 128))
    gu40 = NS(raw=S.gguf_rows(rng, 256, 256, 2), qtype=2, shape=(256, 256))
    assert pack_expert(NS(gu=gu40, down=q40, inter=128)).fmt_down == L.FMT_Q4_F16


def test_pack_refuses_dense_and_takes_mixed_kinds():
    rng = np.random.default_rng(2)
    gr, gsc, dr, dsc = S.int4_expert(rng, 256, 128, 32, f16_scales=False)
    dense = NS(w=np.zeros((256, 128), np.float32))
    assert pack_expert(NS(gu=packed4(gr, gsc, 32), down=dense, inter=128)) is None
    gq, gs_, dq, ds = S.int8_expert(rng, 256, 128, 32)
    p = pack_expert(NS(gu=packed4(gr, gsc, 32), down=NS(q=dq, s=ds, gs=32), inter=128))
    assert (p.fmt_gu, p.fmt_down) == (L.FMT_Q4_F32, L.FMT_Q8_F32)
    q6k = NS(raw=S.gguf_rows(rng, 256, 256, 14), qtype=14, shape=(256, 256))
    assert pack_expert(NS(gu=q6k, down=q6k, inter=128)) is None


def test_pack_gguf_q4_k_reproduces_the_reference_weights():
    """Q4_K gate|up (Stacked) with a Q8_0 down, Mixtral-style: the affine
    int4 tiles hold exactly the reference's dequantised values."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    rng = np.random.default_rng(3)
    H, I = 512, 256
    g = NS(raw=S.gguf_rows(rng, I, H, 12), qtype=12, shape=(I, H))
    u = NS(raw=S.gguf_rows(rng, I, H, 12), qtype=12, shape=(I, H))
    d = NS(raw=S.gguf_rows(rng, H, I, 8), qtype=8, shape=(H, I))
    p = pack_expert(NS(gu=NS(parts=(g, u)), down=d, inter=I))
    assert (p.fmt_gu, p.fmt_down, p.H, p.I) == (L.FMT_Q4K_F32, L.FMT_Q8_F16, H, I)
    assert len(p.gu_tiles) == L.tiles_nbytes(L.FMT_Q4K_F32, 2 * I, H, gu_inter=I)
    nib, sc, bias = L.q4_k_as_affine(g.raw, H)
    w = ((nib.reshape(I, -1, 32).astype(np.float32) - 8) * sc[..., None] + bias[..., None]).reshape(I, H)
    assert np.array_equal(w, O.gguf_dequant(g.raw, 12, H))


def _fake_moelan():
    k = types.ModuleType("fake_moelan.kernels")
    a = types.ModuleType("fake_moelan.accel")
    from distributedmoellm_b200.dropin import ACCEL_NAMES, KERNEL_NAMES
    for n in KERNEL_NAMES:
        setattr(k, n, ("orig", n))
    for n in ACCEL_NAMES:
        setattr(a, n, ("orig", n))
    pkg = types.ModuleType("fake_moelan")
    pkg.kernels, pkg.accel = k, a
    return pkg


def test_install_refuses_without_a_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from distributedmoellm_b200.dropin import install
    pkg = _fake_moelan()
    with pytest.raises(RuntimeError):
        install(pkg)
    assert pkg.kernels.moe_q4 == ("orig", "moe_q4")


def test_install_patches_and_uninstall_restores(monkeypatch):
    from distributedmoellm_b200 import accel, device, kernels
    from distributedmoellm_b200.dropin import ACCEL_NAMES, KERNEL_NAMES, install, uninstall
    monkeypatch.setattr(device, "require_device", lambda: None)
    pkg = _fake_moelan()
    saved = install(pkg)
    for n in KERNEL_NAMES:
        assert getattr(pkg.kernels, n) is getattr(kernels, n)
    for n in ACCEL_NAMES:
        assert getattr(pkg.accel, n) is getattr(accel, n)
    uninstall(saved)
    assert pkg.kernels.moe_q4 == ("orig", "moe_q4") and pkg.accel.GpuTier == ("orig", "GpuTier")


# the reference source tree (moelan), when it is present: MOELAN_REF names its project root
REF = Path(os.environ.get("MOELAN_REF", "")) if os.environ.get("MOELAN_REF") else None


@pytest.mark.skipif(REF is None or not (REF / "moelan").is_dir(), reason="MOELAN_REF does not name the reference here")
def test_install_covers_the_reference_entry_points(monkeypatch):
    """Every name install() replaces exists in the reference's modules with
    the same parameters (so moelan's callers bind to ours unchanged)."""
    import inspect
    monkeypatch.setattr(sys, "dont_write_bytecode", True)       # nothing is written next to the reference
    monkeypatch.syspath_prepend(str(REF))
    monkeypatch.setenv("NUMBA_CACHE_DIR", "/tmp/numba_cache")
    mk = pytest.importorskip("moelan.kernels")
    ma = pytest.importorskip("moelan.accel")
    from distributedmoellm_b200 import accel, kernels
    from distributedmoellm_b200.dropin import ACCEL_NAMES, KERNEL_NAMES
    for mod, ours, names in ((mk, kernels, KERNEL_NAMES), (ma, accel, ACCEL_NAMES)):
        for n in names:
            ref = getattr(mod, n)
            mine = getattr(ours, n)
            rp = list(inspect.signature(ref).parameters)
            mp_ = list(inspect.signature(mine).parameters)
            assert mp_[:len(rp)] == rp, (n, rp, mp_)
    for m in ("expert_bytes", "add", "launch", "launch_held", "release", "collect", "calibrate", "stats"):
        assert list(inspect.signature(getattr(ma.GpuTier, m)).parameters) == \
            list(inspect.signature(getattr(accel.GpuTier, m)).parameters), m


def test_package_install_stays_callable(monkeypatch):
    """distributedmoellm_b200.install is the function on every call: the
    patching code lives in a submodule of another name, so importing it does
    not rebind the package attribute."""
    import distributedmoellm_b200 as mb
    from distributedmoellm_b200 import device
    monkeypatch.setattr(device, "require_device", lambda: None)
    for _ in range(2):
        pkg = _fake_moelan()
        saved = mb.install(pkg)
        assert callable(mb.install) and callable(mb.uninstall)
        mb.uninstall(saved)


def test_device_packing_bookkeeping_matches_the_host_layout():
    """packing.pack_expert_on lays experts out on the device; its formats,
    exponents and tile sizes (worked out on the host before the packers run)
    must be the host layout's, for every packed form."""
    from distributedmoellm_b200 import packing as P
    rng = np.random.default_rng(9)
    H, I = 256, 384
    gr, gsc, dr, dsc = S.int4_expert(rng, H, I, 32, f16_scales=False)
    cases = [NS(gu=packed4(gr, gsc, 32), down=packed4(dr, dsc, 32), inter=I),
             NS(gu=packed4(gr ^ 0x88, gsc.astype(np.float16), 32, offset=True),
                down=packed4(dr ^ 0x88, dsc.astype(np.float16), 32, offset=True), inter=I)]
    gq, gs_, dq, ds = S.int8_expert(rng, H, I, 64)
    cases.append(NS(gu=NS(q=gq, s=gs_, gs=64), down=NS(q=dq, s=ds, gs=64), inter=I))
    for qg, qd, Hm, Im in ((12, 8, 512, 512), (2, 2, 512, 512), (8, 8, 256, 256)):
        g = NS(raw=S.gguf_rows(rng, Im, Hm, qg), qtype=qg, shape=(Im, Hm))
        u = NS(raw=S.gguf_rows(rng, Im, Hm, qg), qtype=qg, shape=(Im, Hm))
        d = NS(raw=S.gguf_rows(rng, Hm, Im, qd), qtype=qd, shape=(Hm, Im))
        cases.append(NS(gu=NS(parts=(g, u)), down=d, inter=Im))
    for i, ex in enumerate(cases):
        want = P.pack_expert(ex)
        gu, dn = P._as_group_matrix(ex.gu), P._as_group_matrix(ex.down)
        (Og, Kg), (Od, Kd) = P._dims(gu), P._dims(dn)
        fg, eg, l1 = P._meta(gu, ex.inter)
        fd, ed, _ = P._meta(dn, 0)
        assert (fg, fd, Od, ex.inter) == (want.fmt_gu, want.fmt_down, want.H, want.I), i
        assert (eg, ed, L.act_exponent(l1, ex.inter)) == tuple(want.eexp), i
        assert L.tiles_nbytes(fg, Og, Kg, gu_inter=ex.inter) == want.gu_tiles.nbytes, i
        assert L.tiles_nbytes(fd, Od, Kd) == want.dn_tiles.nbytes, i
