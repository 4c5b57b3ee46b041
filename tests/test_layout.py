"""The device tile layout (host logic, no GPU): decoding the tile bytes back
with numpy gives the reference's dequantised weights, for every format and
for gate|up interleaving and padding."""

import numpy as np
import pytest

import oracle as O
from distributedmoellm_b200 import layout as L


def untile(buf, fmt, O_rows, K, gu_inter=0):
    """Inverse of layout.q4_tiles / q8_tiles -> (O_rows, K) f32 weights."""
    order = L.row_order(O_rows, gu_inter)
    Kp = (K + 127) // 128 * 128
    NQ, RT = Kp // 128, len(order) // 16
    bb = L.block_bytes(fmt)
    blk = buf.reshape(RT, NQ, bb)
    data_b = 2048 if L.is_q8(fmt) else 1024
    sdt = np.float16 if L.scale_is_f16(fmt) else np.float32
    sc = np.ascontiguousarray(blk[:, :, data_b:]).view(sdt).reshape(RT, NQ, 16, 4).astype(np.float32)
    sc = sc.transpose(0, 2, 1, 3).reshape(RT * 16, NQ * 4)                   # (rows, groups)
    if L.is_q8(fmt):
        v = blk[:, :, :data_b].reshape(RT, NQ, 2, 16, 4, 2, 8)               # (rt, q, half, row, t, gpos, 8)
        v = v.transpose(0, 3, 1, 2, 5, 4, 6)                                  # (rt, row, q, half, gpos, t, 8)
        inv = np.argsort([0, 4, 1, 5, 2, 6, 3, 7])
        v = v[..., inv].reshape(RT * 16, Kp).astype(np.int32) - 128
    else:
        nib = blk[:, :, :data_b].reshape(RT, NQ, 16, 4, 4, 4)                # (rt, q, row, t, group, byte)
        nib = nib.transpose(0, 2, 1, 4, 3, 5).reshape(RT * 16, Kp // 2)       # (rows, bytes)
        v = np.empty((RT * 16, Kp), np.int32)
        v[:, 0::2] = (nib & 15).astype(np.int32) - 8
        v[:, 1::2] = (nib >> 4).astype(np.int32) - 8
    w = v.reshape(RT * 16, Kp // 32, 32).astype(np.float32) * sc[:, :, None]
    w = w.reshape(RT * 16, Kp)
    out = np.zeros((O_rows, K), np.float32)
    ok = order >= 0
    out[order[ok]] = w[ok, :K]
    return out, w, order


@pytest.mark.parametrize("O_rows,K,gs", [(64, 256, 32), (48, 384, 64), (20, 160, 32)])
@pytest.mark.parametrize("f16", [False, True])
@pytest.mark.parametrize("offset", [False, True])
def test_q4_tiles_roundtrip(O_rows, K, gs, f16, offset):
    rng = np.random.default_rng(O_rows + K)
    raw = rng.integers(0, 256, (O_rows, K // 2), dtype=np.uint8)
    s = rng.random((O_rows, K // gs), dtype=np.float32).astype(np.float16 if f16 else np.float32)
    fmt = L.fmt_of("q4", s)
    buf = L.q4_tiles(raw, s, gs, offset)
    assert buf.size == L.tiles_nbytes(fmt, O_rows, K)
    got, w, order = untile(buf, fmt, O_rows, K)
    want = O.q4_dequant(raw, s.astype(np.float32), gs, offset)
    assert np.array_equal(got, want)
    assert not w[order < 0].any() and not w[:, K:].any()            # padding is zero


@pytest.mark.parametrize("I,H,gs", [(24, 256, 32), (20, 128, 32)])
def test_q4_gate_up_interleave(I, H, gs):
    rng = np.random.default_rng(5)
    raw = rng.integers(0, 256, (2 * I, H // 2), dtype=np.uint8)
    s = rng.random((2 * I, H // gs), dtype=np.float32)
    buf = L.q4_tiles(raw, s, gs, False, gu_inter=I)
    got, w, order = untile(buf, L.FMT_Q4_F32, 2 * I, H, gu_inter=I)
    assert np.array_equal(got, O.q4_dequant(raw, s, gs, False))
    tiles = order.reshape(-1, 16)
    assert (tiles[:, :8][tiles[:, :8] >= 0] < I).all() and (tiles[:, 8:][tiles[:, 8:] >= 0] >= I).all()
    assert np.array_equal(tiles[:, 8:][tiles[:, 8:] >= 0] - I, tiles[:, :8][tiles[:, :8] >= 0])


@pytest.mark.parametrize("O_rows,K,gs,f16,inter", [(64, 256, 32, False, 0), (32, 512, 64, True, 0),
                                                   (48, 256, 32, False, 24)])
def test_q8_tiles_roundtrip(O_rows, K, gs, f16, inter):
    rng = np.random.default_rng(K)
    q = rng.integers(-128, 128, (O_rows, K), dtype=np.int8)
    s = rng.random((O_rows, K // gs), dtype=np.float32).astype(np.float16 if f16 else np.float32)
    fmt = L.fmt_of("q8", s)
    buf = L.q8_tiles(q, s, gs, gu_inter=inter)
    assert buf.size == L.tiles_nbytes(fmt, O_rows, K, gu_inter=inter)
    got, _, _ = untile(buf, fmt, O_rows, K, gu_inter=inter)
    assert np.array_equal(got, O.q8_dequant(q, s.astype(np.float32), gs))


def test_gguf_q8_0_and_q4_0_map_onto_tiles():
    import cases as C
    rng = np.random.default_rng(9)
    raw = C.gguf_random_rows(16, 256, 8, rng)
    q, d = L.q8_0_as_q8(raw, 256)
    assert np.array_equal(O.q8_dequant(q, d.astype(np.float32), 32), O.gguf_dequant(raw, 8, 256))
    raw = C.gguf_random_rows(16, 256, 2, rng)
    u, d = L.q4_0_as_q4(raw, 256)
    assert np.array_equal(O.q4_dequant(u, d.astype(np.float32), 32, True), O.gguf_dequant(raw, 2, 256))


def test_bad_group_size_is_refused():
    with pytest.raises(ValueError):
        L.q4_tiles(np.zeros((16, 64), np.uint8), np.ones((16, 8), np.float32), 16)
