"""The drop-in's host caches under concurrent callers, on CPU.

moelan calls its kernels module from several threads at once (the worker's
socketserver threads, the batcher thread, its BLAS pool; moelan/worker.py,
batching.py, experts.py:_POOL).  Here the device work is replaced by CPU
stand-ins that check what the caches hand them, and many threads call the
``kernels`` mirrors over more matrices and experts than the caches hold, so
entries are evicted while other threads use theirs."""

import sys
import threading
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from distributedmoellm_b200 import accel as A  # noqa: E402
from distributedmoellm_b200 import kernels as K  # noqa: E402
from distributedmoellm_b200 import packing as P  # noqa: E402
from distributedmoellm_b200 import synthetic as S  # noqa: E402


@pytest.fixture
def cpu_kernels(monkeypatch):
    monkeypatch.setattr(K, "_dev", lambda: torch.device("cpu"))
    monkeypatch.setattr(K, "_CACHE_MAX", 3)

    def fake_matmul(t, fmt, O, Kc, xd):          # marks the result with the cached matrix's identity
        return torch.full((xd.shape[0], O), float(t.numel() + O), dtype=torch.float32)

    def fake_gguf(t, qtype, cols, xd):
        return torch.full((xd.shape[0], t.shape[0]), float(t.numel() + qtype), dtype=torch.float32)

    def fake_compute(self, x, keys, rows, weights, gemm_min_rows=32):
        for k in keys:                            # every expert of the call is resident while it runs
            assert k in self.entries, k
        allr = np.concatenate([np.asarray(r) for r in rows])
        uniq = np.unique(allr)
        return uniq, torch.ones((len(uniq), x.shape[1])), torch.zeros(1, dtype=torch.int32)

    # the device packer's stand-in: the same tiles, laid out on the host
    monkeypatch.setattr(K, "pack_expert_on", lambda ex, dev, inter=None, max_bytes=None: P.pack_expert(ex, inter))
    # and for single matrices: the host layout's bytes as a (CPU) tensor
    monkeypatch.setattr(K.D, "pack_q4", lambda raw, sc, gs, offset, inter=0, out=None: torch.from_numpy(
        K.layout.q4_tiles(raw.numpy(), sc.numpy(), gs, offset, gu_inter=inter)))
    monkeypatch.setattr(K.D, "pack_q8", lambda q, sc, gs, inter=0, out=None: torch.from_numpy(
        K.layout.q8_tiles(q.numpy(), sc.numpy(), gs, gu_inter=inter)))
    monkeypatch.setattr(K.D, "matmul_t", fake_matmul)
    monkeypatch.setattr(K.D, "gguf_matmul_t", fake_gguf)
    monkeypatch.setattr(A.DevicePool, "compute", fake_compute)
    monkeypatch.setattr(A.DevicePool, "read_back", lambda self, part, status: (part.numpy(), int(status.item())))
    K._mats.clear()
    K._pool.clear()
    yield
    K._mats.clear()
    K._pool.clear()


def _run_threads(fn, n=8):
    errs = []

    def body(i):
        try:
            fn(i)
        except BaseException as e:      # noqa: BLE001
            errs.append(e)
    ts = [threading.Thread(target=body, args=(i,)) for i in range(n)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs, errs[0]


def test_matrix_cache_under_threads(cpu_kernels):
    rng = np.random.default_rng(0)
    mats = []
    for j in range(10):                           # more matrices than the cache holds (3)
        O, Kc = 16 * (j + 1), 64
        raw = np.frombuffer(rng.bytes(O * Kc // 2), np.uint8).reshape(O, Kc // 2).copy()
        s = rng.random((O, Kc // 32), dtype=np.float32)
        mats.append((raw, s))
    gg = S.gguf_rows(rng, 24, 256, 12)
    x = rng.standard_normal((2, 64), dtype=np.float32)
    xg = rng.standard_normal((2, 256), dtype=np.float32)

    def work(i):
        for it in range(60):
            j = (i * 7 + it) % len(mats)
            raw, s = mats[j]
            y = K.q4_matmul_t(x, raw, s, 32, False)
            tiles = K.layout.tiles_nbytes(K.layout.FMT_Q4_F32, raw.shape[0], 64)
            assert y.shape == (2, raw.shape[0]) and (y == tiles + raw.shape[0]).all()
            if it % 5 == 0:
                yg = K.gguf_matmul_t(xg, gg, 12, 256)
                assert (yg == gg.size + 12).all()
    _run_threads(work)
    assert len(K._mats) <= 3


def test_moe_q4_pool_under_threads(cpu_kernels):
    rng = np.random.default_rng(1)
    H, I, gs = 128, 64, 32
    experts = []
    for _ in range(8):                            # more experts than the pool keeps (3 unless a call needs more)
        gr, gsc, dr, dsc = S.int4_expert(rng, H, I, gs, f16_scales=False)
        experts.append((gr, np.ascontiguousarray(gsc), dr, np.ascontiguousarray(dsc)))
    ptrs = [tuple(a.__array_interface__["data"][0] for a in e) + (0x88,) for e in experts]
    x = rng.standard_normal((4, H), dtype=np.float32)

    def work(i):
        for it in range(30):
            picks = [(i + it + j) % len(experts) for j in range(2)]
            items = [(ptrs[e], np.array([j, 3]), np.ones(2, np.float32)) for j, e in enumerate(picks)]
            out = np.zeros((4, H), np.float32)
            K.moe_q4(x, items, H, I, gs, out)
            assert (out[[0, 1, 3]] == 1).all() and (out[2] == 0).all()
    _run_threads(work)
    pool, order = K._pool[None]
    assert len(order) == len(pool.entries) <= 3
