"""Expert parallelism on CPU: world_size-2 gloo ranks run the exchange plan
of distributedmoellm_b200.ep.EPLayer (the same code the NCCL ranks run) with
compute operations from the CPU oracle, and each rank's output must equal
the oracle's one-process MoE layer over that rank's tokens.  Also: the
regrouping plan, and a rank that fails before the first collective (the
other rank gets an error from its collective within the process group's
timeout instead of waiting for ever).  Mirrors the reference's "distributed
= local" tests (tests/test_moelan.py:130-154)."""

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]

E, H, I, K, GS = 8, 128, 128, 2, 32


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _experts():
    sys.path[:0] = [str(ROOT), str(ROOT / "oracle"), str(ROOT / "tests" / "golden")]
    from distributedmoellm_b200 import synthetic as S
    rng = np.random.default_rng(5)
    desc = {}
    for e in range(E):
        gr, gsc, dr, dsc = S.int4_expert(rng, H, I, GS, f16_scales=False)
        desc[e] = (("q4", gr, gsc, GS, False), ("q4", dr, dsc, GS, False))
    router = (rng.standard_normal((E, H), dtype=np.float32)).astype(np.float32)
    return desc, router


class OracleOps:
    """EPLayer's compute operations on the CPU oracle (test infrastructure)."""

    def __init__(self, desc, router, first_expert, k):
        import oracle as O
        import torch
        self.O, self.torch = O, torch
        self.desc, self.router, self.first, self.k = desc, router, first_expert, k
        self.device = torch.device("cpu")

    def route(self, x):
        O, torch = self.O, self.torch
        xn = x.numpy()
        idx, w = O.route(xn @ self.router.T, self.k, True)
        flat = idx.reshape(-1)
        order = np.argsort(flat, kind="stable")
        inv = np.empty_like(order)
        inv[order] = np.arange(len(order))
        counts = np.bincount(flat, minlength=len(self.router)).astype(np.int32)
        return (torch.from_numpy(w.reshape(-1).astype(np.float32)), torch.from_numpy(counts),
                torch.from_numpy((order // self.k).astype(np.int32)), torch.from_numpy(inv.astype(np.int32)))

    def gather_rows(self, src, index):
        return src[index.long()].contiguous()

    def experts(self, xr, counts, offsets, sorted_rows):
        O, torch = self.O, self.torch
        x, off, rows = xr.numpy(), offsets.numpy(), sorted_rows.numpy()
        y = np.zeros((len(rows), x.shape[1]), np.float32)
        for j in range(len(counts)):
            seg = rows[off[j]:off[j + 1]]
            if len(seg):
                gu, dn = self.desc[self.first + j]
                y[off[j]:off[j + 1]] = O.expert_forward(x[seg], gu, dn, I)
        return torch.from_numpy(y)

    def combine(self, y, inv, w, T, k):
        torch = self.torch
        yn, iv, wn = y.numpy(), inv.numpy(), w.numpy()
        out = np.zeros((T, yn.shape[1]), np.float32)
        for j in range(k):
            out += wn[j::k, None] * yn[iv[j::k]]
        return torch.from_numpy(out)


def _worker(rank, world, port, q, fail_rank):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch.distributed as dist
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
        desc, router = _experts()
        import oracle as O
        import torch
        from distributedmoellm_b200.ep import EPLayer
        x = np.random.default_rng(100 + rank).standard_normal((24 + 5 * rank, H), dtype=np.float32)
        layer = EPLayer(None, E, K, H)
        layer.ops = OracleOps(desc, router, layer.first_expert, K)
        if rank == fail_rank:
            q.put((rank, "raised", ""))
            raise SystemExit(0)        # leaves before any collective, as a crashed rank would
        try:
            out = layer(torch.from_numpy(x)).numpy()
        except Exception as exc:       # the peer is gone: the collective must fail, not hang
            q.put((rank, "error", type(exc).__name__))
            return
        want = O.moe_layer(x, router, desc, K, True, I)[0]
        err = float((np.abs(out - want).max(axis=1) / np.abs(want).max(axis=1)).max())
        q.put((rank, "ok", err))
        dist.destroy_process_group()
    except SystemExit:
        pass
    except Exception as exc:           # report instead of dying silently
        q.put((rank, "exception", repr(exc)))


def _run(world, fail_rank=-1, timeout=120):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, kind, val = q.get(timeout=timeout)
            res[r] = (kind, val)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return res


def test_local_plan_regroups_by_local_expert():
    sys.path.insert(0, str(ROOT))
    from distributedmoellm_b200.ep import local_plan
    rng = np.random.default_rng(0)
    for _ in range(20):
        G, El = int(rng.integers(1, 5)), int(rng.integers(1, 6))
        rec = rng.integers(0, 4, size=(G, El))
        counts, offsets, rows, inv = local_plan(rec)
        assert np.array_equal(counts, rec.sum(axis=0))
        assert sorted(rows.tolist()) == list(range(int(rec.sum())))
        assert np.array_equal(inv[rows], np.arange(len(rows)))
        # receive buffer: source-major, expert-minor; local order: expert-major, source-minor
        src_expert = [(s, j) for s in range(G) for j in range(El) for _ in range(rec[s, j])]
        got = [src_expert[p] for p in rows]
        want = [(s, j) for j in range(El) for s in range(G) for _ in range(rec[s, j])]
        assert got == want


def test_oracle_receive_plan_is_the_local_plan_grouping():
    """The peer-memory dispatch's receive order (the oracle's
    ep_receive_plan: by local expert, then source rank, then the source's
    grouping order) is the order local_plan gives the all-to-all's receive
    buffer (source-major) once regrouped."""
    sys.path.insert(0, str(ROOT))
    import oracle as O
    from distributedmoellm_b200.ep import local_plan
    rng = np.random.default_rng(1)
    for _ in range(10):
        G = int(rng.choice([1, 2, 4]))
        El, T = int(rng.integers(1, 4)), int(rng.integers(0, 20))
        Etot = G * El
        k = min(2, Etot)
        idx = [np.stack([rng.choice(Etot, size=k, replace=False) for _ in range(T)]).astype(np.int32)
               if T else np.zeros((0, k), np.int32) for _ in range(G)]
        # each source's grouping order: by expert, ties by pick index (a stable sort)
        order = []
        for s in range(G):
            flat = idx[s].reshape(-1)
            srt = np.argsort(flat, kind="stable")
            inv = np.empty_like(srt)
            inv[srt] = np.arange(len(srt))
            order.append(inv)
        plans = O.ep_receive_plan(idx, order, Etot)
        for d in range(G):
            rows, counts = plans[d]
            rec = np.array([[int((idx[s].reshape(-1) == d * El + j).sum()) for j in range(El)] for s in range(G)])
            lc, lo, sorted_rows, inv = local_plan(rec)
            assert counts.tolist() == lc.tolist()
            # the all-to-all receive buffer: source after source, each source's rows in its grouping order
            buf = []
            for s in range(G):
                flat = idx[s].reshape(-1)
                mine = [p for p in np.argsort(order[s], kind="stable") if d * El <= flat[p] < (d + 1) * El]
                buf.extend((s, int(p)) for p in mine)
            assert [buf[q] for q in sorted_rows] == rows


def test_ep_two_gloo_ranks_match_the_oracle():
    res = _run(2)
    for r in range(2):
        kind, err = res[r]
        assert kind == "ok", res
        assert err < 1e-5, res


def test_ep_four_gloo_ranks_match_the_oracle():
    """Four ranks (two experts each here): uneven token counts per rank, every
    rank's experts fed by all four."""
    assert E % 4 == 0
    res = _run(4)
    for r in range(4):
        kind, err = res[r]
        assert kind == "ok", res
        assert err < 1e-5, res


def test_ep_rank_failure_surfaces_as_an_error():
    res = _run(2, fail_rank=1)
    assert res[1][0] == "raised", res
    assert res[0][0] in ("error", "exception"), res


def test_device_ops_expose_every_operation_ep_uses():
    sys.path.insert(0, str(ROOT))
    import torch
    from distributedmoellm_b200.ep import DeviceOps
    ops = DeviceOps(torch.zeros((E, H)), object(), E, K)
    for name in ("route", "gather_rows", "experts", "combine"):
        assert callable(getattr(ops, name)), name
    assert ops.device == torch.device("cpu")
