"""The ``--gpu cuda`` expert tier of moelan on B200: packed experts on the
device, computed by this library's kernels.

Drop-in for moelan/accel.py:75-188 (``GpuTier``) and 400-411 (``bench_gpu``):
same constructor, methods, attributes and ``stats()`` keys, so moelan's
ExpertStore (experts.py:641-670, 755-795), coordinator and worker use it
unchanged.  Differences, by design: experts stay packed (int4 / int8 / GGUF
Q8_0 and Q4_0 tiles, 2.65 MB for a Qwen3-30B int4 expert instead of 9.4 MB of
fp16), so ``add`` returns False for an expert with no packed form (dense f32
or 16-bit matrices), which then stays on the CPU as when the tier is full;
results are the f32 kernels' (exact products, f32 sums) for decode-sized
groups and the tensor-core grouped GEMMs (2e-3) for large ones.  Only CUDA
devices of compute capability 10.0 are accepted.
"""

from __future__ import annotations

import threading
import time

import numpy as np
import torch

from . import device as D
from .layer import run_experts
from .packing import pack_expert


class _Set:
    """Experts of one signature (formats, group size, H, I) passed to the kernels."""

    def __init__(self, fmt_gu, fmt_down, gs, H, I, table, eexp):
        self.fmt_gu, self.fmt_down, self.gs, self.H, self.I = fmt_gu, fmt_down, gs, H, I
        self.table, self.eexp, self.E = table, eexp, table.shape[0]
        self.missing_exp = ()


class DevicePool:
    """Packed experts, each in its own device buffer (gate|up tiles, down tiles)."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.entries: dict = {}          # key -> (Packed, buffer, gu address, down address)
        self._ws: dict = {}
        self._ws_lock = threading.Lock()

    def put(self, key, packed) -> int:
        g = torch.from_numpy(np.ascontiguousarray(packed.gu_tiles))
        d = torch.from_numpy(np.ascontiguousarray(packed.dn_tiles))
        off = (g.numel() + 255) // 256 * 256
        buf = torch.empty(off + d.numel(), dtype=torch.uint8, device=self.device)
        buf[:g.numel()].copy_(g)
        buf[off:off + d.numel()].copy_(d)
        self.entries[key] = (packed, buf, buf.data_ptr(), buf.data_ptr() + off)
        return buf.numel()

    def pop(self, key) -> int:
        packed, buf, _, _ = self.entries.pop(key)
        return buf.numel()

    def workspace(self, name, nbytes):
        """A device buffer of at least nbytes, reused by later calls on this
        pool's stream order (the kernels of one call finish before the next
        call's reuse them: all run on the caller's current stream)."""
        with self._ws_lock:
            b = self._ws.get(name)
            if b is None or b.numel() < nbytes:
                b = self._ws[name] = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.device)
            return b

    def compute(self, x: torch.Tensor, keys, rows, weights, gemm_min_rows: int = 32):
        """Weighted expert outputs summed per input row: returns (unique rows,
        (U, H) device tensor) with sum_p w_p * expert_p(x[row_p]) for the picks
        (keys[i], rows[i][j], weights[i][j])."""
        H = x.shape[1]
        counts = np.array([len(r) for r in rows], np.int64)
        all_rows = np.concatenate([np.asarray(r, np.int64) for r in rows]) if len(rows) else np.zeros(0, np.int64)
        all_w = np.concatenate([np.asarray(w, np.float32) for w in weights]) if len(rows) else np.zeros(0, np.float32)
        uniq, uidx = np.unique(all_rows, return_inverse=True)
        P = len(all_rows)
        y = torch.empty((max(P, 1), H), dtype=torch.float32, device=self.device)
        row_exp = D.row_exponents(x)
        status = torch.zeros(1, dtype=torch.int32, device=self.device)     # this call's own status word
        # experts of one signature share a launch
        sigs: dict = {}
        for i, k in enumerate(keys):
            sigs.setdefault(self.entries[k][0].signature, []).append(i)
        base = np.concatenate([[0], np.cumsum(counts)])
        for sig, idx in sigs.items():
            table = np.array([[self.entries[keys[i]][2], self.entries[keys[i]][3]] for i in idx], np.int64)
            eexp = np.zeros((len(idx), 4), np.int32)
            eexp[:, :3] = [self.entries[keys[i]][0].eexp for i in idx]
            c = counts[idx]
            sel = np.concatenate([np.arange(base[i], base[i + 1]) for i in idx])
            dev = self.device
            r = D.Routing.from_plan(torch.from_numpy(c.astype(np.int32)).to(dev),
                                    torch.from_numpy(np.concatenate([[0], np.cumsum(c)]).astype(np.int32)).to(dev),
                                    torch.from_numpy(all_rows[sel].astype(np.int32)).to(dev))
            s = _Set(*sig, torch.from_numpy(table).to(dev), torch.from_numpy(eexp).to(dev))
            if len(sigs) == 1:       # one signature (the usual case): its picks are all picks, in order
                run_experts(s, x, row_exp, r, y, self.workspace, status, gemm_min_rows)
            else:
                ys = torch.empty((max(len(sel), 1), H), dtype=torch.float32, device=dev)
                run_experts(s, x, row_exp, r, ys, self.workspace, status, gemm_min_rows)
                y[torch.from_numpy(sel).to(dev)] = ys[:len(sel)]
        # per unique row, its picks in order: CSR for the weighted combine
        order = np.argsort(uidx, kind="stable")
        row_ptr = np.concatenate([[0], np.cumsum(np.bincount(uidx, minlength=len(uniq)))]).astype(np.int32)
        dev = self.device
        part = D.combine(y, torch.from_numpy(order.astype(np.int32)).to(dev),
                         torch.from_numpy(all_w[order]).to(dev), len(uniq), 1,
                         row_ptr=torch.from_numpy(row_ptr).to(dev)) if P else torch.zeros((0, H), device=dev)
        return uniq, part, status


def open_device(spec: str):
    """(torch, device, name) for a CUDA spec ("cuda", "cuda:N" or "auto"), or raise RuntimeError."""
    if not (spec == "auto" or spec.startswith("cuda")):
        raise RuntimeError(f"this GPU tier runs on CUDA (sm_100) devices only, not {spec!r}")
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available to this PyTorch")
    dev = torch.device("cuda" if spec == "auto" else spec)
    with torch.cuda.device(dev):
        D.require_device()
    return torch, dev, f"cuda: {torch.cuda.get_device_name(dev)} (packed experts, sm_100a kernels)"


class GpuTier:
    """Experts resident on one B200 in their packed formats (the interface of
    moelan.accel.GpuTier)."""

    def __init__(self, spec: str, budget_bytes: int):
        self.torch, self.device, self.name = open_device(spec)
        self.spec = spec
        self.budget = int(budget_bytes)
        self.pool = DevicePool(self.device)
        self.experts: dict = {}            # (layer, expert) -> Packed
        self.used = 0
        self.lock = threading.RLock()
        self.calls = 0
        self.busy_s = 0.0
        self.share = 0.0
        self.gpu_ms = self.cpu_ms = None
        self.status = 0

    def expert_bytes(self, inter: int, hidden: int) -> int:
        """Device bytes of one int4 group-32 expert with f32 scales (the
        largest int4 form), for budget planning."""
        from . import layout
        return (layout.tiles_nbytes(layout.FMT_Q4_F32, 2 * inter, hidden, gu_inter=inter)
                + layout.tiles_nbytes(layout.FMT_Q4_F32, hidden, inter))

    def __contains__(self, key) -> bool:
        return key in self.experts

    def add(self, key, expert) -> bool:
        """Upload one moelan Expert in its packed form.  False if the tier is
        full or the expert has no packed form (it then stays on the CPU)."""
        packed = pack_expert(expert)
        if packed is None or self.used + packed.nbytes > self.budget:
            return False
        with self.lock, torch.cuda.device(self.device):
            self.used += self.pool.put(key, packed)
            self.experts[key] = packed
        return True

    def launch(self, layer: int, x: np.ndarray, groups):
        """Queue the given (expert, rows, weights) on the GPU; returns a handle
        (the kernels run while the caller computes its CPU share)."""
        t0 = time.perf_counter()
        with self.lock, torch.cuda.device(self.device):
            xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(self.device)
            keys = [(layer, int(e)) for e, _, _ in groups]
            uniq, part, status = self.pool.compute(xd, keys, [r for _, r, _ in groups], [w for _, _, w in groups])
            self.calls += 1
        return uniq, part, status, t0

    def launch_held(self, layer: int, x: np.ndarray, groups):
        """Launch those of ``groups`` whose experts this GPU holds; returns
        (handle or None, the other groups).  Atomic with :meth:`release`."""
        with self.lock:
            on = [g for g in groups if (layer, int(g[0])) in self.experts]
            if not on:
                return None, groups
            return self.launch(layer, x, on), [g for g in groups if (layer, int(g[0])) not in self.experts]

    def release(self) -> None:
        """Free the GPU's memory; its experts are computed on the CPU from now on."""
        with self.lock:
            for k in list(self.experts):
                self.pool.pop(k)
            self.experts.clear()
            self.used = 0
        torch.cuda.empty_cache()

    def collect(self, handle, out: np.ndarray) -> None:
        """out[rows] += the launched groups' weighted outputs (waits for them);
        raises RuntimeError if a kernel reported a failure."""
        uniq, part, status, t0 = handle
        with torch.cuda.device(self.device):
            out[uniq] += part.cpu().numpy()
            st = int(status.item())
        self.busy_s += time.perf_counter() - t0
        if st:
            raise RuntimeError(f"GPU expert kernels reported status {st}")

    def calibrate(self, sample_expert, cpu_expert_fn, hidden: int, repeats: int = 12) -> float:
        """Time one expert on each device (1 input row, transfers included) and
        set ``share`` = cpu / (gpu + cpu), as moelan/accel.py:141-177 does."""
        if not self.add((-1, 0), sample_expert):
            raise RuntimeError("the sample expert has no packed form for this GPU tier")
        x = np.random.default_rng(0).standard_normal((1, hidden)).astype(np.float32)
        groups = [(0, np.array([0]), np.ones(1, np.float32))]

        def gpu_once():
            o = np.zeros_like(x)
            self.collect(self.launch(-1, x, groups), o)
        for _ in range(3):
            gpu_once()
            cpu_expert_fn(x)
        t0 = time.perf_counter()
        for _ in range(repeats):
            gpu_once()
        g = (time.perf_counter() - t0) / repeats
        t0 = time.perf_counter()
        for _ in range(repeats):
            cpu_expert_fn(x)
        c = (time.perf_counter() - t0) / repeats
        with self.lock:
            self.experts.pop((-1, 0))
            self.used -= self.pool.pop((-1, 0))
        self.calls = 0
        self.busy_s = 0.0
        self.gpu_ms, self.cpu_ms = g * 1000, c * 1000
        self.share = c / (g + c)
        return self.share

    def stats(self) -> dict:
        return {"device": self.name, "experts": len(self.experts), "used_bytes": self.used,
                "budget_bytes": self.budget, "share": round(self.share, 3),
                "gpu_ms_per_expert": self.gpu_ms, "cpu_ms_per_expert": self.cpu_ms,
                "calls": self.calls, "busy_s": round(self.busy_s, 3)}


def bench_gpu(spec: str, budget: int, hidden: int, inter: int, fmt: str, gs: int = 64, make_expert=None) -> dict:
    """GPU side of a node's speed benchmark (moelan/accel.py:400-411): ms per
    expert on the GPU (one input row, transfers included) and how many experts
    fit in ``budget``.  ``make_expert(hidden, inter, fmt, gs)`` defaults to
    moelan.experts.synthetic_expert."""
    if make_expert is None:
        from moelan.experts import synthetic_expert as make_expert
    tier = GpuTier(spec, budget)
    e = make_expert(hidden, inter, fmt, gs)
    tier.calibrate(e, lambda x: e(x), hidden)
    out = {"gpu_ms": tier.gpu_ms, "gpu_experts": int(budget // tier.expert_bytes(inter, hidden)),
           "gpu_name": tier.name}
    tier.release()
    return out
