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
from .layer import GEMM_MIN_ROWS, run_experts
from .packing import pack_expert, pack_expert_on


_TORCH_DTYPE = {"<i4": torch.int32, "<i8": torch.int64, "<f4": torch.float32}


class _Set:
    """Experts of one signature (formats, group size, H, I) passed to the kernels."""

    def __init__(self, fmt_gu, fmt_down, gs, H, I, table, eexp):
        self.fmt_gu, self.fmt_down, self.gs, self.H, self.I = fmt_gu, fmt_down, gs, H, I
        self.table, self.eexp, self.E = table, eexp, table.shape[0]
        self.missing_exp = ()


class DevicePool:
    """Packed experts, each in its own device buffer (gate|up tiles, down tiles)."""

    def __init__(self, device):
        d = torch.device(device)
        if d.type == "cuda" and d.index is None:      # "cuda": the current device, by its index
            d = torch.device("cuda", torch.cuda.current_device())
        self.device = d
        self.entries: dict = {}          # key -> (Packed, buffer, gu address, down address)
        self._ws: dict = {}
        self._ws_lock = threading.Lock()
        self._pin = None            # pinned staging buffer of compute()'s routing arrays, and its device twin
        self._dev_stage = None
        self._stage_done = None     # recorded after the last copy out of the pinned buffer
        self._result = None         # pinned buffer a caller reads results back through (result_buffer)

    def put(self, key, packed) -> int:
        buf = getattr(packed, "buf", None)
        if buf is not None:      # laid out on this device already (packing.pack_expert_on)
            if buf.device != self.device:
                raise ValueError(f"expert {key} was packed on {buf.device}, this pool is on {self.device}")
            self.entries[key] = (packed, buf, buf.data_ptr(), buf.data_ptr() + packed.dn_offset)
            return buf.numel()
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

    def read_back(self, part: torch.Tensor, status: torch.Tensor):
        """(part as a host array, the status word): both come back through one
        pinned buffer with one wait on the current stream.  The array is a view
        of that buffer, valid until the next read_back (the caller serialises
        its calls on this pool)."""
        n = part.numel()
        if self._result is None or self._result.numel() < n + 1:
            self._result = torch.empty(max(n + 1, 1 << 14), dtype=torch.float32).pin_memory()
        hp, hs = self._result[:n].view(part.shape), self._result[n:n + 1].view(torch.int32)
        hp.copy_(part, non_blocking=True)
        hs.copy_(status.view(torch.int32).reshape(1), non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return hp.numpy(), int(hs.item())

    def _stage(self, arrays):
        """Copy the given small host arrays to the device in one transfer through
        a pinned staging buffer; returns device views of them in order.  Each
        array starts on a 16-byte boundary and keeps its dtype."""
        sizes = [(a.nbytes + 15) // 16 * 16 for a in arrays]
        total = max(16, sum(sizes))
        if self._pin is None or self._pin.numel() < total:
            self._pin = torch.empty(max(total, 1 << 16), dtype=torch.uint8).pin_memory()
            self._dev_stage = torch.empty(self._pin.numel(), dtype=torch.uint8, device=self.device)
        if self._stage_done is not None:
            self._stage_done.synchronize()     # the previous call's copy out of the pinned buffer has finished
        host = self._pin.numpy()
        off = 0
        for a, n in zip(arrays, sizes):
            host[off:off + a.nbytes] = np.ascontiguousarray(a).view(np.uint8).reshape(-1)
            off += n
        self._dev_stage[:total].copy_(self._pin[:total], non_blocking=True)
        self._stage_done = torch.cuda.Event()
        self._stage_done.record()
        views, off = [], 0
        for a, n in zip(arrays, sizes):
            t = self._dev_stage[off:off + a.nbytes].view(_TORCH_DTYPE[a.dtype.str]).view(a.shape)
            views.append(t)
            off += n
        return views

    def compute(self, x: torch.Tensor, keys, rows, weights, gemm_min_rows: int = GEMM_MIN_ROWS):
        """Weighted expert outputs summed per input row: returns (unique rows,
        (U, H) device tensor) with sum_p w_p * expert_p(x[row_p]) for the picks
        (keys[i], rows[i][j], weights[i][j]).  The call's routing arrays go to
        the device in one copy; the kernels run on the current stream and the
        result is ready when the stream reaches it (the caller's .cpu() waits)."""
        H = x.shape[1]
        dev = self.device
        counts = np.array([len(r) for r in rows], np.int64)
        all_rows = np.concatenate([np.asarray(r, np.int64) for r in rows]) if len(rows) else np.zeros(0, np.int64)
        all_w = np.concatenate([np.asarray(w, np.float32) for w in weights]) if len(rows) else np.zeros(0, np.float32)
        P = len(all_rows)
        status = torch.zeros(1, dtype=torch.int32, device=dev)     # this call's own status word
        if P == 0:
            return np.zeros(0, np.int64), torch.zeros((0, H), device=dev), status
        uniq, uidx = np.unique(all_rows, return_inverse=True)
        y = torch.empty((P, H), dtype=torch.float32, device=dev)
        row_exp = D.row_exponents(x)
        # experts of one signature share a launch
        sigs: dict = {}
        for i, k in enumerate(keys):
            sigs.setdefault(self.entries[k][0].signature, []).append(i)
        base = np.concatenate([[0], np.cumsum(counts)])
        # per unique row, its picks in order: CSR for the weighted combine
        order = np.argsort(uidx, kind="stable").astype(np.int32)
        row_ptr = np.concatenate([[0], np.cumsum(np.bincount(uidx, minlength=len(uniq)))]).astype(np.int32)
        host = [order, all_w[order], row_ptr]
        plan = []
        for sig, idx in sigs.items():
            ents = [self.entries[keys[i]] for i in idx]
            table = np.array([(en[2], en[3]) for en in ents], np.int64)
            eexp = np.zeros((len(idx), 4), np.int32)
            eexp[:, :3] = [en[0].eexp for en in ents]
            if len(sigs) == 1:       # one signature (the usual case): its picks are all picks, in order
                c, sel = counts.astype(np.int32), None
                host += [table, eexp, c, base.astype(np.int32), all_rows.astype(np.int32)]
            else:
                c = counts[idx].astype(np.int32)
                sel = np.concatenate([np.arange(base[i], base[i + 1]) for i in idx])
                host += [table, eexp, c, np.concatenate([[0], np.cumsum(c)]).astype(np.int32),
                         all_rows[sel].astype(np.int32), sel.astype(np.int64)]
            plan.append((sig, len(host) - (5 if sel is None else 6), sel))
        d = self._stage(host)
        for sig, j, sel in plan:
            table, eexp, c, offs, srows = d[j:j + 5]
            r = D.Routing.from_plan(c, offs, srows)
            s = _Set(*sig, table, eexp)
            if sel is None:
                run_experts(s, x, row_exp, r, y, self.workspace, status, gemm_min_rows)
            else:
                ys = torch.empty((max(len(sel), 1), H), dtype=torch.float32, device=dev)
                run_experts(s, x, row_exp, r, ys, self.workspace, status, gemm_min_rows)
                y[d[j + 5]] = ys[:len(sel)]
        part = D.combine(y, d[0], d[1], len(uniq), 1, row_ptr=d[2])
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
        self.gpu_device_ms = None
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
        """Upload one moelan Expert in its packed form: its bytes as moelan
        holds them go to the device and the library's packers lay them out
        there.  False if the tier is full or the expert has no packed form (it
        then stays on the CPU)."""
        with self.lock:
            packed = pack_expert_on(expert, self.pool.device, max_bytes=self.budget - self.used)
            if packed is None:
                return False
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
        """Launch the groups whose experts this tier holds and hand back the
        rest: (handle or None, groups left for the CPU).  The membership test
        and the launch happen under the tier's lock, so release() cannot
        empty the tier in between."""
        with self.lock:
            mine, rest = [], []
            for g in groups:
                (mine if (layer, int(g[0])) in self.experts else rest).append(g)
            return (self.launch(layer, x, mine) if mine else None), rest

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
        """Set ``share``, the fraction of routed work this GPU should take so it
        and the CPU finish a layer together: share = cpu / (gpu + cpu), from
        the median wall time per expert of each side on one input row (a
        decode step), the GPU side through launch + collect with the host
        copies that a real call makes.  The device time of the GPU side alone
        (CUDA events) is kept in ``gpu_device_ms``.  The sample expert is
        uploaded under a key no layer routes to and dropped afterwards."""
        key = (-1, 0)
        if not self.add(key, sample_expert):
            raise RuntimeError("the sample expert has no packed form for this GPU tier")
        try:
            x = np.random.default_rng(0).standard_normal((1, hidden)).astype(np.float32)
            groups = [(0, np.zeros(1, np.int64), np.ones(1, np.float32))]
            sink = np.zeros_like(x)

            def on_gpu():
                self.collect(self.launch(key[0], x, groups), sink)

            def on_cpu():
                cpu_expert_fn(x)

            def median_s(fn, n):
                ts = []
                for _ in range(n):
                    t0 = time.perf_counter()
                    fn()
                    ts.append(time.perf_counter() - t0)
                return float(np.median(ts))

            n = max(1, int(repeats))
            median_s(on_gpu, 3)                # first calls: kernel set-up, allocator, page-in
            median_s(on_cpu, 3)
            g = median_s(on_gpu, n)
            c = median_s(on_cpu, n)
            with torch.cuda.device(self.device):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                self.launch(key[0], x, groups)
                b.record()
                b.synchronize()
                self.gpu_device_ms = a.elapsed_time(b)
        finally:
            with self.lock:
                self.experts.pop(key, None)
                if key in self.pool.entries:
                    self.used -= self.pool.pop(key)
        self.calls, self.busy_s = 0, 0.0          # calibration traffic is not routed work
        self.gpu_ms, self.cpu_ms = 1e3 * g, 1e3 * c
        self.share = c / (g + c) if g + c > 0 else 0.0
        return self.share

    def stats(self) -> dict:
        return {"device": self.name, "experts": len(self.experts), "used_bytes": self.used,
                "budget_bytes": self.budget, "share": round(self.share, 3),
                "gpu_ms_per_expert": self.gpu_ms, "cpu_ms_per_expert": self.cpu_ms,
                "calls": self.calls, "busy_s": round(self.busy_s, 3)}


def bench_gpu(spec: str, budget: int, hidden: int, inter: int, fmt: str, gs: int = 64, make_expert=None) -> dict:
    """The GPU half of a node's speed benchmark (what moelan/accel.py:400-411
    reports): ``gpu_ms``, the wall time per expert of a one-row call on this
    tier (host copies included), ``gpu_experts``, how many experts of this
    shape fit in ``budget`` in their packed form on the device, and
    ``gpu_name``.  ``make_expert(hidden, inter, fmt, gs)`` builds the sample
    (default moelan.experts.synthetic_expert); the sample's own __call__ is the
    CPU side of the calibration.  Raises RuntimeError when the device cannot
    be opened or the sample has no packed form."""
    if make_expert is None:
        from moelan.experts import synthetic_expert as make_expert
    sample = make_expert(hidden, inter, fmt, gs)
    packed = pack_expert(sample)
    if packed is None:
        raise RuntimeError(f"a {fmt} expert has no packed form for this GPU tier")
    tier = GpuTier(spec, budget)
    try:
        tier.calibrate(sample, sample, hidden)
        return {"gpu_ms": tier.gpu_ms, "gpu_experts": int(budget // max(1, packed.nbytes)), "gpu_name": tier.name}
    finally:
        tier.release()
