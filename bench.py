"""Benchmark of the routed-expert hot path on B200.

One step = one MoE layer of the Qwen3-30B-A3B shape (config 2 of the
benchmark: d_model 2048, 128 experts, top-8, expert intermediate 768, int4
group-32 experts with f16 scales) over a decode batch of T tokens: router
logits -> softmax top-k -> permute by expert -> fused gate|up/SiLU/down
mat-vecs over the packed experts -> weighted combine.  The line's "prefill"
object times the same layer at 2048 / 4096 tokens (config 3: int8 group-32
experts with f32 scales; and the int4 layer), where the experts run as
grouped GEMMs on the tensor cores.  Synthetic seeded inputs (numpy PCG64)
with the benchmark's shapes and distributions.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl reference]

Prints one JSON line (rank 0).  ``--impl reference`` times the reference's
CPU algorithm for the same step (the oracle restatement in oracle/, with all
host threads) instead of the GPU.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

# the reference runs BLAS single-threaded and parallelises over experts
# (moelan/__init__.py:9-12); both CPU timings below follow it
os.environ["OPENBLAS_NUM_THREADS"] = "1"

import numpy as np

ROOT = Path(__file__).resolve().parent
H, I, E, K_TOP, GS = 2048, 768, 128, 8, 32
EXPERT_BYTES = 2 * I * H // 2 + 2 * I * (H // GS) * 2 + H * I // 2 + H * (I // GS) * 2   # 2,654,208
METRIC = "moe_layer_tokens_per_s"
UNIT = "tokens/s"
L2_ROTATE_LAYERS = 4
# DRAM bytes (read + write) of one decode step's two expert-kernel launches at
# T=64, from one ncu capture of `bench.py --profile` (the dominant kernel's
# traffic; other token counts report None)
NCU_DECODE_TRAFFIC = {64: 343_900_000}
# this library's kernels per decode step: router logits + top-k, permute, the
# decode's clear of its activation maxima, gate|up and down phases, combine
LAUNCHES_PER_STEP = 7
# expert parallelism adds no kernel of ours (NCCL all-gather and reduce-scatter,
# one torch.where for the local pick mask)
LAUNCHES_PER_EP_STEP = 7


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=400)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--tokens", type=int, default=64)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--no-sweep", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--profile", action="store_true",
                   help="only the main timed loop (for ncu): no e2e, sweep, prefill or CPU baseline")
    p.add_argument("--profile-prefill", action="store_true",
                   help="only a few prefill steps of the int4 layer at 2048 tokens (for ncu)")
    p.add_argument("--no-prefill", action="store_true")
    p.add_argument("--no-dropin", action="store_true", help="skip the drop-in moe_q4 end-to-end figure")
    p.add_argument("--no-parity", action="store_true", help="skip the multi-GPU step's check against one GPU")
    p.add_argument("--phases", action="store_true",
                   help="with --gpus N > 1: time each phase of the expert-parallel decode step (eager, CUDA events)")
    return p.parse_args()


def peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def make_experts(seed=0):
    from distributedmoellm_b200 import synthetic as S
    rng = np.random.default_rng(seed)
    experts = {e: S.int4_expert(rng, H, I, GS, f16_scales=True) for e in range(E)}
    router = S.router(rng, E, H)
    make_experts.router = router
    return experts, router


def int8_layer(router, dev, seed=3):
    """Config 3: the same layer with int8 group-32 experts and f32 scales (5.3 MB each, 680 MB)."""
    import torch
    from distributedmoellm_b200 import layout as L
    from distributedmoellm_b200 import synthetic as S
    from distributedmoellm_b200.layer import MoELayer
    from distributedmoellm_b200.store import LayerExperts
    rng = np.random.default_rng(seed)
    ex = LayerExperts(E, H, I, GS, L.FMT_Q8_F32, L.FMT_Q8_F32, dev)
    for e in range(E):
        ex.put_int8(e, *S.int8_expert(rng, H, I, GS))
    ex.publish()
    return MoELayer(torch.from_numpy(router).to(dev), ex, K_TOP, True)


PREFILL_FLOPS_PER_TOKEN = 2 * K_TOP * 3 * H * I      # 75.5 MFLOP


def gguf_layer(dev, seed=4):
    """Config 4: Mixtral-8x7B MoE layer shape (d_model 4096, 8 experts top-2,
    intermediate 14336) with GGUF experts: gate and up Q4_K, down Q8_0, the
    f16 block scales pinned to 0.001 as the reference's random GGUF experts
    do (128.45 MB per expert)."""
    import types
    import torch
    from distributedmoellm_b200 import layout as L
    from distributedmoellm_b200 import synthetic as S
    from distributedmoellm_b200.layer import MoELayer
    from distributedmoellm_b200.store import LayerExperts
    NS = types.SimpleNamespace
    Hm, Im, Em = 4096, 14336, 8
    rng = np.random.default_rng(seed)
    ex = LayerExperts(Em, Hm, Im, 32, L.FMT_Q4K_F32, L.FMT_Q8_F16, dev)
    for e in range(Em):
        g, u, d = S.gguf_rows(rng, Im, Hm, 12), S.gguf_rows(rng, Im, Hm, 12), S.gguf_rows(rng, Hm, Im, 8)
        ex.put_expert(e, NS(gu=NS(parts=(NS(raw=g, qtype=12, shape=(Im, Hm)), NS(raw=u, qtype=12, shape=(Im, Hm)))),
                            down=NS(raw=d, qtype=8, shape=(Hm, Im)), inter=Im))
    ex.publish()
    return MoELayer(torch.from_numpy(S.router(rng, Em, Hm)).to(dev), ex, 2, True)


def measure_prefill(layer, T, steps, warmup, world, dev, seed=5):
    """Graph replays of the whole layer and of its expert kernels alone at T
    tokens (weights > L2, so every step streams them from HBM)."""
    import torch
    import torch.distributed as dist
    x = torch.from_numpy(np.random.default_rng(seed).standard_normal((T, layer.H), dtype=np.float32)).to(dev)
    full = layer.capture(x)
    ex = layer.capture(x, experts_only=True)
    torch.cuda.synchronize()

    def timed(g, n):
        for _ in range(warmup):
            g.replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    full.replay()
    check_status([layer], T)
    ms, ex_ms = timed(full, steps), timed(ex, steps)
    st = int(layer.status(T))
    plan = layer.kernel_plan(T)
    del full, ex
    return ms, ex_ms, st, plan


def check_status(layers, T):
    """Stop at once when a kernel reported a failure (a wait that ran out of
    time sets a status bit and every later wait of that launch gives up), so a
    broken build does not run its whole timed loop at two seconds a launch."""
    st = max(int(l.status(T)) for l in layers)
    if st:
        raise RuntimeError(f"the expert kernels reported status {st} at T={T}")


# ---- clocks sampled during the timed region ------------------------------------------

class Clocks:
    """SM clock, power and clock-event reasons sampled through NVML (what
    nvidia-smi reads) every few ms while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, gpu_index: int, period_s: float = 0.005):
        self.idx, self.period, self.rows, self.stop, self.t = gpu_index, period_s, [], threading.Event(), None

    def __enter__(self):
        try:
            import pynvml as N
            N.nvmlInit()
            h = N.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_sm = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)

            def poll():
                while not self.stop.is_set():
                    try:
                        self.rows.append((N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM),
                                          N.nvmlDeviceGetCurrentClocksEventReasons(h),
                                          N.nvmlDeviceGetPowerUsage(h) / 1000.0))
                    except Exception:
                        pass
                    time.sleep(self.period)
            self.t = threading.Thread(target=poll, daemon=True)
            self.t.start()
        except Exception:
            self.max_sm = None
        return self

    def __exit__(self, *a):
        self.stop.set()
        if self.t is not None:
            self.t.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_sm, "reasons": ["unsampled"], "samples": 0}
        reasons = sorted({n for _, r, _ in self.rows for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": self.max_sm,
                "reasons": reasons, "samples": len(self.rows),
                "power_w_max": round(max(r[2] for r in self.rows), 1)}


# ---- CPU side: the reference's algorithm (oracle restatement) -----------------------------

REF = ROOT / "baseline" / "_ref"


class _Threads:
    """Thread control of one CPU implementation: ``set(n)`` / ``get()``."""

    def __init__(self, set_fn, get_fn):
        self.set, self.get = set_fn, get_fn


def cpu_step_fn(experts, router, T, seed=7):
    """One MoE-layer step of the reference's CPU algorithm on the same inputs:
    moelan itself when it is installed under baseline/_ref (model.route,
    group_by_expert and ExpertStore.compute over in-memory Packed4 experts,
    numba kernels with exact f32 activations, MOELAN_INT8_ACT=0), else the C
    restatement in oracle/.  Returns (step, threads control, kind, what)."""
    x = np.random.default_rng(seed).standard_normal((T, H), dtype=np.float32)
    if (REF / "moelan").is_dir():
        import tempfile
        os.environ["MOELAN_INT8_ACT"] = "0"
        os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba_"))
        sys.path.insert(0, str(REF))
        import numba
        from moelan import model as M
        from moelan.experts import Expert, ExpertStore, Packed4

        class MemSource:
            zero_copy = False

            def __init__(self, ex):
                self.ex = ex

            def has(self, key):
                return key[1] in self.ex

            def load(self, key):
                return self.ex[key[1]]

        objs = {e: Expert(Packed4(gr, np.ascontiguousarray(gsc, np.float32), GS, (2 * I, H)),
                          Packed4(dr, np.ascontiguousarray(dsc, np.float32), GS, (H, I)), I)
                for e, (gr, gsc, dr, dsc) in experts.items()}
        store = ExpertStore([MemSource(objs)], fmt="int4")

        def step():
            idx, w = M.route(x @ router.T, K_TOP, True)
            ex, off, rows, wts = M.group_by_expert(idx, w)
            groups = [(ex[i], rows[off[i]:off[i + 1]], wts[off[i]:off[i + 1]]) for i in range(len(ex))]
            return store.compute(0, x, groups)
        thr = _Threads(numba.set_num_threads, numba.get_num_threads)
        return step, thr, "reference", "moelan (baseline/_ref): route + group_by_expert + ExpertStore.compute, numba"
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    desc = {e: (("q4", gr, gsc.astype(np.float32), GS, False), ("q4", dr, dsc.astype(np.float32), GS, False))
            for e, (gr, gsc, dr, dsc) in experts.items()}

    def step():
        return O.moe_layer(x, router, desc, K_TOP, True, I)[0]
    return step, _Threads(O.set_threads, O.threads), "port", "C+OpenMP restatement of moelan's fused int4 layer"


def host_threads() -> int:
    """Host cores this process may run on (torchrun sets OMP_NUM_THREADS=1;
    the CPU timings use every core regardless)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def time_cpu(step, thr, warmup=1, max_steps=200, budget_s=12.0):
    """The one CPU timing of the reference's algorithm, used by both the GPU
    arm's cpu_baseline and the reference arm: its threads set to every host
    core, ``warmup`` untimed steps (numba compiles on the first), then up to
    ``max_steps`` steps or ``budget_s`` seconds.  Returns (seconds per step,
    steps, threads)."""
    thr.set(host_threads())
    for _ in range(max(1, warmup)):
        step()  # warm (thread pools, page-in)
    n, t0 = 0, time.perf_counter()
    while n < max_steps and (n == 0 or time.perf_counter() - t0 < budget_s):
        step()
        n += 1
    return (time.perf_counter() - t0) / n, n, thr.get()


# ---- GPU side ---------------------------------------------------------------------------------

def build_layers(experts, router, dev, n_layers):
    import torch
    from distributedmoellm_b200 import layout as L
    from distributedmoellm_b200.layer import MoELayer
    from distributedmoellm_b200.store import LayerExperts
    base = LayerExperts(E, H, I, GS, L.FMT_Q4_F16, L.FMT_Q4_F16, dev)
    for e, (gr, gsc, dr, dsc) in experts.items():
        base.put_int4(e, gr, gsc, dr, dsc, offset=False)
    base.publish()
    rt = torch.from_numpy(router).to(dev)
    return [MoELayer(rt, ex, K_TOP, True) for ex in clone_experts(base, n_layers)]


def clone_experts(base, n):
    """n layers of the same expert bytes at different addresses (so that
    rotating over them streams every step's weights from HBM, not L2)."""
    from distributedmoellm_b200.store import LayerExperts
    out = [base]
    for _ in range(n - 1):
        ex = LayerExperts(base.E, base.H, base.I, base.gs, base.fmt_gu, base.fmt_down, base.device)
        ex.buf.copy_(base.buf)
        off = ex.buf.data_ptr() - base.buf.data_ptr()
        ex._table_host = base._table_host + np.where(base._table_host != 0, off, 0)
        ex._eexp_host = base._eexp_host.copy()
        ex.present = set(base.present)
        ex.publish()
        out.append(ex)
    return out


def run_gpu_ep(args, rank, world, dev):
    """Expert parallelism over the world's GPUs: rank r holds experts
    r*E/N .. (r+1)*E/N - 1 and T tokens of its own.  Decode: the all-gather
    form (ep.EPGatherLayer); prefill (int8, 2048 tokens per rank): the
    peer-memory form (ep.EPPeerLayer), rows to their experts' ranks and
    results back by stores into the other GPUs' memory."""
    import torch
    import torch.distributed as dist
    from distributedmoellm_b200 import device as D
    from distributedmoellm_b200 import layout as L
    from distributedmoellm_b200 import synthetic as S
    from distributedmoellm_b200.ep import EPPeerLayer
    from distributedmoellm_b200.store import LayerExperts
    D.require_device()
    experts, router = make_experts(0)
    El = E // world
    rt = torch.from_numpy(router).to(dev)
    base = LayerExperts(El, H, I, GS, L.FMT_Q4_F16, L.FMT_Q4_F16, dev)
    for j in range(El):
        base.put_int4(j, *experts[rank * El + j])
    base.publish()
    from distributedmoellm_b200.ep import EPGatherLayer
    layers = [EPGatherLayer(rt, ex, E, K_TOP) for ex in clone_experts(base, L2_ROTATE_LAYERS * world)]
    pk, pk_kind = peaks()

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def measure(lays, T, steps, warmup, seed, host=False, graphs=False):
        rng = np.random.default_rng(seed + 31 * rank)
        hx = [torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)) for _ in lays]
        if host:
            hx = [h.pin_memory() for h in hx]
            hout = torch.empty((T, H), dtype=torch.float32).pin_memory()
        xs = [h.to(dev) for h in hx]
        n = len(lays)
        gs = [l.capture(x) for l, x in zip(lays, xs)] if graphs else None

        def step(i):
            if host:
                xs[i % n].copy_(hx[i % n], non_blocking=True)
            if graphs:
                gs[i % n].replay()
                out = lays[i % n].buffers(T).out
            else:
                out = lays[i % n](xs[i % n])
            if host:
                hout.copy_(out, non_blocking=True)

        for i in range(warmup):
            step(i)
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(steps):
            step(i)
        b.record()
        torch.cuda.synchronize()
        dist.barrier()
        del gs                          # graphs holding collectives go before the process group does
        return max_over_ranks(a.elapsed_time(b) / steps)

    T = args.tokens
    parity = {}
    if not args.no_parity:
        # the EP step's own output against one GPU holding every expert over all ranks' tokens
        from distributedmoellm_b200.layer import MoELayer, kernel_plan
        full = LayerExperts(E, H, I, GS, L.FMT_Q4_F16, L.FMT_Q4_F16, dev) if rank == 0 else None
        if rank == 0:
            for e in range(E):
                full.put_int4(e, *experts[e])
            full.publish()
        ep_gemm = any(k == "gemm" for k, _ in kernel_plan(base, T * K_TOP, layers[0].gemm_min_rows))
        parity["decode"] = ep_parity(layers[0], lambda: MoELayer(rt, full, K_TOP, True, gemm_min_rows=0),
                                     T, rank, world, dev, 2e-3 if ep_gemm else 1e-5, 4000)
        del full
    phases = ep_phase_times(layers[0], T, rank, dev, 50, 5) if args.phases else None
    gpu_index = dev.index or 0
    with Clocks(gpu_index) as clk:
        ms = measure(layers, T, args.steps, args.warmup, 1000, graphs=True)
    value = world * T / (ms / 1e3)
    e_ms = measure(layers, T, max(10, args.steps // 2), 3, 2000, host=True, graphs=True)
    e2e = {"value": round(world * T / (e_ms / 1e3), 1), "unit": UNIT, "h2d_bytes_per_step": T * H * 4,
           "d2h_bytes_per_step": T * H * 4,
           "api": "distributedmoellm_b200.ep.EPGatherLayer (CUDA graph of forward, collectives included)"}
    # whole-step HBM fraction of one rank: its local expert bytes streamed per step over the step time
    alg = El * EXPERT_BYTES + T * H * 4 * 2
    roof = {"bound": "hbm", "achieved": round(alg / (ms / 1e3) / 1e9, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": round(alg / (ms / 1e3) / 1e9 / pk["hbm_gbs"], 4), "traffic": None, "peak_kind": pk_kind,
            "kernel": "whole EP step per rank (all-gather, route, local experts, combine, reduce-scatter)",
            "alg_bytes_per_launch": int(alg)}
    prefill = {}
    if not args.no_prefill:
        rng = np.random.default_rng(3)
        q8 = LayerExperts(El, H, I, GS, L.FMT_Q8_F32, L.FMT_Q8_F32, dev)
        for e in range(E):
            parts = S.int8_expert(rng, H, I, GS)
            if e // El == rank:
                q8.put_int8(e - rank * El, *parts)
        q8.publish()
        pl = [EPPeerLayer(rt, q8, E, K_TOP)]
        if not args.no_parity:
            def full_q8():
                from distributedmoellm_b200.layer import MoELayer
                rng8 = np.random.default_rng(3)
                f8 = LayerExperts(E, H, I, GS, L.FMT_Q8_F32, L.FMT_Q8_F32, dev)
                for e in range(E):
                    f8.put_int8(e, *S.int8_expert(rng8, H, I, GS))
                f8.publish()
                return MoELayer(rt, f8, K_TOP, True)
            parity["prefill_int8_T2048"] = ep_parity(pl[0], full_q8, 2048, rank, world, dev, 2e-3, 6000)
        for Tp in (2048,):
            m = measure(pl, Tp, max(10, args.steps // 8), 3, 3000, graphs=True)
            prefill[f"int8_T{Tp}_ep{world}"] = {
                "tokens_per_s": round(world * Tp / (m / 1e3), 1), "ms_per_step": round(m, 5),
                "api": "distributedmoellm_b200.ep.EPPeerLayer (CUDA graph: counts all-gather, peer-store "
                       "dispatch, grouped GEMMs storing results to the source ranks, combine)"}
            if args.phases:
                prefill[f"int8_T{Tp}_ep{world}"]["phases_us"] = ep_phase_times(
                    pl[0], Tp, rank, dev, 20, 3, PEER_PHASES)
        pl[0].close()
    if parity:
        prefill["parity"] = parity
    if phases:
        prefill["decode_phases_us"] = phases
    return value, ms, roof, e2e, {}, None, clk.summary(), 0, prefill, None


GATHER_PHASES = ("route", "gather", "permute", "experts", "combine", "reduce")
PEER_PHASES = ("route", "counts", "dispatch", "experts", "combine")


def ep_phase_times(layer, T, rank, dev, steps, warmup, names=GATHER_PHASES):
    """Per-phase device time of an expert-parallel step (eager launches,
    CUDA events recorded between the phases on the current stream; a phase
    that ends in a collective includes the wait for the slowest rank), the
    mean over ``steps`` steps, then the max over ranks, in microseconds."""
    import torch
    import torch.distributed as dist
    x = torch.from_numpy(np.random.default_rng(77 + rank).standard_normal((T, H), dtype=np.float32)).to(dev)
    names = list(names)
    tot = {n: 0.0 for n in names}
    for it in range(warmup + steps):
        ev = {"start": torch.cuda.Event(enable_timing=True)}
        ev["start"].record()

        def mark(name):
            ev[name] = torch.cuda.Event(enable_timing=True)
            ev[name].record()
        layer(x, mark=mark)
        torch.cuda.synchronize()
        if it >= warmup:
            prev = "start"
            for n in names:
                tot[n] += ev[prev].elapsed_time(ev[n]) * 1e3
                prev = n
    dist.barrier()
    t = torch.tensor([tot[n] / steps for n in names], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return {n: round(float(v), 2) for n, v in zip(names, t.tolist())}


def ep_parity(ep_layer, make_full, T, rank, world, dev, bar, seed):
    """One step of ``ep_layer`` on every rank's own T tokens, gathered to rank
    0 and compared there with ``make_full()`` (one GPU holding every expert)
    over all ranks' tokens in rank order, in chunks of at most 4096 tokens
    (each token's result does not depend on the others in its batch).  The
    error is max|ep - one| / max|one| per output row; returns
    {"max_row_err", "bar", "ok", "tokens"} on rank 0, None elsewhere."""
    import torch
    import torch.distributed as dist
    x = torch.from_numpy(np.random.default_rng(seed + rank).standard_normal((T, H), dtype=np.float32)).to(dev)
    out = ep_layer(x).clone()
    xs = [torch.empty_like(x) for _ in range(world)]
    outs = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(xs, x)
    dist.all_gather(outs, out)
    res = None
    if rank == 0:
        one = make_full()
        xa = torch.cat(xs)
        ref = torch.cat([one(xa[i:i + 4096]).clone() for i in range(0, xa.shape[0], 4096)])
        got = torch.cat(outs).double()
        ref = ref.double()
        err = ((got - ref).abs().amax(dim=1) / ref.abs().amax(dim=1).clamp_min(1e-30)).max().item()
        res = {"max_row_err": float(err), "bar": bar, "ok": bool(err <= bar and torch.isfinite(got).all().item()),
               "tokens": int(xa.shape[0])}
        del one
    dist.barrier()
    return res


def run_gpu(args, rank, world, dev):
    import torch
    import torch.distributed as dist
    from distributedmoellm_b200 import device as D
    D.require_device()
    experts, router = make_experts(0)
    layers = build_layers(experts, router, dev, L2_ROTATE_LAYERS)
    pk, pk_kind = peaks()

    def measure(T, steps, warmup):
        """Step time (graph replays of the whole layer) and expert-kernel time
        (graph replays of the decode kernels alone), both by CUDA events."""
        rng = np.random.default_rng(1000 + 17 * rank + T)
        xs = [torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(dev) for _ in range(len(layers))]
        full = [l.capture(x) for l, x in zip(layers, xs)]
        dec = [l.capture(x, experts_only=True) for l, x in zip(layers, xs)]
        torch.cuda.synchronize()
        uniq = [int(l.buffers(T).routing.n_unique.item()) for l in layers]
        L = len(layers)
        for i in range(warmup):
            full[i % L].replay()
        check_status(layers, T)

        def timed(graphs):
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for i in range(steps):
                graphs[i % L].replay()
            b.record()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            return a.elapsed_time(b) / steps

        ms = timed(full)
        dec_ms = timed(dec)
        u_avg = statistics.mean(uniq[i % L] for i in range(steps))
        status = max(int(l.status(T)) for l in layers)
        del full, dec
        return ms, dec_ms, u_avg, status

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    T = args.tokens
    gpu_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(dev.index or 0)).split(",")[dev.index or 0]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES", "").replace(",", "").isdigit() else (dev.index or 0)
    if args.profile_prefill:
        ms, ex_ms, status, _ = measure_prefill(layers[0], 2048, args.steps, args.warmup, world, dev)
        return world * 2048 / (ms / 1e3), ms, {}, {}, {}, None, {}, status, {}, None
    with Clocks(gpu_index) as clk:
        ms, dec_ms, u_avg, status = measure(T, args.steps, args.warmup)
    if args.profile:
        return world * T / (ms / 1e3), ms, {}, {}, {}, None, clk.summary(), status, {}, None
    ms = max_over_ranks(ms)
    value = world * T / (ms / 1e3)

    # roofline of the dominant kernel (the fused decode: both phases)
    alg_bytes = u_avg * EXPERT_BYTES + T * H * 4 + T * K_TOP * H * 4
    achieved = alg_bytes / (dec_ms / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": NCU_DECODE_TRAFFIC.get(T), "peak_kind": pk_kind,
            "kernel": "moe_decode_kernel (gate|up + down phases)", "kernel_ms": round(dec_ms, 5),
            "alg_bytes_per_launch": int(alg_bytes), "unique_experts": u_avg}

    # end to end through the public API with host buffers (pinned), H2D + D2H inside the timed region
    e2e = measure_e2e(layers, T, args.steps, args.warmup, world, dev)
    e2e["value"] = world * T / (max_over_ranks(e2e.pop("ms")) / 1e3)

    sweep = {}
    if not args.no_sweep:
        for Ts in (1, 8, 32, 64):
            if Ts == T:
                continue
            m, dm, u, st = measure(Ts, max(10, args.steps // 2), 3)
            ab = u * EXPERT_BYTES + Ts * H * 4 + Ts * K_TOP * H * 4
            sweep[f"decode_T{Ts}"] = {"tokens_per_s": round(world * Ts / (max_over_ranks(m) / 1e3), 1),
                                      "ms_per_step": round(m, 5), "kernel_ms": round(dm, 5),
                                      "hbm_frac": round(ab / (dm / 1e3) / 1e9 / pk["hbm_gbs"], 4),
                                      "unique_experts": u}
            status = max(status, st)

    prefill = {}
    if not args.no_prefill:
        l8 = int8_layer(router, dev)
        tf_peak = pk.get("bf16_tflops", 1590.0)
        for name, layer, Tp in (("int8_T2048", l8, 2048), ("int8_T4096", l8, 4096), ("int4_T2048", layers[0], 2048)):
            m, em, st, plan = measure_prefill(layer, Tp, max(10, args.steps // 8), 3, world, dev)
            m, em = max_over_ranks(m), max_over_ranks(em)
            fl = Tp * PREFILL_FLOPS_PER_TOKEN
            prefill[name] = {"tokens_per_s": round(world * Tp / (m / 1e3), 1), "ms_per_step": round(m, 5),
                             "experts_ms": round(em, 5), "grouped_gemm": any(k == "gemm" for k, _ in plan),
                             "kernels": [list(p) for p in plan],
                             "roofline": {"bound": "tensor", "achieved": round(fl / (em / 1e3) / 1e12, 1),
                                          "peak": tf_peak, "unit": "TFLOP/s",
                                          "frac": round(fl / (em / 1e3) / 1e12 / tf_peak, 4),
                                          "peak_kind": pk_kind + " bf16 dense (f16 runs at the same rate)",
                                          "kernel": "expert kernels (gather + gate|up GEMM + down GEMM)"}}
            status = max(status, st)
        del l8
        # config 4: Mixtral-shaped GGUF experts (Q4_K gate/up, Q8_0 down), 1 and 512 tokens
        lg = gguf_layer(dev)
        bytes_per_expert = 2 * (14336 * 4096 // 256 * 144) + 4096 * (14336 // 32 * 34)
        for Tp in (1, 512):
            m, em, st, plan = measure_prefill(lg, Tp, max(10, args.steps // 8), 3, world, dev)
            m, em = max_over_ranks(m), max_over_ranks(em)
            fl = Tp * 2 * 2 * 3 * 4096 * 14336
            used = min(8, 2 * Tp)
            ent = {"tokens_per_s": round(world * Tp / (m / 1e3), 1), "ms_per_step": round(m, 5),
                   "experts_ms": round(em, 5), "grouped_gemm": any(k == "gemm" for k, _ in plan),
                   "kernels": [list(p) for p in plan],
                   "tflops": round(fl / (em / 1e3) / 1e12, 1),
                   "hbm_gbs": round(used * bytes_per_expert / (em / 1e3) / 1e9, 1)}
            ent["roofline"] = ({"bound": "hbm", "achieved": ent["hbm_gbs"], "peak": pk["hbm_gbs"], "unit": "GB/s",
                                "frac": round(ent["hbm_gbs"] / pk["hbm_gbs"], 4)} if Tp == 1 else
                               {"bound": "tensor", "achieved": ent["tflops"], "peak": tf_peak, "unit": "TFLOP/s",
                                "frac": round(ent["tflops"] / tf_peak, 4)})
            prefill[f"gguf_mixtral_T{Tp}"] = ent
            status = max(status, st)
        del lg

    # end to end through the reference-facing drop-in: moelan's own call moe_q4(x, items, H, I, gs, out)
    # with pageable numpy arrays (moelan/experts.py:729-753)
    e2e_dropin = None
    if not args.no_dropin:
        dm = measure_dropin(experts, T, max(10, args.steps // 20), 3)
        e2e_dropin = {"value": round(world * T / (dm / 1e3), 1), "unit": UNIT, "ms_per_step": round(dm, 4),
                      "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": None,
                      "api": "distributedmoellm_b200.kernels.moe_q4 (the install() replacement of "
                             "moelan.kernels.moe_q4), numpy in and out; moelan's host routing before the call "
                             "is not timed"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        step, tc, kind, what = cpu_step_fn(experts, router, T)
        s_per, n, thr = time_cpu(step, tc, warmup=2)
        cpu = {"value": round(T / s_per, 2), "unit": UNIT, "cores": thr, "kind": kind,
               "sample": f"{n} MoE-layer steps of T={T} tokens (all 128 experts resident in host RAM), {what}"}
    return value, ms, roof, e2e, sweep, cpu, clk.summary(), status, prefill, e2e_dropin


def measure_dropin(experts, T, steps, warmup):
    """ms per call of the drop-in moe_q4 with moelan's own arguments: items of
    (q4_expert_ptrs(expert), rows, weights) over host arrays (f32 scales, as
    moelan's fused path requires, kernels.py:929-939), x and out pageable
    numpy; the call copies x in, runs the kernels and adds the result into out
    on the host.  Four token sets with their own routings rotate."""
    import types
    from distributedmoellm_b200 import kernels as Kn
    NS = types.SimpleNamespace
    objs = {}
    for e, (gr, gsc, dr, dsc) in experts.items():
        gu = NS(raw=gr, s=np.ascontiguousarray(gsc, np.float32), gs=GS, offset=False)
        dn = NS(raw=dr, s=np.ascontiguousarray(dsc, np.float32), gs=GS, offset=False)
        objs[e] = NS(gu=gu, down=dn)
    router = make_experts.router
    sets = []
    for i in range(4):
        x = np.random.default_rng(5000 + i).standard_normal((T, H), dtype=np.float32)
        logits = x @ router.T                                       # moelan/model.py:597, 154-167, 226-236
        z = np.exp(logits - logits.max(-1, keepdims=True))
        probs = z / z.sum(-1, keepdims=True)
        idx = np.argsort(-probs, axis=-1, kind="stable")[:, :K_TOP]
        w = np.take_along_axis(probs, idx, axis=-1)
        w = (w / w.sum(-1, keepdims=True)).astype(np.float32)
        order = np.argsort(idx.reshape(-1), kind="stable")
        es, starts = np.unique(idx.reshape(-1)[order], return_index=True)
        offs = np.append(starts, T * K_TOP)
        items = [(Kn.q4_expert_ptrs(objs[int(e)]), order[offs[j]:offs[j + 1]] // K_TOP,
                  w.reshape(-1)[order[offs[j]:offs[j + 1]]]) for j, e in enumerate(es)]
        sets.append((x, items))
    out = np.zeros((T, H), np.float32)
    for i in range(warmup):
        x, items = sets[i % 4]
        Kn.moe_q4(x, items, H, I, GS, out)
    t0 = time.perf_counter()
    for i in range(steps):
        x, items = sets[i % 4]
        Kn.moe_q4(x, items, H, I, GS, out)
    return (time.perf_counter() - t0) / steps * 1e3


def measure_e2e(layers, T, steps, warmup, world, dev):
    """The same step through the public API with host buffers: per step the
    inputs are copied from pinned host memory, the layer runs (its CUDA graph)
    and the output is read back to pinned host memory, all inside the timed
    region."""
    import torch
    import torch.distributed as dist
    rng = np.random.default_rng(999)
    hx = [torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).pin_memory() for _ in layers]
    hout = torch.empty((T, H), dtype=torch.float32).pin_memory()
    dx = [torch.empty((T, H), dtype=torch.float32, device=dev) for _ in layers]
    for x, h in zip(dx, hx):
        x.copy_(h)
    graphs = [l.capture(x) for l, x in zip(layers, dx)]
    outs = [l.buffers(T).out for l in layers]
    L = len(layers)

    def step(i):
        dx[i % L].copy_(hx[i % L], non_blocking=True)
        graphs[i % L].replay()
        hout.copy_(outs[i % L], non_blocking=True)

    for i in range(warmup):
        step(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        step(i)
    b.record()
    torch.cuda.synchronize()
    return {"ms": a.elapsed_time(b) / steps, "unit": UNIT, "h2d_bytes_per_step": T * H * 4,
            "d2h_bytes_per_step": T * H * 4, "api": "distributedmoellm_b200.layer.MoELayer (CUDA graph of forward)"}


def run_reference(args):
    """The reference arm: moelan's CPU algorithm (oracle restatement) on all host cores."""
    experts, router = make_experts(0)
    step, tc, kind, what = cpu_step_fn(experts, router, args.tokens)
    s_per, n, thr = time_cpu(step, tc, warmup=max(2, args.warmup), max_steps=args.steps, budget_s=120.0)
    ms = 1e3 * s_per
    value = args.tokens / (ms / 1e3)
    return {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "impl": "reference",
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args),
            "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": thr, "kind": kind,
                             "sample": f"{n} MoE-layer steps of T={args.tokens}, {what}"},
            "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def workload_config(args):
    return {"workload": f"qwen3-30b-a3b moe layer decode, T={args.tokens} tokens/step per GPU",
            "d_model": H, "experts": E, "top_k": K_TOP, "expert_inter": I, "weights": "int4 g32 f16 scales",
            "tokens_per_gpu": args.tokens,
            "parallelism": f"ep{args.gpus} (experts {E // args.gpus} per GPU; decode: NCCL all-gather of tokens + "
                           f"reduce-scatter of partial sums; prefill: all-to-all of routed rows)"
            if args.gpus > 1 else "single",
            "l2": f"{L2_ROTATE_LAYERS} layers of experts rotated per step (each ~340 MB > 126 MB L2)"}


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return
    import torch
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if world > 1:
        value, ms, roof, e2e, sweep, cpu, clocks, status, prefill, dropin = run_gpu_ep(args, rank, world, dev)
    else:
        value, ms, roof, e2e, sweep, cpu, clocks, status, prefill, dropin = run_gpu(args, rank, world, dev)
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32",
                "dtype_note": "decode: int4 weights x f32 activations, products exact (f16 pieces), f32 sums; "
                              "prefill: f16 tensor-core operands with power-of-two range scaling, f32 sums",
                "data": "synthetic", "config": workload_config(args), "roofline": roof, "cpu_baseline": cpu,
                "e2e": e2e, "e2e_dropin": dropin, "clocks": clocks,
                "gpu_launches": (LAUNCHES_PER_STEP if world == 1 else LAUNCHES_PER_EP_STEP) * args.steps,
                "sweep": sweep, "prefill": prefill, "kernel_status": status}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
