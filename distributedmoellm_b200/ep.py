"""Expert parallelism: one MoE layer over G GPUs, one process per GPU.

The reference's own multi-machine design (moelan/coordinator.py:475-535)
sends each worker one request per layer carrying only the rows routed to its
experts and adds the partial sums back.  Here the workers are the GPUs of
one node and the transport is NCCL all-to-all over NVLink:

1. every rank routes its own tokens (the router is replicated) and sorts its
   picks by expert (mb_router_route, mb_permute);
2. experts are placed in contiguous slices (expert e on rank e // (E/G)), so
   the sorted picks are already grouped by destination; the per-expert
   counts go to the host (they size the exchange) and are exchanged;
3. the picked rows go out in one all_to_all_single, each rank runs its local
   experts over what it received (the decode / grouped-GEMM kernels, with
   the rows regrouped by local expert), and the expert outputs come back in a
   second all_to_all_single;
4. the weighted combine runs in each token's fixed k-slot order, so a
   token's result does not depend on G.

Only the routed rows cross NVLink.  The exchange plan is plain host code over
the compute operations of an ``ops`` object: ``DeviceOps`` (this module)
binds them to the library's CUDA kernels; tests drive the same plan with
other ops over gloo on CPU.

``EPGatherLayer`` is the form for decode-sized batches, where the host round
trip of the exchange plan would cost more than the experts: every rank
routes its own tokens, all-gathers the tokens together with their routing
(one NCCL group of four gathers), sorts all ranks' picks by expert (the same
kernel on the same data gives every rank the same order), runs its own
expert slice over the picks that fall in it, sums each token's local picks
(the other picks are skipped) and a reduce-scatter adds the ranks' partial
sums.  All sizes are fixed by T, nothing goes through the host, and the step
can be captured in a CUDA graph, collectives included.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import device as D
from .layout import FMT_Q4K_F32
from .layer import GEMM_MIN_ROWS, run_experts


def local_plan(recv_ec: np.ndarray):
    """Regroup received rows by local expert.

    ``recv_ec[s, j]``: rows source rank s sent for local expert j, laid out
    in the receive buffer source after source, each source's rows grouped by
    expert in order.  Returns (counts (Eloc,), offsets (Eloc+1,), sorted_rows
    (P,): the receive-buffer row of local pick q, local experts in order and
    within an expert the sources in rank order, inv (P,): the local pick of
    receive-buffer row p)."""
    recv_ec = np.asarray(recv_ec, np.int64)
    G, El = recv_ec.shape
    src_off = np.concatenate([[0], np.cumsum(recv_ec.sum(axis=1))])
    intra = np.concatenate([np.zeros((G, 1), np.int64), np.cumsum(recv_ec, axis=1)], axis=1)
    counts = recv_ec.sum(axis=0)
    offsets = np.concatenate([[0], np.cumsum(counts)])
    parts = [np.arange(src_off[s] + intra[s, j], src_off[s] + intra[s, j] + recv_ec[s, j])
             for j in range(El) for s in range(G)]
    sorted_rows = np.concatenate(parts) if parts else np.zeros(0, np.int64)
    inv = np.empty_like(sorted_rows)
    inv[sorted_rows] = np.arange(len(sorted_rows))
    return (counts.astype(np.int32), offsets.astype(np.int32), sorted_rows.astype(np.int32), inv.astype(np.int32))


class EPLayer:
    """One MoE layer with its E experts spread over the ranks of ``group``.

    ``ops`` provides: ``route(x) -> (w (T*k,), counts (E,), sorted_rows (P,),
    inv (P,))`` on the device, ``gather_rows(src, index) -> rows``,
    ``experts(x_rows, counts, offsets, sorted_rows) -> y`` (the local experts,
    y in local pick order), ``combine(y, inv, w, T, k) -> out`` and ``device``.
    """

    def __init__(self, ops, E: int, top_k: int, H: int, group=None):
        self.ops, self.E, self.k, self.H, self.group = ops, E, top_k, H, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if E % self.world:
            raise ValueError(f"E={E} experts do not split evenly over {self.world} ranks")
        self.E_local = E // self.world
        self.first_expert = self.rank * self.E_local

    def _a2a(self, inp: torch.Tensor, out_rows, in_rows) -> torch.Tensor:
        out = torch.empty((int(sum(out_rows)),) + tuple(inp.shape[1:]), dtype=inp.dtype, device=inp.device)
        dist.all_to_all_single(out, inp, [int(v) for v in out_rows], [int(v) for v in in_rows], group=self.group)
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        ops, G, El = self.ops, self.world, self.E_local
        T = x.shape[0]
        w, counts, sorted_rows, inv = ops.route(x)
        send_ec = counts.reshape(G, El).to(torch.int32)
        recv_ec_t = self._a2a(send_ec.contiguous(), [1] * G, [1] * G)          # row s: what rank s sends here
        send_ec_h = send_ec.cpu().numpy().astype(np.int64)
        recv_ec = recv_ec_t.cpu().numpy().astype(np.int64)
        send_rows, recv_rows = send_ec_h.sum(axis=1), recv_ec.sum(axis=1)
        xs = ops.gather_rows(x, sorted_rows)                                     # picks, grouped by destination
        xr = self._a2a(xs, recv_rows, send_rows)
        lc, lo, lsr, linv = local_plan(recv_ec)
        dev = ops.device
        y_local = ops.experts(xr, torch.from_numpy(lc).to(dev), torch.from_numpy(lo).to(dev),
                              torch.from_numpy(lsr).to(dev))
        yr = ops.gather_rows(y_local, torch.from_numpy(linv).to(dev))          # back to receive order
        yb = self._a2a(yr, send_rows, recv_rows)                                 # my picks' outputs, sorted order
        return ops.combine(yb, inv, w, T, self.k)

    __call__ = forward


class DeviceOps:
    """The compute operations of EPLayer on this GPU's kernels.  ``experts``
    is the rank's LayerExperts holding its E/G local experts as local ids
    0 .. E/G-1 (global id = rank * E/G + local id)."""

    def __init__(self, router: torch.Tensor, experts, E: int, top_k: int, normalize: bool = True,
                 gemm_min_rows: int = GEMM_MIN_ROWS):
        self.router = router.contiguous()
        self.store = experts
        self.E, self.k, self.normalize = E, top_k, normalize
        self.gemm_min_rows = gemm_min_rows
        self.device = router.device
        self._ws = {}

    def _buf(self, name, nbytes):
        b = self._ws.get(name)
        if b is None or b.numel() < nbytes:
            b = self._ws[name] = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.device)
        return b

    def route(self, x):
        T, H = x.shape
        idx = torch.empty((T, self.k), dtype=torch.int32, device=self.device)
        w = torch.empty((T, self.k), dtype=torch.float32, device=self.device)
        rws = self._buf("router", D.router_workspace_bytes(T, H, self.E))
        D.router_route(x, self.router, self.k, self.normalize, idx, w, workspace=rws)
        r = D.permute(idx, w, self.E)
        return w.view(-1), r.counts, r.sorted_rows[:r.P], r.inv[:r.P]

    def gather_rows(self, src, index):
        n = index.numel()
        out = torch.empty((n, src.shape[1]), dtype=torch.float32, device=self.device)
        if n:
            ones = torch.ones(n, dtype=torch.float32, device=self.device)
            D.combine(src, index.to(torch.int32).contiguous(), ones, n, 1, out=out)
        return out

    def experts(self, xr, counts, offsets, sorted_rows):
        ex = self.store
        P, H = xr.shape
        y = torch.empty((max(P, 1), H), dtype=torch.float32, device=self.device)
        if P == 0:
            return y[:0]
        r = D.Routing.from_plan(counts, offsets, sorted_rows)
        row_exp = D.row_exponents(xr)
        status = self._ws.get("status")
        if status is None:
            status = self._ws["status"] = torch.zeros(1, dtype=torch.int32, device=self.device)
        run_experts(ex, xr, row_exp, r, y, self._buf, status, self.gemm_min_rows)
        return y[:P]

    def combine(self, y, inv, w, T, k):
        out = torch.empty((T, y.shape[1]), dtype=torch.float32, device=self.device)
        return D.combine(y, inv, w, T, k, out=out)


def _capture(forward, x: torch.Tensor) -> torch.cuda.CUDAGraph:
    """A CUDA graph of forward(x) after one warm-up call on a side stream."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        forward(x)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        forward(x)
    return g


class _GatherBuffers:
    def __init__(self, T, world, E, k, H, I, dev):
        TA, P = T * world, T * world * k
        self.x_all = torch.empty((TA, H), dtype=torch.float32, device=dev)
        self.row_exp = torch.empty(TA, dtype=torch.int32, device=dev)
        self.idx = torch.empty((TA, k), dtype=torch.int32, device=dev)
        self.w = torch.empty((TA, k), dtype=torch.float32, device=dev)
        # this rank's own tokens' routing, gathered next to the tokens
        self.row_exp_own = torch.empty(T, dtype=torch.int32, device=dev)
        self.idx_own = torch.empty((T, k), dtype=torch.int32, device=dev)
        self.w_own = torch.empty((T, k), dtype=torch.float32, device=dev)
        self.routing = D.Routing(TA, k, E, dev)
        self.rws = torch.empty(D.router_workspace_bytes(T, H, E), dtype=torch.uint8, device=dev)
        self.y = torch.empty((max(P, 1), H), dtype=torch.float32, device=dev)
        self.inv_local = torch.empty(max(P, 1), dtype=torch.int32, device=dev)
        self.partial = torch.empty((TA, H), dtype=torch.float32, device=dev)
        self.out = torch.empty((T, H), dtype=torch.float32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ws = {}

    def workspace(self, name, nbytes):
        b = self.ws.get(name)
        if b is None or b.numel() < nbytes:
            b = self.ws[name] = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.out.device)
        return b


class EPGatherLayer:
    """One MoE layer over the ranks of ``group`` for decode-sized batches:
    each rank routes its own tokens, all-gather of the tokens with their
    routing, the rank's own experts
    (``experts``: its E/G local experts as local ids 0 .. E/G-1), combine of
    its picks, reduce-scatter of the partial sums.  Token results equal the
    one-GPU layer's up to the order of the final sum over ranks."""

    def __init__(self, router: torch.Tensor, experts, E: int, top_k: int, normalize: bool = True, group=None,
                 gemm_min_rows: int = GEMM_MIN_ROWS):
        self.router = router.contiguous()
        self.experts, self.E, self.k, self.normalize, self.group = experts, E, top_k, normalize, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if E % self.world or experts.E != E // self.world:
            raise ValueError(f"E={E} experts do not split into {self.world} slices of {experts.E}")
        self.E_local = E // self.world
        self.first_expert = self.rank * self.E_local
        self.gemm_min_rows = gemm_min_rows
        self._bufs: dict = {}

    def buffers(self, T: int) -> _GatherBuffers:
        b = self._bufs.get(T)
        if b is None:
            ex = self.experts
            b = self._bufs[T] = _GatherBuffers(T, self.world, self.E, self.k, ex.H, ex.I, self.router.device)
        return b

    def forward(self, x: torch.Tensor, mark=None) -> torch.Tensor:
        """``mark(name)``, when given, is called after each phase (route,
        gather, permute, experts, combine, reduce) on the host as the phase's
        work is enqueued, e.g. to record CUDA events between the phases."""
        mark = mark or (lambda name: None)
        T = x.shape[0]
        b = self.buffers(T)
        e0, El, k = self.first_expert, self.E_local, self.k
        x = x.contiguous()
        # each rank routes its own tokens; the tokens and their routing are gathered in one NCCL group
        D.router_route(x, self.router, k, self.normalize, b.idx_own, b.w_own, row_exp=b.row_exp_own, workspace=b.rws)
        mark("route")
        with dist._coalescing_manager(group=self.group, device=x.device):
            dist.all_gather_into_tensor(b.x_all, x, group=self.group)
            dist.all_gather_into_tensor(b.idx, b.idx_own, group=self.group)
            dist.all_gather_into_tensor(b.w, b.w_own, group=self.group)
            dist.all_gather_into_tensor(b.row_exp, b.row_exp_own, group=self.group)
        mark("gather")
        r = D.permute(b.idx, b.w, self.E, b.routing)
        mark("permute")
        P = r.P
        local = D.Routing.from_plan(r.counts[e0:e0 + El], r.offsets[e0:e0 + El + 1], r.sorted_rows[:P])
        run_experts(self.experts, b.x_all, b.row_exp, local, b.y, b.workspace, b.status, self.gemm_min_rows,
                    picks=P // self.world)
        mark("experts")
        # the other ranks' picks are skipped by the combine (pick index -1)
        mine = (b.idx.view(-1) >= e0) & (b.idx.view(-1) < e0 + El)
        torch.where(mine, r.inv[:P], torch.full_like(r.inv[:P], -1), out=b.inv_local[:P])
        D.combine(b.y, b.inv_local[:P], b.w.view(-1), T * self.world, k, out=b.partial)
        mark("combine")
        dist.reduce_scatter_tensor(b.out, b.partial, group=self.group)
        mark("reduce")
        return b.out

    __call__ = forward

    def capture(self, x: torch.Tensor) -> torch.cuda.CUDAGraph:
        """A CUDA graph of forward(x), collectives included, on x's current
        contents; replay it after writing new inputs into x.  Output:
        buffers(T).out.  Release the graph before destroying the process group."""
        return _capture(self.forward, x)

    def status(self, T: int) -> int:
        return int(self.buffers(T).status.item())


class _DeviceView:
    """A device address as a torch tensor (CUDA array interface, no copy)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "strides": None, "version": 3}


def _r1k(n: int) -> int:
    return (n + 1023) // 1024 * 1024


class _PeerBuffers:
    """EPPeerLayer's buffers for batches of T tokens on one rank.  The arena
    (mapped by every rank) holds: receive rows (cap, H) f16 | their exponents
    (cap,) | their return addresses (cap,) | the result rows of this rank's
    own picks (T*k, H) f32; cap = G*T*k, the most any rank can receive."""

    def __init__(self, T, world, rank, E, k, H, I, dev, group):
        P = T * k
        self.T, self.P = T, P
        self.cap = cap = world * P
        self.off_exp = _r1k(cap * H * 2)
        self.off_ret = self.off_exp + _r1k(cap * 4)
        self.off_y = self.off_ret + _r1k(cap * 4)
        nbytes = self.off_y + _r1k(max(P, 1) * H * 4)
        self.opened: list[int] = []
        self.base, handle = D.peer_alloc(nbytes)
        try:
            mine = torch.tensor(list(handle), dtype=torch.uint8, device=dev)
            every = torch.empty((world, D.PEER_HANDLE_BYTES), dtype=torch.uint8, device=dev)
            dist.all_gather_into_tensor(every, mine, group=group)
            every = every.cpu().numpy()
            bases = []
            for s in range(world):
                if s == rank:
                    bases.append(self.base)
                else:
                    self.opened.append(D.peer_open(every[s].tobytes()))
                    bases.append(self.opened[-1])
        except BaseException:
            self.close()
            raise

        def table(off):
            return torch.tensor([b + off for b in bases], dtype=torch.int64, device=dev)
        self.peer_rows, self.peer_exp, self.peer_ret, self.peer_y = (table(0), table(self.off_exp),
                                                                     table(self.off_ret), table(self.off_y))
        self.y_home = torch.as_tensor(_DeviceView(self.base + self.off_y, (max(P, 1), H), "<f4"), device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        self.row_exp = torch.empty(T, **i32)
        self.idx = torch.empty((T, k), **i32)
        self.w = torch.empty((T, k), dtype=torch.float32, device=dev)
        self.routing = D.Routing(T, k, E, dev)
        self.rws = torch.empty(D.router_workspace_bytes(T, H, E), dtype=torch.uint8, device=dev)
        self.counts_all = torch.zeros((world, E), **i32)
        El = E // world
        self.local_counts = torch.zeros(El, **i32)
        self.local_offsets = torch.zeros(El + 1, **i32)
        self.ws = torch.empty(D.prefill_rows_workspace_bytes(cap, I), dtype=torch.uint8, device=dev)
        self.status = torch.zeros(1, **i32)
        self.flag = torch.zeros(1, **i32)
        self.ident = torch.arange(max(P, 1), **i32)
        self.out = torch.empty((T, H), dtype=torch.float32, device=dev)

    def close(self):
        for p in self.opened:
            D.peer_close(p)
        self.opened = []

    def free(self):
        if self.base:
            D.peer_free(self.base)
            self.base = 0


class EPPeerLayer:
    """One MoE layer over the ranks of ``group`` for prefill-sized batches,
    with no host round trip: every rank routes its own tokens, an all-gather
    of the per-expert pick counts (E integers per rank) fixes where every
    rank's rows land, mb_ep_dispatch stores each pick's token row into its
    expert's rank's receive rows (as the grouped GEMM's f16 operand), the
    rank's grouped GEMMs run over what it received and their epilogue stores
    each result row back into the source rank's result rows, and each rank
    combines its own picks.  Two one-integer all-reduces order the ranks
    (rows complete before the GEMMs read them; results complete before the
    combine).  ``experts``: this rank's E/G local experts as local ids
    0 .. E/G-1.  Every rank calls forward (and buffers) with the same T in
    the same order; close() on every rank releases the peer memory."""

    def __init__(self, router: torch.Tensor, experts, E: int, top_k: int, normalize: bool = True, group=None):
        self.router = router.contiguous()
        self.experts, self.E, self.k, self.normalize, self.group = experts, E, top_k, normalize, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if E % self.world or experts.E != E // self.world:
            raise ValueError(f"E={E} experts do not split into {self.world} slices of {experts.E}")
        if experts.fmt_gu == FMT_Q4K_F32:
            raise ValueError("EPPeerLayer: Q4_K experts need the precise gate|up form over f32 rows; use EPLayer")
        self.E_local = E // self.world
        self._bufs: dict = {}

    def buffers(self, T: int) -> _PeerBuffers:
        b = self._bufs.get(T)
        if b is None:
            ex = self.experts
            b = self._bufs[T] = _PeerBuffers(T, self.world, self.rank, self.E, self.k, ex.H, ex.I,
                                             self.router.device, self.group)
        return b

    def forward(self, x: torch.Tensor, mark=None) -> torch.Tensor:
        """``mark(name)``, when given, is called after each phase (route,
        counts, dispatch, experts, combine) as its work is enqueued."""
        mark = mark or (lambda name: None)
        T = x.shape[0]
        b = self.buffers(T)
        x = x.contiguous()
        D.router_route(x, self.router, self.k, self.normalize, b.idx, b.w, row_exp=b.row_exp, workspace=b.rws)
        r = D.permute(b.idx, b.w, self.E, b.routing)
        mark("route")
        dist.all_gather_into_tensor(b.counts_all, r.counts, group=self.group)
        mark("counts")
        D.ep_dispatch(x, b.row_exp, b.idx, r, b.counts_all, self.rank, b.peer_rows, b.peer_exp, b.peer_ret, b.cap,
                      b.local_counts, b.local_offsets, b.status)
        dist.all_reduce(b.flag, op=dist.ReduceOp.MAX, group=self.group)     # every rank's rows have landed
        mark("dispatch")
        D.moe_prefill_rows(self.experts, b.base, b.base + b.off_exp, b.local_counts, b.local_offsets, b.cap, b.ws,
                           y_ret=b.base + b.off_ret, y_peers=b.peer_y, peer_rows=b.P, status=b.status)
        dist.all_reduce(b.flag, op=dist.ReduceOp.MAX, group=self.group)     # every result row has landed
        mark("experts")
        D.combine(b.y_home, b.ident[:b.P], b.w.view(-1), T, self.k, out=b.out)
        mark("combine")
        return b.out

    __call__ = forward

    def capture(self, x: torch.Tensor) -> torch.cuda.CUDAGraph:
        """A CUDA graph of forward(x), collectives included (see
        EPGatherLayer.capture)."""
        return _capture(self.forward, x)

    def status(self, T: int) -> int:
        return int(self.buffers(T).status.item())

    def close(self) -> None:
        """Unmap the other ranks' arenas, wait for every rank to do the same,
        then free this rank's own (collective: every rank calls it)."""
        torch.cuda.synchronize()
        for b in self._bufs.values():
            b.close()
        dist.barrier(group=self.group)
        for b in self._bufs.values():
            b.free()
        self._bufs = {}
