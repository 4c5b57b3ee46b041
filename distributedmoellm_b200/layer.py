"""One MoE layer on the device: router logits -> top-k -> permute by expert ->
fused expert mat-vecs -> weighted combine, every step a kernel of
libmoelan_b200.so on the current stream.

This is the device-side form of moelan/model.py:593-606 (_ffn: logits,
route, backend.moe) with a local backend (model.py:267-278) and
ExpertStore.compute (moelan/experts.py:641-670).  All buffers for a given
token count are allocated once and reused, so a forward can be captured in
a CUDA graph.
"""

from __future__ import annotations

import torch

from . import device as D
from .store import LayerExperts

# average picks per expert from which a layer's experts run as grouped GEMMs (see kernel_plan)
GEMM_MIN_ROWS = 12


def uses_gemm(experts: LayerExperts, P: int, gemm_min_rows: int) -> bool:
    """Whether the grouped-GEMM kernels take the experts' P picks: once the
    picks average at least gemm_min_rows per expert (and the shape allows
    them: H % 128, I % 64, P <= 65536; experts stored without the tensor-core
    exponents stay on the decode kernels)."""
    m = gemm_min_rows
    return (m > 0 and experts.H % 128 == 0 and experts.I % 64 == 0 and P >= experts.E * m and P <= 65536
            and not experts.missing_exp)


def kernel_plan(experts, P: int, gemm_min_rows: int) -> list:
    """Which kernels run for P picks over these experts: ("gemm", 1), every
    expert as a grouped GEMM, or ("decode", 0), every expert on the decode
    mat-vecs.  Timed on B200 at the Qwen3-30B shape (expert kernels, graph
    replays): 128 experts at 1024 / 2048 / 4096 picks take 170 / 172 / 180 us
    as GEMMs against 163 / 266 / 473 us decoded, and a 16-expert slice with 512
    picks 46 us against 88 us; splitting a layer between the two (experts
    below some pick count decoded, the rest as GEMMs) was never faster than the
    better of the two (96, 257-282, 355 us), so one of them takes every
    expert: the GEMM from 12 picks per expert on average (at 8 the two are
    even on one GPU and the decode kernel measured ahead in a 2-GPU
    expert-parallel step, where each rank's 64 experts get 8 picks)."""
    return [("gemm", 1)] if uses_gemm(experts, P, gemm_min_rows) else [("decode", 0)]


def run_experts(experts: LayerExperts, x: torch.Tensor, row_exp: torch.Tensor, routing, y: torch.Tensor,
                workspace, status: torch.Tensor, gemm_min_rows: int, picks: int | None = None) -> None:
    """Every expert's picks through its gate|up, SiLU, down into y (one row
    per pick, in routing order), with the kernels of :func:`kernel_plan`.
    ``workspace(name, nbytes)`` returns a uint8 device buffer of at least
    nbytes that stays the same between calls of the same size.  ``picks``:
    the picks these experts get (default routing.P; smaller when routing
    covers other ranks' experts too), for the choice of kernels."""
    ex, P = experts, routing.P
    plan = kernel_plan(ex, P if picks is None else picks, gemm_min_rows)
    for kind, rows in plan:
        if kind == "decode":
            D.moe_decode(ex.table, ex.E, ex.H, ex.I, ex.gs, ex.fmt_gu, ex.fmt_down, x, row_exp, routing, y,
                         workspace("decode", D.decode_workspace_bytes(P, ex.I)), max_rows=rows, status=status)
        else:
            D.moe_prefill(ex.table, ex.eexp, ex.E, ex.H, ex.I, ex.gs, ex.fmt_gu, ex.fmt_down, x, row_exp, routing,
                          y, workspace("prefill", D.prefill_workspace_bytes(P, ex.H, ex.I, ex.fmt_gu)),
                          min_rows=rows, status=status)


class _Buffers:
    def __init__(self, T: int, E: int, k: int, H: int, I: int, dev):
        P = T * k
        self.logits = torch.empty((T, E), dtype=torch.float32, device=dev)
        self.row_exp = torch.empty(T, dtype=torch.int32, device=dev)
        self.idx = torch.empty((T, k), dtype=torch.int32, device=dev)
        self.w = torch.empty((T, k), dtype=torch.float32, device=dev)
        self.routing = D.Routing(T, k, E, dev)
        self.y = torch.empty((max(P, 1), H), dtype=torch.float32, device=dev)
        self.ws = torch.empty(D.decode_workspace_bytes(P, I), dtype=torch.uint8, device=dev)
        self.rws = torch.empty(D.router_workspace_bytes(T, H, E), dtype=torch.uint8, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.out = torch.empty((T, H), dtype=torch.float32, device=dev)
        self.pws = None     # grouped-GEMM workspace, made on first use


class MoELayer:
    """``router`` (E, H) f32 on the device; ``experts`` the layer's packed experts.

    Once the layer's picks average ``gemm_min_rows`` per expert (prefill-sized
    batches) every expert runs as a grouped GEMM on the tensor cores (f16
    operands, f32 accumulation; the reference's dense path for 8 or more
    rows, experts.py:148-151, 216-219), below that through the f32-exact
    decode mat-vecs (see kernel_plan); ``gemm_min_rows=0`` keeps every expert
    on the decode kernels."""

    def __init__(self, router: torch.Tensor, experts: LayerExperts, top_k: int, normalize: bool = True,
                 gemm_min_rows: int = GEMM_MIN_ROWS):
        self.router = router.contiguous()
        self.experts = experts
        self.E, self.H, self.I = experts.E, experts.H, experts.I
        self.k, self.normalize = top_k, normalize
        self.gemm_min_rows = int(gemm_min_rows)
        self._bufs: dict[int, _Buffers] = {}

    def uses_gemm(self, T: int) -> bool:
        """Whether the grouped-GEMM kernels run for T tokens."""
        return any(kind == "gemm" for kind, _ in self.kernel_plan(T))

    def kernel_plan(self, T: int) -> list:
        """The expert kernels run for T tokens (see :func:`kernel_plan`)."""
        return kernel_plan(self.experts, T * self.k, self.gemm_min_rows)

    def buffers(self, T: int) -> _Buffers:
        b = self._bufs.get(T)
        if b is None:
            b = self._bufs[T] = _Buffers(T, self.E, self.k, self.H, self.I, self.router.device)
        return b

    def route(self, x: torch.Tensor) -> _Buffers:
        b = self.buffers(x.shape[0])
        D.router_route(x, self.router, self.k, self.normalize, b.idx, b.w, b.logits, b.row_exp, b.rws)
        D.permute(b.idx, b.w, self.E, b.routing)
        return b

    def experts_forward(self, x: torch.Tensor, b: _Buffers) -> None:
        def workspace(name, nbytes):
            if name == "decode":
                return b.ws
            if b.pws is None:
                b.pws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
            return b.pws
        run_experts(self.experts, x, b.row_exp, b.routing, b.y, workspace, b.status, self.gemm_min_rows)

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """out (T, H) = sum over each token's k picks of weight * expert(x)."""
        x = x.contiguous()
        b = self.route(x)
        self.experts_forward(x, b)
        T = x.shape[0]
        return D.combine(b.y, b.routing.inv, b.w.view(-1), T, self.k, out=b.out if out is None else out)

    __call__ = forward

    def capture(self, x: torch.Tensor, experts_only: bool = False) -> torch.cuda.CUDAGraph:
        """A CUDA graph of forward(x) (or of the expert kernels alone, on the
        routing of the last forward of this x) on x's current contents; replay
        it after writing new inputs into x.  Output: buffers(T).out."""
        b = self.buffers(x.shape[0])
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):          # warm-up outside capture (one-time set-up calls)
            self.forward(x)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            if experts_only:
                self.experts_forward(x, b)
            else:
                self.forward(x)
        return g

    def status(self, T: int) -> int:
        """The kernels' status word for token count T (0 = no failure)."""
        return int(self.buffers(T).status.item())
