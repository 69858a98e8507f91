"""MoE verify expert block on B200 (routed experts + shared expert).

Restates mlx-lm's ``SwitchGLU`` / ``SwitchLinear`` -> ``mx.gather_qmm`` path
(third party: mlx-lm >= 0.31.0, not vendored in the reference) that the
reference reaches from the decoder layers at
``dflash_mlx/engine/target_qwen_gdn.py:863-865``:

1. ``route``: top-k experts per token by router logit, softmax over the k kept
   logits (= softmax over all experts, then renormalised), and a device-side
   route table of the active experts and their tokens;
2. ``gate``/``up`` = grouped int4 qmm over the active experts (each expert's
   weights are read once), ``h = silu(gate) * up``;
3. ``down`` = grouped int4 qmm on the (token, slot) rows of h;
4. ``y_t = sum_j w[t, j] * down[t, j] + shared_expert(x_t)``.

Every intermediate is rounded to bf16 as the MLX ops return it; the combine
accumulates in fp32 in slot order.  Nothing is synchronised with the host.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._runtime import require_cuda, stream_ptr, workspace
from .verify_qmm import qmm_w4g64


@dataclass
class QuantWeight:
    """One affine int4 g64 weight: ``q`` uint32 ``[.., N, K/8]``, bf16 ``s``/``b`` ``[.., N, K/64]``."""

    q: torch.Tensor
    s: torch.Tensor
    b: torch.Tensor

    @property
    def n(self) -> int:
        return int(self.q.shape[-2])

    @property
    def k(self) -> int:
        return int(self.q.shape[-1]) * 8


def _check_stack(w: QuantWeight, name: str) -> None:
    """An expert stack: contiguous CUDA ``q`` int32/uint32 ``[E, N, K/8]`` and
    bf16 ``s``/``b`` ``[E, N, K/64]`` (the grouped kernel's tensor maps assume
    exactly this layout)."""
    for part, t in (("q", w.q), ("s", w.s), ("b", w.b)):
        require_cuda(t, f"{name}.{part}")
        if not t.is_contiguous():
            raise ValueError(f"{name}.{part} must be contiguous")
    if w.q.dim() != 3 or w.q.dtype not in (torch.int32, torch.uint32):
        raise ValueError(f"{name}.q must be int32/uint32 [E, N, K/8], got {w.q.dtype} {tuple(w.q.shape)}")
    e, n, k8 = w.q.shape
    if k8 % 8 != 0:
        raise ValueError(f"{name}: K = {8 * k8} is not a multiple of the group size 64")
    for part, t in (("s", w.s), ("b", w.b)):
        if t.dtype != torch.bfloat16 or tuple(t.shape) != (e, n, k8 // 8):
            raise ValueError(f"{name}.{part} must be bf16 {(e, n, k8 // 8)}, got {t.dtype} {tuple(t.shape)}")


def _moe_ws_bytes(max_problems: int, k: int, n: int) -> int:
    st = ctypes.c_int(0)
    nb = _lib.load().dfl_moe_qmm_workspace_bytes(int(max_problems), int(k), int(n), ctypes.byref(st))
    _lib.check("dfl_moe_qmm_workspace_bytes", st.value)
    return int(nb)


def route(router_logits: torch.Tensor, top_k: int = 8):
    """Returns (route_table int32, weights fp32 [T, k], topk_ids int32 [T, k])."""
    require_cuda(router_logits, "router_logits")
    lg = router_logits.to(torch.float32).contiguous()
    t, e = lg.shape
    dev = lg.device
    table = torch.empty(int(_lib.load().dfl_moe_route_table_ints(e)), dtype=torch.int32, device=dev)
    w = torch.empty((t, top_k), dtype=torch.float32, device=dev)
    ids = torch.empty((t, top_k), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = _lib.load().dfl_moe_route(lg.data_ptr(), t, e, int(top_k), table.data_ptr(),
                                       w.data_ptr(), ids.data_ptr(), stream_ptr(dev))
    _lib.check("dfl_moe_route", st)
    return table, w, ids


def gather_qmm(x: torch.Tensor, weight: QuantWeight, table: torch.Tensor, *, rows_out: int,
               gather_by_pair: bool, max_problems: Optional[int] = None,
               out: Optional[torch.Tensor] = None, silu: bool = False,
               table_ready: bool = False) -> torch.Tensor:
    """Grouped int4 qmm over the route table's active experts -> bf16 ``[rows_out, N]``.

    ``silu=True``: each expert's weights are its gate/up pair interleaved
    (:func:`fuse_expert_gate_up`) and the result is ``silu(gate) * up``,
    ``[rows_out, N/2]``.  ``table_ready``: the route table was complete before
    the previous launch on the stream started, so weights may stream early."""
    require_cuda(x, "x")
    require_cuda(table, "table")
    _check_stack(weight, "weight")
    e = int(weight.q.shape[0])
    k, n = weight.k, weight.n
    if x.dim() != 2 or x.dtype != torch.bfloat16 or x.shape[1] != k:
        raise ValueError(f"x must be bf16 [rows, {k}], got {x.dtype} {tuple(x.shape)}")
    if gather_by_pair and x.shape[0] < rows_out:
        raise ValueError(f"gather_by_pair reads one x row per output row: {x.shape[0]} < {rows_out}")
    if table.dtype != torch.int32 or table.numel() < int(_lib.load().dfl_moe_route_table_ints(e)):
        raise ValueError("table must be the int32 route table of route() for this expert count")
    x = x.contiguous()
    n_out = n // 2 if silu else n
    if out is None:
        out = torch.empty((rows_out, n_out), dtype=torch.bfloat16, device=x.device)
    elif out.dtype != torch.bfloat16 or tuple(out.shape) != (rows_out, n_out) or not out.is_contiguous():
        raise ValueError(f"out must be contiguous bf16 {(rows_out, n_out)}")
    mp = e if max_problems is None else int(max_problems)
    entry = "dfl_moe_qmm_w4g64_silu" if silu else "dfl_moe_qmm_w4g64"
    with torch.cuda.device(x.device):
        ws = workspace(x.device, _moe_ws_bytes(mp, k, n))
        st = getattr(_lib.load(), entry)(
            x.data_ptr(), weight.q.data_ptr(), weight.s.data_ptr(), weight.b.data_ptr(),
            out.data_ptr(), table.data_ptr(), (1 if gather_by_pair else 0) | (2 if table_ready else 0),
            mp, e, k, n,
            ws.data_ptr(), ws.numel(), stream_ptr(x.device))
    _lib.check(entry, st)
    return out


def fuse_expert_gate_up(gate: QuantWeight, up: QuantWeight) -> QuantWeight:
    """Stacked expert gate and up weights ``[E, I, *]`` interleaved per expert in
    16-row blocks -> ``[E, 2I, *]`` (the layout of ``gather_qmm(..., silu=True)``)."""
    from .verify_qmm import interleave_gate_up

    return QuantWeight(interleave_gate_up(gate.q, up.q, dim=-2).contiguous(),
                       interleave_gate_up(gate.s, up.s, dim=-2).contiguous(),
                       interleave_gate_up(gate.b, up.b, dim=-2).contiguous())


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``bf16(silu(gate) * up)`` (fp32 math).  2-D ``gate``/``up`` may be
    row-strided views with the same row stride (e.g. the two halves of a
    fused gate|up projection output); the result is contiguous."""
    require_cuda(gate, "gate")
    require_cuda(up, "up")
    if gate.dtype != torch.bfloat16 or up.dtype != torch.bfloat16:
        raise ValueError(f"silu_mul takes bf16 gate and up, got {gate.dtype} and {up.dtype}")
    if gate.shape != up.shape:
        raise ValueError(f"gate {tuple(gate.shape)} and up {tuple(up.shape)} differ")
    if (gate.dim() == 2 and gate.stride() == up.stride() and gate.stride(1) == 1
            and not (gate.is_contiguous() and up.is_contiguous())):
        rows, cols = gate.shape
        out = torch.empty((rows, cols), dtype=gate.dtype, device=gate.device)
        with torch.cuda.device(gate.device):
            st = _lib.load().dfl_silu_mul_rows_bf16(gate.data_ptr(), up.data_ptr(), gate.stride(0),
                                                    out.data_ptr(), rows, cols, stream_ptr(gate.device))
        _lib.check("dfl_silu_mul_rows_bf16", st)
        return out
    gate = gate.contiguous()
    out = torch.empty_like(gate)
    with torch.cuda.device(gate.device):
        st = _lib.load().dfl_silu_mul_bf16(gate.data_ptr(), up.contiguous().data_ptr(), out.data_ptr(),
                                           gate.numel(), stream_ptr(gate.device))
    _lib.check("dfl_silu_mul_bf16", st)
    return out


def combine(pair_out: torch.Tensor, weights: torch.Tensor, shared: Optional[torch.Tensor]) -> torch.Tensor:
    """``y[t] = sum_j weights[t, j] * pair_out[t * k + j] (+ shared[t])``, bf16 ``[T, H]``."""
    require_cuda(pair_out, "pair_out")
    require_cuda(weights, "weights")
    if weights.dim() != 2 or weights.dtype != torch.float32:
        raise ValueError(f"weights must be fp32 [T, k], got {weights.dtype} {tuple(weights.shape)}")
    t, k = weights.shape
    h = pair_out.shape[-1]
    if pair_out.dtype != torch.bfloat16 or tuple(pair_out.shape) != (t * k, h) or not pair_out.is_contiguous():
        raise ValueError(f"pair_out must be contiguous bf16 {(t * k, h)}, got {tuple(pair_out.shape)}")
    if shared is not None:
        require_cuda(shared, "shared")
        if shared.dtype != torch.bfloat16 or tuple(shared.shape) != (t, h):
            raise ValueError(f"shared must be bf16 {(t, h)}, got {shared.dtype} {tuple(shared.shape)}")
    y = torch.empty((t, h), dtype=torch.bfloat16, device=pair_out.device)
    with torch.cuda.device(y.device):
        st = _lib.load().dfl_moe_combine(pair_out.data_ptr(), weights.contiguous().data_ptr(),
                                         None if shared is None else shared.contiguous().data_ptr(),
                                         y.data_ptr(), t, k, h, stream_ptr(y.device))
    _lib.check("dfl_moe_combine", st)
    return y


def dense_mlp_fused(x: torch.Tensor, gate_up: QuantWeight, down: QuantWeight) -> torch.Tensor:
    """The shared-expert MLP on an interleaved gate/up weight (MLX packing):
    one fused gate/up + SiLU launch, then down."""
    from .verify_qmm import gate_up_silu

    h = gate_up_silu(x.contiguous(), gate_up.q, gate_up.s, gate_up.b, layout="mlx")
    return qmm_w4g64(h, down.q, down.s, down.b)


def dense_mlp(x: torch.Tensor, gate: QuantWeight, up: QuantWeight, down: QuantWeight) -> torch.Tensor:
    g = qmm_w4g64(x, gate.q, gate.s, gate.b)
    u = qmm_w4g64(x, up.q, up.s, up.b)
    return qmm_w4g64(silu_mul(g, u), down.q, down.s, down.b)


def moe_layer(x: torch.Tensor, router_logits: torch.Tensor, experts: dict, shared: Optional[dict],
              top_k: int = 8) -> torch.Tensor:
    """One MoE verify layer: ``x`` bf16 ``[T, H]`` -> bf16 ``[T, H]``.

    ``experts``: QuantWeight stacks ``gate`` / ``up`` ``[E, I, H/8]`` (or one
    interleaved ``gate_up`` stack ``[E, 2I, H/8]``, :func:`fuse_expert_gate_up`)
    and ``down`` ``[E, H, I/8]``; ``shared``: unstacked QuantWeights ``gate`` /
    ``up`` (or an interleaved ``gate_up``) and ``down``, or None.
    """
    require_cuda(x, "x")
    t = x.shape[0]
    table, w, _ = route(router_logits, top_k)
    # The shared expert does not depend on the routing: run it first, so the
    # grouped launches after it find the route table already complete and can
    # stream their weights while the launch before them finishes.
    so = None
    if shared is not None:
        if "gate_up" in shared:
            so = dense_mlp_fused(x, shared["gate_up"], shared["down"])
        else:
            so = dense_mlp(x, shared["gate"], shared["up"], shared["down"])
    ready = shared is not None
    fused = "gate_up" in experts
    e = int((experts["gate_up"] if fused else experts["gate"]).q.shape[0])
    mp = min(e, t * top_k)
    if fused:
        h = gather_qmm(x, experts["gate_up"], table, rows_out=t * top_k, gather_by_pair=False,
                       max_problems=mp, silu=True, table_ready=ready)
    else:
        g = gather_qmm(x, experts["gate"], table, rows_out=t * top_k, gather_by_pair=False,
                       max_problems=mp, table_ready=ready)
        u = gather_qmm(x, experts["up"], table, rows_out=t * top_k, gather_by_pair=False, max_problems=mp,
                       table_ready=True)
        h = silu_mul(g, u)
    d = gather_qmm(h, experts["down"], table, rows_out=t * top_k, gather_by_pair=True, max_problems=mp,
                   table_ready=True)
    return combine(d, w, so)


def sort_pairs(topk_ids: torch.Tensor, x: torch.Tensor, n_experts: int, *,
               route_out: Optional[torch.Tensor] = None, x_sorted: Optional[torch.Tensor] = None,
               x_copy: Optional[torch.Tensor] = None):
    """Sorted route table of grouped plan phases + the x rows in sorted order.

    ``topk_ids`` int32 ``[T, k]`` (from :func:`route`), ``x`` bf16 ``[T, H]``
    -> (``route`` int32, ``x_sorted`` bf16 ``[T*k, H]``): pairs (token, slot)
    ordered by expert, then pair index; ``route[0]`` active experts P,
    ``route[1 + 2i]`` first sorted row of problem i, ``route[2 + 2i]`` its
    expert, ``route[514 + r]`` the pair row of sorted row r.  ``x_copy``
    (optional, bf16 ``[T, H]``) receives ``x`` in the same launch."""
    from .qmm_plan import sorted_route_ints

    require_cuda(topk_ids, "topk_ids")
    require_cuda(x, "x")
    if topk_ids.dtype != torch.int32 or topk_ids.dim() != 2 or not topk_ids.is_contiguous():
        raise ValueError("topk_ids must be a contiguous int32 [T, k] tensor")
    t, k = (int(v) for v in topk_ids.shape)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[0] != t or x.stride(1) != 1:
        raise ValueError(f"x must be bf16 [{t}, H] with unit column stride")
    h = int(x.shape[1])
    dev = x.device
    if route_out is None:
        route_out = torch.empty(sorted_route_ints(), dtype=torch.int32, device=dev)
    elif route_out.dtype != torch.int32 or route_out.numel() < sorted_route_ints():
        raise ValueError("route_out must be int32 with dfl_moe_sorted_route_ints() entries")
    if x_sorted is None:
        x_sorted = torch.empty((t * k, h), dtype=torch.bfloat16, device=dev)
    elif x_sorted.dtype != torch.bfloat16 or tuple(x_sorted.shape) != (t * k, h) or not x_sorted.is_contiguous():
        raise ValueError(f"x_sorted must be contiguous bf16 {(t * k, h)}")
    if x_copy is not None and (x_copy.dtype != torch.bfloat16 or tuple(x_copy.shape) != (t, h)
                               or not x_copy.is_contiguous()):
        raise ValueError(f"x_copy must be contiguous bf16 {(t, h)}")
    with torch.cuda.device(dev):
        st = _lib.load().dfl_moe_sort_pairs(topk_ids.data_ptr(), t, k, int(n_experts), x.data_ptr(),
                                            int(x.stride(0)), h, route_out.data_ptr(), x_sorted.data_ptr(),
                                            None if x_copy is None else x_copy.data_ptr(), stream_ptr(dev))
    _lib.check("dfl_moe_sort_pairs", st)
    return route_out, x_sorted


def route_sorted(router_logits: torch.Tensor, x: torch.Tensor, top_k: int, *,
                 route_out: torch.Tensor, x_sorted: torch.Tensor, x_copy: Optional[torch.Tensor] = None,
                 weights_out: Optional[torch.Tensor] = None, ids_out: Optional[torch.Tensor] = None,
                 shared_expert: bool = False):
    """:func:`route` and :func:`sort_pairs` in one launch -> (weights fp32
    ``[T, k]``, topk_ids int32 ``[T, k]``); the sorted route table, rows and
    x copy go to ``route_out`` / ``x_sorted`` / ``x_copy``.
    ``shared_expert``: one more problem, expert E (a shared expert stacked
    after the routed ones), over the T tokens themselves (``x_sorted`` rows
    ``T*k .. T*k+T-1``, scattered to pair rows ``T*k + t``)."""
    from .qmm_plan import sorted_route_ints

    require_cuda(router_logits, "router_logits")
    require_cuda(x, "x")
    lg = router_logits.to(torch.float32).contiguous()
    t, e = (int(v) for v in lg.shape)
    k = int(top_k)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[0] != t or x.stride(1) != 1:
        raise ValueError(f"x must be bf16 [{t}, H] with unit column stride")
    h = int(x.shape[1])
    dev = x.device
    if route_out.dtype != torch.int32 or route_out.numel() < sorted_route_ints():
        raise ValueError("route_out must be int32 with dfl_moe_sorted_route_ints() entries")
    rows = t * k + (t if shared_expert else 0)
    if x_sorted.dtype != torch.bfloat16 or tuple(x_sorted.shape) != (rows, h) or not x_sorted.is_contiguous():
        raise ValueError(f"x_sorted must be contiguous bf16 {(rows, h)}")
    if x_copy is not None and (x_copy.dtype != torch.bfloat16 or tuple(x_copy.shape) != (t, h)
                               or not x_copy.is_contiguous()):
        raise ValueError(f"x_copy must be contiguous bf16 {(t, h)}")
    w = weights_out if weights_out is not None else torch.empty((t, k), dtype=torch.float32, device=dev)
    ids = ids_out if ids_out is not None else torch.empty((t, k), dtype=torch.int32, device=dev)
    if w.dtype != torch.float32 or tuple(w.shape) != (t, k) or not w.is_contiguous():
        raise ValueError(f"weights_out must be contiguous fp32 {(t, k)}")
    if ids.dtype != torch.int32 or tuple(ids.shape) != (t, k) or not ids.is_contiguous():
        raise ValueError(f"ids_out must be contiguous int32 {(t, k)}")
    with torch.cuda.device(dev):
        st = _lib.load().dfl_moe_route_sorted(lg.data_ptr(), t, e, k, 1 if shared_expert else 0, x.data_ptr(),
                                              int(x.stride(0)), h,
                                              route_out.data_ptr(), w.data_ptr(), ids.data_ptr(),
                                              x_sorted.data_ptr(),
                                              None if x_copy is None else x_copy.data_ptr(), stream_ptr(dev))
    _lib.check("dfl_moe_route_sorted", st)
    return w, ids


class MoEPlanLayer:
    """One MoE verify layer with every expert projection in one plan launch.

    Per call: :func:`route_sorted` (top-k + weights, sorted route table, x
    rows in sorted order: one launch), one
    :class:`~dflash_mlx_b200.qmm_plan.ProjectionPlan` run -- gate|up + SiLU
    and down as two grouped phases over the active experts (down scattered
    to pair rows; each active expert's weights read once, the problems of a
    phase spread over all SMs), with a shared expert of the routed experts'
    shape stacked after them as one more problem over all tokens (a shared
    expert of another shape runs as two dense phases of the same plan) --
    and :func:`combine`.  No host synchronisation, CUDA-graph
    capturable.  Same results as :func:`moe_layer` up to fp32
    summation order.  Three launches per call.

    ``experts``: QuantWeight stacks ``gate`` / ``up`` ``[E, I, H/8]`` or an
    interleaved ``gate_up`` (:func:`fuse_expert_gate_up`) and ``down``
    ``[E, H, I/8]``; ``shared``: QuantWeights ``gate`` / ``up`` (or
    ``gate_up``) and ``down``, or None.  ``stack_shared=False`` keeps a
    same-shaped shared expert in dense phases too.  Needs I % 64 == 0,
    H % 128 == 0 and ``tokens * top_k`` <= 240.
    """

    def __init__(self, experts: dict, shared: Optional[dict], tokens: int, top_k: int = 8,
                 stack_shared: bool = True):
        from .qmm_plan import PlanPhase, ProjectionPlan, sorted_route_ints, tile_expert_stack, tile_weight
        from .verify_qmm import interleave_gate_up

        gu = experts["gate_up"] if "gate_up" in experts else fuse_expert_gate_up(experts["gate"], experts["up"])
        down = experts["down"]
        _check_stack(gu, "gate_up")
        _check_stack(down, "down")
        e, h = int(gu.q.shape[0]), gu.k
        inter = gu.n // 2
        if down.k != inter or down.n != h or int(down.q.shape[0]) != e:
            raise ValueError("down must be [E, H, I/8] for gate_up [E, 2I, H/8]")
        t, k = int(tokens), int(top_k)
        if not 1 <= t * k <= 240 or t > 16:
            raise ValueError(f"{t} tokens x top-{k}: the route kernels take <= 16 tokens, <= 240 pairs")
        dev = gu.q.device
        self.tokens, self.top_k, self.experts, self.hidden, self.inter = t, k, e, h, inter
        bf = dict(dtype=torch.bfloat16, device=dev)
        pairs = t * k
        sgu = sdown = None
        if shared is not None:
            if "gate_up" in shared:
                sgu = shared["gate_up"]
            else:
                g, u = shared["gate"], shared["up"]
                sgu = QuantWeight(interleave_gate_up(g.q, u.q).contiguous(),
                                  interleave_gate_up(g.s, u.s).contiguous(),
                                  interleave_gate_up(g.b, u.b).contiguous())
            sdown = shared["down"]
        # a shared expert of the routed experts' shape is stacked after them
        # and runs as one more grouped problem over all T tokens (two plan
        # phases per layer); another shape keeps two dense phases of its own
        self.shared_stacked = (stack_shared and sgu is not None and tuple(sgu.q.shape) == tuple(gu.q.shape[1:])
                               and tuple(sdown.q.shape) == tuple(down.q.shape[1:]))
        if self.shared_stacked:
            cat = lambda st, one: torch.cat([st, one.unsqueeze(0)]).contiguous()  # noqa: E731
            self.gate_up = tile_expert_stack(cat(gu.q, sgu.q), cat(gu.s, sgu.s), cat(gu.b, sgu.b))
            self.down = tile_expert_stack(cat(down.q, sdown.q), cat(down.s, sdown.s), cat(down.b, sdown.b))
        else:
            self.gate_up = tile_expert_stack(gu.q, gu.s, gu.b)
            self.down = tile_expert_stack(down.q, down.s, down.b)
        rows = pairs + (t if self.shared_stacked else 0)
        self.x_in = torch.zeros((t, h), **bf)
        self.x_sorted = torch.zeros((rows, h), **bf)
        self.h_sorted = torch.zeros((rows, inter), **bf)
        self.pair_out = torch.zeros((rows, h), **bf)
        self.route = torch.zeros(sorted_route_ints(), dtype=torch.int32, device=dev)
        self.weights = torch.zeros((t, k), dtype=torch.float32, device=dev)
        self.ids = torch.zeros((t, k), dtype=torch.int32, device=dev)
        phases = []
        self.shared_out = None
        if sgu is not None and not self.shared_stacked:
            self.shared_gate_up = tile_weight(sgu.q, sgu.s, sgu.b)
            self.shared_down = tile_weight(sdown.q, sdown.s, sdown.b)
            self.h_shared = torch.zeros((t, sgu.n // 2), **bf)
            self.shared_out = torch.zeros((t, h), **bf)
            phases.append(PlanPhase(self.x_in, self.shared_gate_up, self.h_shared, silu=True))
        elif self.shared_stacked:
            self.shared_out = self.pair_out[pairs:]
        g_idx = len(phases)
        phases.append(PlanPhase(self.x_sorted, self.gate_up, self.h_sorted, silu=True, route=self.route,
                                problem_rows=t))
        if sgu is not None and not self.shared_stacked:
            phases.append(PlanPhase(self.h_shared, self.shared_down, self.shared_out, dep=0))
        phases.append(PlanPhase(self.h_sorted, self.down, self.pair_out, dep=g_idx, route=self.route,
                                problem_rows=t, scatter=True))
        self.plan = ProjectionPlan(phases)

    def __call__(self, x: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        require_cuda(x, "x")
        if x.dtype != torch.bfloat16 or tuple(x.shape) != (self.tokens, self.hidden):
            raise ValueError(f"x must be bf16 {(self.tokens, self.hidden)}")
        if tuple(router_logits.shape) != (self.tokens, self.experts):
            raise ValueError(f"router_logits must be {(self.tokens, self.experts)}")
        dense_shared = self.shared_out is not None and not self.shared_stacked
        w, _ = route_sorted(router_logits, x, self.top_k, route_out=self.route, x_sorted=self.x_sorted,
                            x_copy=self.x_in if dense_shared else None, weights_out=self.weights,
                            ids_out=self.ids, shared_expert=self.shared_stacked)
        self.plan.run()
        pairs = self.tokens * self.top_k
        return combine(self.pair_out[:pairs], w, self.shared_out)
