"""Projection plans: many int4 g64 verify projections in one persistent launch.

The reference runs one Metal kernel per quantized linear of the verify
forward (``dflash_mlx/verify_linear.py:266-286`` -> ``verify_qmm.py``).  On
B200 the projections of a decoder layer (or a whole layer stack) go through
one launch of ``dfl_qmm_plan_run``: the weights of the next projection
stream from HBM while the current one drains, and a projection that reads
an earlier one's output waits for it on the device (``dep``).

* :func:`tile_weight` -- load-time repack of MLX-packed weights into the
  tiled layout the plan kernel streams (36 KB contiguous blocks).  Scales
  below 2^-5 (the common case) select the kernel's subnormal dequantiser;
  both dequantisers give the reference's ``nib * s + b`` rounded to bf16.
* :class:`ProjectionPlan` -- phases (x, tiled weight, y, SiLU, dep) encoded
  once, run many times (CUDA-graph capturable: the run allocates nothing).
* :func:`qmm_tiled` -- one projection through a one-phase plan.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from . import _lib
from ._runtime import as_u32_bits, require_cuda, stream_ptr

PHASE_SILU = 1
PHASE_SUBNORMAL = 2
PHASE_GROUPED = 4
PHASE_SCATTER = 8
MAX_ROWS = 128          # token rows per phase (one token tile of the plan kernel)
MAX_GROUPED_ROWS = 256  # sorted rows of a grouped phase (all problems together)
MAX_PROBLEM_ROWS = 32   # rows of one problem (plans with grouped phases use <= 32-row tiles)
SUBNORMAL_SCALE_LIMIT = 2.0 ** -5


class _Phase(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("y", ctypes.c_void_p), ("w_tiled", ctypes.c_void_p),
                ("M", ctypes.c_int), ("K", ctypes.c_int), ("N", ctypes.c_int),
                ("ldx", ctypes.c_int), ("ldy", ctypes.c_int), ("flags", ctypes.c_int),
                ("dep", ctypes.c_int), ("route", ctypes.c_void_p), ("experts", ctypes.c_int),
                ("problem_rows", ctypes.c_int)]


@dataclass
class TiledWeight:
    """A weight [N, K] in the plan kernel's tiled layout (``blob`` uint8);
    ``experts`` > 1: that many [N, K] weights tiled one after the other (the
    stacked experts of a grouped phase)."""
    blob: torch.Tensor
    n: int
    k: int
    subnormal: bool
    experts: int = 1


def scales_fit_subnormal(scales: torch.Tensor) -> bool:
    """True when every scale is finite with magnitude below 2^-5 (the
    subnormal dequantiser's range).  Reads one value back to the host."""
    s = scales.float()
    return bool(torch.isfinite(s).all().item()) and float(s.abs().max().item()) < SUBNORMAL_SCALE_LIMIT


def tiled_bytes(n: int, k: int) -> int:
    return int(_lib.load().dfl_w4_tiled_bytes(int(n), int(k)))


def sorted_route_ints() -> int:
    """int32 entries of a sorted route table (dfl_moe_sorted_route_ints)."""
    return int(_lib.load().dfl_moe_sorted_route_ints())


def tile_weight(w_q: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, *,
                subnormal: Optional[bool] = None) -> TiledWeight:
    """MLX-packed ``w_q`` uint32 [N, K/8] + bf16 ``scales`` / ``biases``
    [N, K/64] -> :class:`TiledWeight`.  ``subnormal=None`` checks the scales."""
    for t, name in ((w_q, "w"), (scales, "scales"), (biases, "biases")):
        require_cuda(t, name)
    if scales.dtype != torch.bfloat16 or biases.dtype != torch.bfloat16:
        raise NotImplementedError("the tiled layout takes bfloat16 scales and biases")
    w_q = as_u32_bits(w_q)
    n, k = int(w_q.shape[0]), int(w_q.shape[1]) * 8
    if k % 64 != 0:
        raise ValueError(f"K={k} must be a multiple of 64")
    scales, biases = scales.contiguous(), biases.contiguous()
    if tuple(scales.shape) != (n, k // 64) or tuple(biases.shape) != (n, k // 64):
        raise ValueError("scales/biases must be [N, K/64]")
    if subnormal is None:
        subnormal = scales_fit_subnormal(scales)
    nbytes = tiled_bytes(n, k)
    blob = torch.empty(nbytes, dtype=torch.uint8, device=w_q.device)
    with torch.cuda.device(w_q.device):
        st = _lib.load().dfl_repack_w4_tiled(w_q.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                                             n, k, 1 if subnormal else 0, blob.data_ptr(), nbytes,
                                             stream_ptr(w_q.device))
    _lib.check("dfl_repack_w4_tiled", st)
    return TiledWeight(blob, n, k, bool(subnormal))


def tile_expert_stack(w_q: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, *,
                      subnormal: Optional[bool] = None) -> TiledWeight:
    """Stacked experts ``w_q`` [E, N, K/8] + bf16 ``scales`` / ``biases``
    [E, N, K/64] (N % 128 == 0) -> one :class:`TiledWeight` with the experts'
    tiled blocks one after the other (the weight of a grouped phase)."""
    for t, name in ((w_q, "w"), (scales, "scales"), (biases, "biases")):
        require_cuda(t, name)
    if w_q.dim() != 3:
        raise ValueError(f"expert weights must be [E, N, K/8], got {tuple(w_q.shape)}")
    e, n, k = int(w_q.shape[0]), int(w_q.shape[1]), int(w_q.shape[2]) * 8
    if n % 128 != 0:
        raise ValueError(f"grouped phases need N % 128 == 0 (whole tiles per expert), got N={n}")
    if subnormal is None:
        subnormal = scales_fit_subnormal(scales)
    per = tiled_bytes(n, k)
    blob = torch.empty(e * per, dtype=torch.uint8, device=w_q.device)
    lib = _lib.load()
    w_q = as_u32_bits(w_q)
    scales, biases = scales.contiguous(), biases.contiguous()
    if tuple(scales.shape) != (e, n, k // 64) or tuple(biases.shape) != (e, n, k // 64):
        raise ValueError("scales/biases must be [E, N, K/64]")
    if scales.dtype != torch.bfloat16 or biases.dtype != torch.bfloat16:
        raise NotImplementedError("the tiled layout takes bfloat16 scales and biases")
    with torch.cuda.device(w_q.device):
        for i in range(e):
            st = lib.dfl_repack_w4_tiled(w_q[i].data_ptr(), scales[i].data_ptr(), biases[i].data_ptr(),
                                         n, k, 1 if subnormal else 0, blob[i * per:].data_ptr(), per,
                                         stream_ptr(w_q.device))
            _lib.check("dfl_repack_w4_tiled", st)
    return TiledWeight(blob, n, k, bool(subnormal), experts=e)


@dataclass
class PlanPhase:
    """One projection of a plan: ``y = x @ W.T`` (or ``silu(gate) * up`` with
    ``silu`` over gate/up rows interleaved by ``interleave_gate_up``); ``dep``
    = index of an earlier phase whose outputs ``x`` reads (-1: none).

    Grouped phase (``route`` given, the int32 table of
    :func:`dflash_mlx_b200.moe.sort_pairs`): ``x`` / ``y`` are the sorted
    rows of every problem (up to 256), ``weight`` a stack of experts
    (:func:`tile_expert_stack`) and problem i multiplies its rows by its
    expert's weight; ``problem_rows`` bounds the rows of one problem (<= 32,
    and a plan with grouped phases takes at most 32 rows in its dense ones);
    ``scatter`` writes sorted row r to ``y`` row ``route[514 + r]``."""
    x: torch.Tensor
    weight: TiledWeight
    y: torch.Tensor
    silu: bool = False
    dep: int = -1
    route: Optional[torch.Tensor] = None
    problem_rows: int = 0
    scatter: bool = False


def _check_rows(t: torch.Tensor, name: str, cols: int) -> int:
    if t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a bfloat16 [rows, cols] tensor with unit column stride")
    if t.shape[1] != cols:
        raise ValueError(f"{name} has {t.shape[1]} columns, expected {cols}")
    return int(t.stride(0))


class ProjectionPlan:
    """A sequence of projections encoded once and launched as one kernel.

    The tensors' addresses are baked into the plan: keep them (the plan holds
    references) and write new inputs into them in place between runs."""

    def __init__(self, phases: Sequence[PlanPhase]):
        if not phases:
            raise ValueError("a plan needs at least one phase")
        lib = _lib.load()
        dev = phases[0].x.device
        arr = (_Phase * len(phases))()
        for i, ph in enumerate(phases):
            for t, name in ((ph.x, "x"), (ph.y, "y"), (ph.weight.blob, "weight")):
                require_cuda(t, name)
                if t.device != dev:
                    raise ValueError("every tensor of a plan must be on one device")
            w = ph.weight
            m = int(ph.x.shape[0])
            grouped = ph.route is not None
            if grouped:
                require_cuda(ph.route, "route")
                if ph.route.dtype != torch.int32 or ph.route.numel() < sorted_route_ints():
                    raise ValueError(f"phase {i}: route must be the int32 table of sort_pairs")
                if not 1 <= m <= MAX_GROUPED_ROWS:
                    raise ValueError(f"phase {i}: {m} sorted rows (1..{MAX_GROUPED_ROWS})")
                if not 1 <= ph.problem_rows <= MAX_PROBLEM_ROWS:
                    raise ValueError(f"phase {i}: problem_rows must be 1..{MAX_PROBLEM_ROWS}")
                if w.n % 128 != 0:
                    raise ValueError(f"phase {i}: grouped phases need N % 128 == 0")
            elif ph.scatter:
                raise ValueError(f"phase {i}: scatter needs a route table (grouped phase)")
            elif not 1 <= m <= MAX_ROWS:
                raise ValueError(f"phase {i}: {m} rows (a plan takes 1..{MAX_ROWS} rows per phase; "
                                 "split more rows into one phase per token tile)")
            ldx = _check_rows(ph.x, f"phase {i} x", w.k)
            n_out = w.n // 2 if ph.silu else w.n
            ldy = _check_rows(ph.y, f"phase {i} y", n_out)
            if int(ph.y.shape[0]) != m:
                raise ValueError(f"phase {i}: y has {ph.y.shape[0]} rows, x has {m}")
            if ph.silu and w.n % 32 != 0:
                raise ValueError(f"phase {i}: SiLU needs N % 32 == 0 (interleaved gate/up rows)")
            if not -1 <= ph.dep < i:
                raise ValueError(f"phase {i}: dep {ph.dep} must name an earlier phase or be -1")
            flags = (PHASE_SILU if ph.silu else 0) | (PHASE_SUBNORMAL if w.subnormal else 0)
            if grouped:
                flags |= PHASE_GROUPED | (PHASE_SCATTER if ph.scatter else 0)
            arr[i] = _Phase(ph.x.data_ptr(), ph.y.data_ptr(), w.blob.data_ptr(), m, w.k, w.n,
                            ldx, ldy, flags, int(ph.dep),
                            ph.route.data_ptr() if grouped else None, w.experts if grouped else 0,
                            int(ph.problem_rows) if grouped else 0)
        nbytes = int(lib.dfl_qmm_plan_bytes(len(phases)))
        if nbytes == 0:
            raise ValueError(f"{len(phases)} phases is outside the plan limit")
        self._host = (ctypes.c_uint8 * nbytes)()
        with torch.cuda.device(dev):
            st = lib.dfl_qmm_plan_encode(arr, len(phases), self._host, nbytes)
            _lib.check("dfl_qmm_plan_encode", st)
            status = ctypes.c_int(0)
            ws_bytes = int(lib.dfl_qmm_plan_workspace_bytes(self._host, ctypes.byref(status)))
            _lib.check("dfl_qmm_plan_workspace_bytes", status.value)
            host_t = torch.frombuffer(bytearray(self._host), dtype=torch.uint8)
            self.plan_dev = host_t.to(dev)
            self.workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        self.device = dev
        self.phases: List[PlanPhase] = list(phases)

    def run(self) -> None:
        """Launch the plan on the current stream of its device."""
        with torch.cuda.device(self.device):
            st = _lib.load().dfl_qmm_plan_run(self._host, self.plan_dev.data_ptr(),
                                              self.workspace.data_ptr(), self.workspace.numel(),
                                              stream_ptr(self.device))
        _lib.check("dfl_qmm_plan_run", st)

    def reset_workspace(self) -> None:
        """Zero the workspace again (needed after a reported device error)."""
        self.workspace.zero_()

    def set_test_fault(self, skip_partial_cta: int = -1, wait_limit_ns: int = 1_000_000_000) -> None:
        """Tests only: make CTA ``skip_partial_cta`` withhold its split-K
        partials and bound every wait by ``wait_limit_ns`` (the run then ends
        with a device error instead of results); -1 / 1 s restore normal runs."""
        _lib.check("dfl_qmm_plan_set_test_fault",
                   _lib.load().dfl_qmm_plan_set_test_fault(self._host, int(skip_partial_cta),
                                                           int(wait_limit_ns)))

    def last_timeout(self):
        """(role, phase, cta) of the first wait that ran out in the last run,
        role 0 when none did (reads the workspace back to the host)."""
        words = self.workspace[:64 * 1024].cpu().numpy()
        role, phase, cta = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
        _lib.check("dfl_qmm_plan_last_timeout",
                   _lib.load().dfl_qmm_plan_last_timeout(words.ctypes.data, ctypes.byref(role),
                                                         ctypes.byref(phase), ctypes.byref(cta)))
        return role.value, phase.value, cta.value


def qmm_tiled(x: torch.Tensor, weight: TiledWeight, out: Optional[torch.Tensor] = None, *,
              silu: bool = False) -> torch.Tensor:
    """``x [M, K] @ W.T`` (or the fused SiLU*up) through a plan with one
    phase per token tile of up to 128 rows."""
    require_cuda(x, "x")
    if x.dtype != torch.bfloat16:
        raise NotImplementedError("the plan kernel takes bfloat16 activations")
    x = x.contiguous()
    m = int(x.shape[0])
    n_out = weight.n // 2 if silu else weight.n
    if out is None:
        out = torch.empty((m, n_out), dtype=torch.bfloat16, device=x.device)
    # the plan's device buffers are freed to torch's stream-ordered allocator
    # after the launch is queued, so they are not reused before it ran
    ProjectionPlan([PlanPhase(x[r0:r0 + MAX_ROWS], weight, out[r0:r0 + MAX_ROWS], silu=silu)
                    for r0 in range(0, m, MAX_ROWS)]).run()
    return out
