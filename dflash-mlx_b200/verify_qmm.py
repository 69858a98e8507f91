"""``verify_matmul``: the int4 verify quantized matmul on B200.

Mirrors ``dflash_mlx/verify_qmm.py:905-1022`` (``verify_matmul``) and
``:15-16`` (``is_enabled``).  Same arguments and weight layout (MLX affine:
uint32 ``w [N, K/8]`` low nibble first, ``scales`` / ``biases`` ``[N, K/64]``),
same result up to fp32 summation order.

Differences by design:

* the reference dispatches between Metal variants and falls back to stock
  ``mx.quantized_matmul`` for anything its verify kernels do not cover; here
  one sm_100a kernel (``dfl_verify_qmm_w4g64``) serves every row count (rows
  are processed 32 at a time), so there is no fallback;
* layouts the kernel does not implement (8-bit, group sizes other than 64,
  ``transpose=False``, non-bf16 activations) raise ``NotImplementedError``
  instead of silently taking another path.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._runtime import as_u32_bits, require_cuda, stream_ptr, workspace
from . import settings as _settings

MAX_ROWS_PER_CALL = 32


def is_enabled() -> bool:
    """``DFLASH_VERIFY_QMM == "1"`` (reference ``verify_qmm.py:15-16``).

    Reports the switch for callers that read it; the sm_100a kernel is the
    only implementation, so it does not change which code runs.
    """
    return _settings.read().qmm


def workspace_bytes(m: int, k: int, n: int) -> int:
    st = ctypes.c_int(0)
    nbytes = _lib.load().dfl_verify_qmm_workspace_bytes(int(m), int(k), int(n), ctypes.byref(st))
    _lib.check("dfl_verify_qmm_workspace_bytes", st.value)
    return int(nbytes)


_ENTRY = {("mlx", torch.bfloat16): "dfl_verify_qmm_w4g64",
          ("mlx", torch.float16): "dfl_verify_qmm_w4g64_f16",
          ("pairs", torch.bfloat16): "dfl_verify_qmm_w4g64_pairs",
          ("pairs", torch.float16): "dfl_verify_qmm_w4g64_pairs_f16"}


def _check_out(out: torch.Tensor, shape: tuple, dtypes, device: torch.device) -> None:
    """A caller-provided output must be exactly what the kernel writes:
    contiguous, of this shape and dtype, on the inputs' device."""
    require_cuda(out, "out")
    dtypes = dtypes if isinstance(dtypes, tuple) else (dtypes,)
    if (out.dtype not in dtypes or tuple(out.shape) != tuple(shape) or not out.is_contiguous()
            or out.device != device):
        raise ValueError(f"out must be a contiguous {dtypes[0]} tensor of shape {tuple(shape)} on {device}, "
                         f"got {out.dtype} {tuple(out.shape)} on {out.device}")


def repack_pairs(w_q: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """MLX-packed int4 weights -> the pair-packed order (``out`` may be ``w_q``).

    In the pair-packed order nibble ``j`` of each uint32 holds column
    ``8p + 2j`` and nibble ``4 + j`` column ``8p + 2j + 1``; the qmm then
    dequantises straight to natural K order and streams x without a
    permutation step.  A load-time layout, like concatenating projections
    that share an input: done once per weight, never per call.
    """
    require_cuda(w_q, "w")
    src = as_u32_bits(w_q)
    if out is None:
        dst = torch.empty_like(src)
    else:
        # written in place: never through a contiguous copy of ``out``
        _check_out(out, tuple(src.shape), (torch.int32, torch.uint32), src.device)
        dst = out
    with torch.cuda.device(src.device):
        st = _lib.load().dfl_repack_w4_pairs(src.data_ptr(), dst.data_ptr(), src.numel(),
                                             stream_ptr(src.device))
    _lib.check("dfl_repack_w4_pairs", st)
    return dst if out is None else out


def qmm_w4g64(x2: torch.Tensor, w_q: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
              out: torch.Tensor | None = None, *, layout: str = "mlx") -> torch.Tensor:
    """``x2 [M, K] @ dequant(w_q).T`` through the C ABI -> ``[M, N]`` in x's dtype.

    Activations, scales and biases are all bfloat16 or all float16 (the two
    kernel instantiations of the reference, ``verify_linear.py:163-164``).
    ``layout`` is ``"mlx"`` (the reference's packing) or ``"pairs"``
    (weights passed through :func:`repack_pairs`)."""
    for t, name in ((x2, "x"), (w_q, "w"), (scales, "scales"), (biases, "biases")):
        require_cuda(t, name)
    if layout not in ("mlx", "pairs"):
        raise ValueError(f"unknown weight layout {layout!r}")
    entry = _ENTRY.get((layout, x2.dtype))
    if entry is None:
        raise NotImplementedError(f"activations must be bfloat16 or float16, got {x2.dtype}")
    if scales.dtype != x2.dtype or biases.dtype != x2.dtype:
        raise NotImplementedError(
            f"scales/biases ({scales.dtype}, {biases.dtype}) must match the activations' {x2.dtype}")
    w_q = as_u32_bits(w_q)
    x2 = x2.contiguous()
    scales = scales.contiguous()
    biases = biases.contiguous()
    m, k = x2.shape
    n = w_q.shape[0]
    if w_q.shape[1] * 8 != k:
        raise ValueError(f"weight shape {tuple(w_q.shape)} does not match K={k}")
    if scales.shape != (n, k // 64) or biases.shape != (n, k // 64):
        raise ValueError("scales/biases must be [N, K/64]")
    if out is None:
        out = torch.empty((m, n), dtype=x2.dtype, device=x2.device)
    else:
        _check_out(out, (m, n), x2.dtype, x2.device)
    if m == 0 or n == 0:
        return out
    fn = getattr(_lib.load(), entry)
    with torch.cuda.device(x2.device):
        sp = stream_ptr(x2.device)
        for r0 in range(0, m, MAX_ROWS_PER_CALL):
            r1 = min(m, r0 + MAX_ROWS_PER_CALL)
            need = workspace_bytes(r1 - r0, k, n)
            ws = workspace(x2.device, need)
            xs = x2[r0:r1]
            ys = out[r0:r1]
            st = fn(xs.data_ptr(), w_q.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                    ys.data_ptr(), ws.data_ptr(), ws.numel(), r1 - r0, k, n, sp)
            _lib.check(entry, st)
    return out


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, dim: int = 0) -> torch.Tensor:
    """Row-interleave two tensors along ``dim`` (size I) in blocks of 16 rows:
    ``[gate 0..15, up 0..15, gate 16..31, up 16..31, ...]`` -> size 2I.

    The layout :func:`gate_up_silu` (and the grouped MoE variant, with
    ``dim=1`` over an expert stack) takes for the packed weights, scales and
    biases of an MLP's gate/up pair (a load-time layout, like concatenating
    projections that share an input)."""
    dim = dim % gate.dim()
    if gate.shape != up.shape or gate.shape[dim] % 16 != 0:
        raise ValueError("gate and up must have the same shape with rows % 16 == 0")
    i = gate.shape[dim]
    lead, tail = gate.shape[:dim], gate.shape[dim + 1:]
    return torch.stack((gate.reshape(*lead, i // 16, 16, *tail), up.reshape(*lead, i // 16, 16, *tail)),
                       dim=dim + 1).reshape(*lead, 2 * i, *tail)


_SILU_ENTRY = {("pairs", torch.bfloat16): "dfl_verify_qmm_w4g64_pairs_silu",
               ("pairs", torch.float16): "dfl_verify_qmm_w4g64_pairs_silu_f16",
               ("mlx", torch.bfloat16): "dfl_verify_qmm_w4g64_silu"}


def gate_up_silu(x2: torch.Tensor, w_q: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                 out: torch.Tensor | None = None, *, layout: str = "pairs") -> torch.Tensor:
    """``silu(x2 @ Wg.T) * (x2 @ Wu.T)`` in one launch -> ``[M, I]``.

    ``w_q`` / ``scales`` / ``biases`` are the gate and up projections
    interleaved by :func:`interleave_gate_up`; ``layout`` is ``"pairs"``
    (weights passed through :func:`repack_pairs`) or ``"mlx"`` (bf16 only).
    Each projection is rounded to the activation dtype before the SiLU, so the
    result equals :func:`silu_mul` of the two projections computed separately
    by the same kernel."""
    for t, name in ((x2, "x"), (w_q, "w"), (scales, "scales"), (biases, "biases")):
        require_cuda(t, name)
    entry = _SILU_ENTRY.get((layout, x2.dtype))
    if entry is None:
        raise NotImplementedError(f"no fused SiLU kernel for layout {layout!r} and {x2.dtype}")
    if scales.dtype != x2.dtype or biases.dtype != x2.dtype:
        raise NotImplementedError("scales/biases must match the activations' dtype")
    w_q = as_u32_bits(w_q)
    x2, scales, biases = x2.contiguous(), scales.contiguous(), biases.contiguous()
    m, k = x2.shape
    n = w_q.shape[0]
    if w_q.shape[1] * 8 != k or n % 32 != 0:
        raise ValueError(f"weight shape {tuple(w_q.shape)} does not fit K={k} (rows % 32 == 0)")
    if scales.shape != (n, k // 64) or biases.shape != (n, k // 64):
        raise ValueError("scales/biases must be [N, K/64]")
    if out is None:
        out = torch.empty((m, n // 2), dtype=x2.dtype, device=x2.device)
    else:
        _check_out(out, (m, n // 2), x2.dtype, x2.device)
    if m == 0:
        return out
    fn = getattr(_lib.load(), entry)
    with torch.cuda.device(x2.device):
        sp = stream_ptr(x2.device)
        for r0 in range(0, m, MAX_ROWS_PER_CALL):
            r1 = min(m, r0 + MAX_ROWS_PER_CALL)
            ws = workspace(x2.device, workspace_bytes(r1 - r0, k, n))
            st = fn(x2[r0:r1].data_ptr(), w_q.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                    out[r0:r1].data_ptr(), ws.data_ptr(), ws.numel(), r1 - r0, k, n, sp)
            _lib.check(entry, st)
    return out


def verify_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                  *, transpose: bool = True, group_size: int = 64, bits: int = 4) -> torch.Tensor:
    """``x @ dequant(w).T`` for MLX affine int4 g64 weights (reference ``verify_qmm.py:905``)."""
    if bits != 4 or group_size != 64:
        raise NotImplementedError(
            f"only bits=4, group_size=64 is implemented (got bits={bits}, group_size={group_size})")
    if not transpose:
        raise NotImplementedError("only transpose=True (y = x @ W.T) is implemented")
    if biases is None:
        raise ValueError("affine quantization needs biases")
    orig = x.shape
    k = orig[-1]
    m = 1
    for d in orig[:-1]:
        m *= int(d)
    y = qmm_w4g64(x.reshape(m, k), w, scales, biases)
    return y.reshape(*orig[:-1], w.shape[0])
