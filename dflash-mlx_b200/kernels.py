"""GatedDeltaNet tape recording and tape replay on B200.

Mirrors ``dflash_mlx/kernels.py``:

* ``gated_delta_kernel_with_tape(q, k, v, g, beta, state, mask=None)`` --
  ``kernels.py:169-219``: the verify forward over T steps returning
  ``(y, state, tape)`` (y bf16 ``[B, T, Hv, Dv]``, new fp32 state, fp32
  innovation tape); q, k, v bf16, g and beta fp32.  Its state updates are the
  replay's operations in the same order, so replaying its tape over a prefix
  of a steps gives exactly its state after a steps.
* ``tape_replay_kernel(tape, k, g, state, mask=None)`` -- ``kernels.py:822-868``.
  Functional like the reference: returns a new state and leaves ``state``
  untouched.  Same shapes: tape fp32 ``[B, T, Hv, Dv]``, k ``[B, T, Hk, Dk]``
  (bf16 or fp32), g ``[B, T, Hv]`` or ``[B, T, Hv, Dk]``, state fp32
  ``[B, Hv, Dv, Dk]``, optional bool mask ``[B, T]``.
* ``tape_replay_(state, tape, k, g, steps)`` -- the in-place form the
  rollback uses on B200: replays the first ``steps[b]`` steps of each
  sequence and does not touch sequences with nothing to replay.

The update per replayed step is ``S <- S * g_t`` then ``S <- S + delta_t k_t``,
two separately rounded fp32 operations in the order of the mx-op reference
(``kernels.py:790-820``).  Only fp32 states are supported (the reference
re-rounds the state to its own dtype after every step, ``kernels.py:745-747``,
which is the identity for fp32).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from ._runtime import require_cuda, stream_ptr


def _check(tape, k, g, state, steps=None, mask=None):
    for t, name in ((tape, "tape"), (k, "k"), (g, "g"), (state, "state")):
        require_cuda(t, name)
    if state.dtype != torch.float32:
        raise NotImplementedError(f"state must be float32, got {state.dtype}")
    if tape.dtype != torch.float32:
        raise NotImplementedError(f"tape must be float32, got {tape.dtype}")
    if k.dtype not in (torch.bfloat16, torch.float32):
        raise NotImplementedError(f"k must be bfloat16 or float32, got {k.dtype}")
    if g.dtype != torch.float32:
        raise NotImplementedError(f"g must be float32, got {g.dtype}")
    b, t_steps, hk, dk = k.shape
    hv, dv = tape.shape[2:]
    if hv % hk != 0:
        raise ValueError(f"Cannot align K heads {hk} to tape heads {hv}")
    if tape.shape[:2] != (b, t_steps):
        raise ValueError("tape and k disagree on [B, T]")
    if state.shape != (b, hv, dv, dk):
        raise ValueError(f"state must be [B, Hv, Dv, Dk] = {(b, hv, dv, dk)}, got {tuple(state.shape)}")
    if g.dim() == 3:
        if g.shape != (b, t_steps, hv):
            raise ValueError("scalar g must be [B, T, Hv]")
    elif g.dim() == 4:
        if g.shape != (b, t_steps, hv, dk):
            raise ValueError("vector g must be [B, T, Hv, Dk]")
    else:
        raise ValueError(f"Unsupported gating shape {tuple(g.shape)}")
    return b, t_steps, hv, hk, dv, dk


def _launch(tape, k, g, state_in, state_out, steps, mask, dims):
    b, t_steps, hv, hk, dv, dk = dims
    tape = tape.contiguous()
    k = k.contiguous()
    g = g.contiguous()
    steps_ptr = 0
    mask_ptr = 0
    if steps is not None:
        steps = steps.to(device=state_in.device, dtype=torch.int32).contiguous()
        steps_ptr = steps.data_ptr()
    if mask is not None:
        mask = mask.to(device=state_in.device, dtype=torch.uint8).contiguous()
        mask_ptr = mask.data_ptr()
    with torch.cuda.device(state_in.device):
        st = _lib.load().dfl_gdn_tape_replay(
            tape.data_ptr(), k.data_ptr(), 1 if k.dtype == torch.bfloat16 else 0, g.data_ptr(),
            1 if g.dim() == 4 else 0, steps_ptr or None, mask_ptr or None, state_in.data_ptr(),
            state_out.data_ptr(), b, t_steps, hv, hk, dv, dk, stream_ptr(state_in.device))
    _lib.check("dfl_gdn_tape_replay", st)
    return state_out


def tape_replay_kernel(tape: torch.Tensor, k: torch.Tensor, g: torch.Tensor, state: torch.Tensor,
                       mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Replay the recorded innovation tape onto ``state`` (reference ``kernels.py:822``)."""
    dims = _check(tape, k, g, state, mask=mask)
    state = state.contiguous()
    out = torch.empty_like(state)
    return _launch(tape, k, g, state, out, None, mask, dims)


def tape_replay_(state: torch.Tensor, tape: torch.Tensor, k: torch.Tensor, g: torch.Tensor,
                 steps: Optional[torch.Tensor] = None) -> torch.Tensor:
    """In-place replay of the first ``steps[b]`` steps of each sequence."""
    if not state.is_contiguous():
        raise ValueError("in-place replay needs a contiguous state")
    dims = _check(tape, k, g, state, steps=steps)
    return _launch(tape, k, g, state, state, steps, None, dims)


def gated_delta_kernel_with_tape(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                                 beta: torch.Tensor, state: torch.Tensor,
                                 mask: Optional[torch.Tensor] = None):
    """GDN verify forward recording the innovation tape (reference ``kernels.py:169``).

    Returns ``(y, new_state, tape)``; ``state`` is left untouched.
    """
    for t, name in ((q, "q"), (k, "k"), (v, "v"), (g, "g"), (beta, "beta"), (state, "state")):
        require_cuda(t, name)
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        if t.dtype != torch.bfloat16:
            raise NotImplementedError(f"{name} must be bfloat16, got {t.dtype}")
    if g.dtype != torch.float32 or beta.dtype != torch.float32:
        raise NotImplementedError("g and beta must be float32")
    if state.dtype != torch.float32:
        raise NotImplementedError(f"state must be float32, got {state.dtype}")
    b, t_steps, hk, dk = k.shape
    hv, dv = v.shape[2:]
    if q.shape != k.shape:
        raise ValueError("q and k must have the same shape")
    if hv % hk != 0:
        raise ValueError(f"Cannot align K heads {hk} to V heads {hv}")
    if v.shape[:2] != (b, t_steps) or beta.shape != (b, t_steps, hv):
        raise ValueError("v must be [B, T, Hv, Dv] and beta [B, T, Hv]")
    if g.shape not in ((b, t_steps, hv), (b, t_steps, hv, dk)):
        raise ValueError(f"Unsupported gating shape {tuple(g.shape)}")
    if state.shape != (b, hv, dv, dk):
        raise ValueError(f"state must be [B, Hv, Dv, Dk] = {(b, hv, dv, dk)}, got {tuple(state.shape)}")
    q, k, v, g, beta, state = (t.contiguous() for t in (q, k, v, g, beta, state))
    y = torch.empty((b, t_steps, hv, dv), dtype=torch.bfloat16, device=state.device)
    tape = torch.empty((b, t_steps, hv, dv), dtype=torch.float32, device=state.device)
    out = torch.empty_like(state)
    mask_ptr = None
    if mask is not None:
        mask = mask.to(device=state.device, dtype=torch.uint8).reshape(b, t_steps).contiguous()
        mask_ptr = mask.data_ptr()
    with torch.cuda.device(state.device):
        st = _lib.load().dfl_gdn_forward_tape(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), 1 if g.dim() == 4 else 0,
            beta.data_ptr(), mask_ptr, state.data_ptr(), out.data_ptr(), y.data_ptr(),
            tape.data_ptr(), b, t_steps, hv, hk, dv, dk, stream_ptr(state.device))
    _lib.check("dfl_gdn_forward_tape", st)
    return y, out, tape
