"""GatedDeltaNet tape replay on B200.

Mirrors ``dflash_mlx/kernels.py``:

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
