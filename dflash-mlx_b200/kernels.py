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
    # the kernel reads steps[b] for every sequence and mask[b, t] for every step
    if steps is not None and steps.numel() != b:
        raise ValueError(f"steps must hold one count per sequence ({b}), got {steps.numel()}")
    if mask is not None and mask.numel() != b * t_steps:
        raise ValueError(f"mask must be [B, T] = {(b, t_steps)}, got {tuple(mask.shape)}")
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


# ------------------------------------------------------------------ DDTree
def _tree_inputs(q, k, v, g, beta, state, parent_ids):
    for t, name in ((q, "q"), (k, "k"), (v, "v"), (g, "g"), (beta, "beta"), (state, "state")):
        require_cuda(t, name)
    if q.dtype not in (torch.bfloat16, torch.float32) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise NotImplementedError("q, k, v must all be bfloat16 or all float32")
    if state.dtype != torch.float32:
        raise NotImplementedError(f"state must be float32, got {state.dtype}")
    b, t_steps, hk, dk = k.shape
    hv, dv = v.shape[2:]
    if q.shape != k.shape:
        raise ValueError("q and k must have the same shape")
    if hv % hk != 0:
        raise ValueError(f"Cannot align K heads {hk} to V heads {hv}")
    if g.shape not in ((b, t_steps, hv), (b, t_steps, hv, dk)):
        raise ValueError(f"Unsupported gating shape {tuple(g.shape)}")
    if beta.shape != (b, t_steps, hv) or state.shape != (b, hv, dv, dk):
        raise ValueError("beta must be [B, T, Hv] and state [B, Hv, Dv, Dk]")
    parent_ids = torch.as_tensor(parent_ids).to(device=state.device, dtype=torch.int32).reshape(-1)
    if parent_ids.numel() != t_steps:
        raise ValueError("parent_ids must have one entry per tree node")
    # g and beta enter the kernel as fp32 (bf16 values widen exactly)
    g = g.to(torch.float32)
    beta = beta.to(torch.float32)
    q, k, v, g, beta, state, parent_ids = (x.contiguous() for x in (q, k, v, g, beta, state, parent_ids))
    return q, k, v, g, beta, state, parent_ids, (b, t_steps, hv, hk, dv, dk)


def _tree_launch(q, k, v, g, beta, state, parent_ids, dims, want_tape):
    b, t_steps, hv, hk, dv, dk = dims
    y = torch.empty((b, t_steps, hv, dv), dtype=q.dtype, device=state.device)
    nodes = torch.empty((b, t_steps, hv, dv, dk), dtype=torch.float32, device=state.device)
    tape = torch.empty((b, t_steps, hv, dv), dtype=torch.float32, device=state.device) if want_tape else None
    with torch.cuda.device(state.device):
        st = _lib.load().dfl_gdn_tree_forward(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), 1 if g.dim() == 4 else 0,
            beta.data_ptr(), state.data_ptr(), parent_ids.data_ptr(), y.data_ptr(), nodes.data_ptr(),
            tape.data_ptr() if tape is not None else None, b, t_steps, hv, hk, dv, dk,
            1 if q.dtype == torch.float32 else 0, stream_ptr(state.device))
    _lib.check("dfl_gdn_tree_forward", st)
    return y, nodes, tape


def gated_delta_tree_kernel(q, k, v, g, beta, state, parent_ids):
    """GDN over a token tree (reference ``kernels.py:501``): ``(y, tree_states)``,
    node t starting from node ``parent_ids[t]`` (or ``state`` when < 0)."""
    q, k, v, g, beta, state, parent_ids, dims = _tree_inputs(q, k, v, g, beta, state, parent_ids)
    y, nodes, _ = _tree_launch(q, k, v, g, beta, state, parent_ids, dims, want_tape=False)
    return y, nodes


def gated_delta_tree_tape_kernel(q, k, v, g, beta, state, parent_ids):
    """The tree recurrence recording the innovation tape (reference
    ``kernels.py:545``): ``(y, tape)``; replaying a root-to-node path's tape rows
    with ``tape_replay_kernel`` reproduces that node's state."""
    q, k, v, g, beta, state, parent_ids, dims = _tree_inputs(q, k, v, g, beta, state, parent_ids)
    y, _, tape = _tree_launch(q, k, v, g, beta, state, parent_ids, dims, want_tape=True)
    return y, tape


def tree_depthwise_conv1d(qkv, prefix, weight, bias, path_indices):
    """Depthwise conv1d along tree paths + SiLU (reference ``kernels.py:647``).

    ``qkv [B, T, C]``, ``prefix [B, K-1, C]`` (same dtype, bf16 or fp32),
    ``weight [C, K, 1]`` (or ``[C, K]``), ``bias [C]`` or None,
    ``path_indices [T, K]`` into ``concat(prefix, qkv)``."""
    for t, name in ((qkv, "qkv"), (prefix, "prefix"), (weight, "weight")):
        require_cuda(t, name)
    if qkv.dtype not in (torch.bfloat16, torch.float32):
        raise NotImplementedError(f"qkv must be bfloat16 or float32, got {qkv.dtype}")
    b, t_steps, c = qkv.shape
    w = weight[..., 0] if weight.dim() == 3 else weight
    if w.shape[0] != c:
        raise ValueError(f"weight must be [C, K(, 1)] with C = {c}")
    kk = int(w.shape[1])
    if prefix.shape != (b, kk - 1, c) or prefix.dtype != qkv.dtype:
        raise ValueError(f"prefix must be [B, K-1, C] = {(b, kk - 1, c)} in qkv's dtype")
    if bias is not None and bias.numel() != c:
        raise ValueError(f"bias must hold one value per channel ({c}), got {bias.numel()}")
    path = torch.as_tensor(path_indices).to(device=qkv.device, dtype=torch.int32).reshape(t_steps, kk)
    w = w.to(torch.float32).contiguous()
    bias = bias.to(device=qkv.device, dtype=torch.float32).contiguous() if bias is not None else None
    qkv, prefix, path = qkv.contiguous(), prefix.contiguous(), path.contiguous()
    out = torch.empty_like(qkv)
    with torch.cuda.device(qkv.device):
        st = _lib.load().dfl_tree_depthwise_conv1d(
            qkv.data_ptr(), prefix.data_ptr(), w.data_ptr(), bias.data_ptr() if bias is not None else None,
            path.data_ptr(), out.data_ptr(), b, t_steps, c, kk, 1 if qkv.dtype == torch.float32 else 0,
            stream_ptr(qkv.device))
    _lib.check("dfl_tree_depthwise_conv1d", st)
    return out
