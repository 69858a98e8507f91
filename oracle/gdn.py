"""Oracle for GatedDeltaNet tape recording and tape-replay rollback.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Shapes follow the reference kernels (``dflash_mlx/kernels.py``):
q, k ``[B, T, Hk, Dk]``; v ``[B, T, Hv, Dv]``; g ``[B, T, Hv]`` (scalar decay)
or ``[B, T, Hv, Dk]`` (vector decay); beta ``[B, T, Hv]``;
state ``[B, Hv, Dv, Dk]`` (fp32); tape ``[B, T, Hv, Dv]`` (fp32).
K heads are shared by ``Hv // Hk`` consecutive value heads
(``kernels.py:31-33,712``: ``hk = hv / (Hv / Hk)``).
All inputs here are float32 arrays (bf16 inputs are passed already widened).
"""

from __future__ import annotations

import numpy as np


def _expand_heads(a: np.ndarray, hv: int) -> np.ndarray:
    hk = a.shape[2]
    if hv % hk != 0:
        raise ValueError(f"Cannot align K heads {hk} to V heads {hv}")
    r = hv // hk
    return np.repeat(a, r, axis=2) if r > 1 else a


def _decay(g: np.ndarray, t: int) -> np.ndarray:
    if g.ndim == 4:
        return g[:, t, :, None, :]
    if g.ndim == 3:
        return g[:, t, :, None, None]
    raise ValueError(f"Unsupported gating shape {g.shape}")


def gated_delta_with_tape(q, k, v, g, beta, state, mask=None):
    """``_gated_delta_ops_with_tape`` restated (``kernels.py:125-167``).

    Returns (y float32 [B,T,Hv,Dv], final state float32, tape float32).
    The innovation recorded per step is ``delta = (v - (g*S)·k) * beta``.
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    g = np.asarray(g, np.float32)
    beta = np.asarray(beta, np.float32)
    state = np.array(state, np.float32, copy=True)
    hv = v.shape[2]
    q = _expand_heads(q, hv)
    k = _expand_heads(k, hv)
    t_steps = k.shape[1]
    ys, tape = [], []
    for t in range(t_steps):
        old = state
        decayed = state * _decay(g, t)
        kv_mem = (decayed * k[:, t, :, None, :]).sum(axis=-1, dtype=np.float32)
        delta = (v[:, t] - kv_mem) * beta[:, t, :, None]
        new = decayed + k[:, t, :, None, :] * delta[..., None]
        y = (new * q[:, t, :, None, :]).sum(axis=-1, dtype=np.float32)
        if mask is not None:
            m = np.asarray(mask, bool)[:, t]
            new = np.where(m[:, None, None, None], new, old)
            delta = np.where(m[:, None, None], delta, 0.0).astype(np.float32)
            y = np.where(m[:, None, None], y, 0.0).astype(np.float32)
        state = new.astype(np.float32)
        ys.append(y.astype(np.float32))
        tape.append(delta.astype(np.float32))
    if t_steps == 0:
        b, _, hv_, dv = v.shape
        empty = np.zeros((b, 0, hv_, dv), dtype=np.float32)
        return empty, state, empty.copy()
    return np.stack(ys, 1), state, np.stack(tape, 1)


def gated_delta_tree(q, k, v, g, beta, state, parent_ids):
    """``_gated_delta_tree_ops`` restated (``kernels.py:421-458``).

    Returns (y [B,T,Hv,Dv], per-node states [B,T,Hv,Dv,Dk]).
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    g = np.asarray(g, np.float32)
    beta = np.asarray(beta, np.float32)
    state = np.asarray(state, np.float32)
    hv = v.shape[2]
    q = _expand_heads(q, hv)
    k = _expand_heads(k, hv)
    ys, states = [], []
    for t, parent in enumerate(int(p) for p in np.asarray(parent_ids).reshape(-1)):
        s_in = state if parent < 0 else states[parent]
        decayed = s_in * _decay(g, t)
        kv_mem = (decayed * k[:, t, :, None, :]).sum(axis=-1, dtype=np.float32)
        delta = (v[:, t] - kv_mem) * beta[:, t, :, None]
        s_t = (decayed + k[:, t, :, None, :] * delta[..., None]).astype(np.float32)
        ys.append((s_t * q[:, t, :, None, :]).sum(axis=-1, dtype=np.float32))
        states.append(s_t)
    return np.stack(ys, 1), np.stack(states, 1)


def gated_delta_tree_tape(q, k, v, g, beta, state, parent_ids):
    """``_gated_delta_tree_tape_ops`` restated (``kernels.py:460-498``): (y, tape)."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    g = np.asarray(g, np.float32)
    beta = np.asarray(beta, np.float32)
    state = np.asarray(state, np.float32)
    hv = v.shape[2]
    q = _expand_heads(q, hv)
    k = _expand_heads(k, hv)
    ys, tape, states = [], [], []
    for t, parent in enumerate(int(p) for p in np.asarray(parent_ids).reshape(-1)):
        s_in = state if parent < 0 else states[parent]
        decayed = s_in * _decay(g, t)
        kv_mem = (decayed * k[:, t, :, None, :]).sum(axis=-1, dtype=np.float32)
        delta = ((v[:, t] - kv_mem) * beta[:, t, :, None]).astype(np.float32)
        s_t = (decayed + k[:, t, :, None, :] * delta[..., None]).astype(np.float32)
        ys.append((s_t * q[:, t, :, None, :]).sum(axis=-1, dtype=np.float32))
        tape.append(delta)
        states.append(s_t)
    return np.stack(ys, 1), np.stack(tape, 1)


def tape_replay(tape, k, g, state, mask=None):
    """``_tape_replay_ops`` restated (``kernels.py:790-820``).

    For each step t with ``mask[:, t]`` true (all steps when mask is None):
    ``S <- S * g_t``, then ``S <- S + delta_t (x) k_t`` -- two separately
    rounded fp32 operations per element, in that order.
    """
    tape = np.asarray(tape, np.float32)
    k = np.asarray(k, np.float32)
    g = np.asarray(g, np.float32)
    state = np.array(state, np.float32, copy=True)
    hv = tape.shape[2]
    k = _expand_heads(k, hv)
    for t in range(tape.shape[1]):
        prev = state
        s = state * _decay(g, t)
        s = s + tape[:, t, :, :, None] * k[:, t, :, None, :]
        if mask is not None:
            m = np.asarray(mask, bool)[:, t]
            s = np.where(m[:, None, None, None], s, prev)
        state = s.astype(np.float32)
    return state


def tape_replay_accepted(tape, k, g, state, accepted_steps):
    """Replay the first ``accepted_steps[b]`` steps of each sequence b.

    Equivalent to :func:`tape_replay` with ``mask[b, t] = t < accepted_steps[b]``
    (the masked reference variant, ``kernels.py:695,737``); with one shared
    count it is the slice ``tape[:, :a]`` that
    ``recurrent_rollback_cache.py:154-161`` replays.
    """
    a = np.asarray(accepted_steps).reshape(-1)
    t_steps = np.asarray(tape).shape[1]
    mask = np.arange(t_steps)[None, :] < a[:, None]
    return tape_replay(tape, k, g, state, mask)


def tree_depthwise_conv1d(qkv, prefix, weight, bias, path_indices):
    """``_tree_depthwise_conv1d_ops`` restated (``kernels.py:631-644``).

    ``qkv [B, T, C]``, ``prefix [B, K-1, C]``, ``weight [C, K, 1]`` or
    ``[C, K]``, ``bias [C]`` or None, ``path_indices [T, K]`` into
    ``concat(prefix, qkv, axis=1)``; fp32 accumulation in window order, then
    silu(x) = x / (1 + exp(-x)).
    """
    qkv = np.asarray(qkv, np.float32)
    prefix = np.asarray(prefix, np.float32)
    w = np.asarray(weight, np.float32)
    if w.ndim == 3:
        w = w[..., 0]
    pool = np.concatenate([prefix, qkv], axis=1)
    path = np.asarray(path_indices, np.int64)
    b, t_steps, c = qkv.shape
    acc = np.zeros((b, t_steps, c), np.float32)
    for j in range(w.shape[1]):
        acc = (acc + pool[:, path[:, j], :] * w[None, None, :, j]).astype(np.float32)
    if bias is not None:
        acc = (acc + np.asarray(bias, np.float32)[None, None, :]).astype(np.float32)
    return (acc / (np.float32(1.0) + np.exp(-acc))).astype(np.float32)
