"""Oracle for the lm_head verify epilogue -- TEST INFRASTRUCTURE ONLY.

Restates, for a batch of B verify blocks of T=16 positions:

* logits = h @ E.T in the activation dtype (``engine/target_qwen_gdn.py:774-778``:
  ``embed_tokens.as_linear`` / ``lm_head``; bf16 in, fp32 accumulate, bf16 out);
* ``greedy_tokens_with_mask`` (``engine/sampling.py:47-55``): suppressed ids get
  the floor ``-1e9`` cast to the logits dtype, then ``argmax`` (first index of
  the maximum);
* ``match_acceptance_length`` (``engine/acceptance.py:9-16``): the sum of the
  cumulative product of ``drafted == posterior``;
* the composition at ``engine/spec_epoch.py:2067-2072,2129``: the drafts are
  ``verify_ids[1:]``, they are compared with ``posterior[:-1]`` and the next
  staged token is ``posterior[acceptance]``.
"""

from __future__ import annotations

import numpy as np

from . import bf16

SUPPRESS_FLOOR_BF16 = int(bf16.from_f32(np.array([-1e9], dtype=np.float32))[0])


def match_acceptance_length(drafted, posterior) -> int:
    """``engine/acceptance.py:9-16`` restated."""
    d = np.asarray(drafted).astype(np.int64).reshape(-1)
    p = np.asarray(posterior).astype(np.int64).reshape(-1)
    if d.shape[0] == 0:
        return 0
    matches = (d == p).astype(np.int32)
    return int(np.cumprod(matches).sum())


def logits_bf16(h: np.ndarray, w: np.ndarray) -> np.ndarray:
    """bf16 logits ``[R, V]`` (float32 values that are exactly bf16).

    ``h`` is bf16 bits ``[R, D]``, ``w`` bf16 bits ``[V, D]``.  Accumulation in
    float32 via BLAS (blocked, so the sum order differs from any GPU kernel by
    fp32 rounding only).
    """
    hf = bf16.to_f32(h)
    wf = bf16.to_f32(w)
    return bf16.round_f32(hf @ wf.T)


def greedy_tokens(logits: np.ndarray, suppress_mask=None) -> np.ndarray:
    """``engine/sampling.py:47-55``: argmax over the last axis, first index wins."""
    lg = np.array(logits, dtype=np.float32, copy=True)
    if suppress_mask is not None:
        floor = bf16.to_f32(np.array([SUPPRESS_FLOOR_BF16], dtype=np.uint16))[0]
        lg[..., np.asarray(suppress_mask, dtype=bool)] = floor
    return np.argmax(lg, axis=-1).astype(np.int64)


def verify_accept(logits: np.ndarray, verify_ids: np.ndarray, suppress_mask=None):
    """Posterior tokens, acceptance length and next staged token per block.

    ``logits`` is ``[B, T, V]``, ``verify_ids`` int ``[B, T]`` (``verify_ids[:, 0]``
    is the staged token, ``verify_ids[:, 1:]`` the drafts).
    Returns (posterior int32 [B, T], acceptance int32 [B], next_token int32 [B]).
    """
    post = greedy_tokens(logits, suppress_mask)
    b = post.shape[0]
    acc = np.zeros(b, dtype=np.int32)
    nxt = np.zeros(b, dtype=np.int32)
    for i in range(b):
        acc[i] = match_acceptance_length(verify_ids[i, 1:], post[i, :-1])
        nxt[i] = post[i, acc[i]]
    return post.astype(np.int32), acc, nxt


def shard_partials(logits: np.ndarray, v_begin: int, suppress_mask=None):
    """Per-row (max value, global argmax) over one vocab shard.

    ``logits`` is the shard's ``[R, V_shard]`` slice; the index returned is
    global (``v_begin + local``).  Ties resolve to the lowest index.
    """
    lg = np.array(logits, dtype=np.float32, copy=True)
    if suppress_mask is not None:
        floor = bf16.to_f32(np.array([SUPPRESS_FLOOR_BF16], dtype=np.uint16))[0]
        lg[:, np.asarray(suppress_mask, dtype=bool)] = floor
    idx = np.argmax(lg, axis=-1)
    return lg[np.arange(lg.shape[0]), idx], (idx + v_begin).astype(np.int64)


def reduce_partials(vals: np.ndarray, idxs: np.ndarray) -> np.ndarray:
    """Combine per-shard (max, idx) ``[G, R]`` into the global argmax ``[R]``.

    Larger value wins; on equal values the lower global index wins, which is
    what a single ``argmax`` over the whole vocabulary returns.
    """
    vals = np.asarray(vals, dtype=np.float32)
    idxs = np.asarray(idxs, dtype=np.int64)
    best_v = vals[0].copy()
    best_i = idxs[0].copy()
    for g in range(1, vals.shape[0]):
        better = (vals[g] > best_v) | ((vals[g] == best_v) & (idxs[g] < best_i))
        best_v = np.where(better, vals[g], best_v)
        best_i = np.where(better, idxs[g], best_i)
    return best_i


def top2_margin(logits: np.ndarray, suppress_mask=None) -> np.ndarray:
    """Gap between the largest and second-largest logit of each row."""
    lg = np.array(logits, dtype=np.float32, copy=True)
    if suppress_mask is not None:
        floor = bf16.to_f32(np.array([SUPPRESS_FLOOR_BF16], dtype=np.uint16))[0]
        lg[..., np.asarray(suppress_mask, dtype=bool)] = floor
    part = np.partition(lg, -2, axis=-1)
    return part[..., -1] - part[..., -2]


def synth_verify_ids(rng: np.random.Generator, posterior: np.ndarray, vocab: int,
                     p_match: float = 0.88) -> np.ndarray:
    """Verify ids with P(d_j == posterior_{j-1}) = p_match (0.88 by default).

    ``verify_ids[:, 0]`` (the staged token) is uniform; each later position
    copies the target argmax of the previous position with probability
    ``p_match`` and is otherwise a uniform random token.
    """
    b, t = posterior.shape
    ids = rng.integers(0, vocab, size=(b, t)).astype(np.int32)
    hit = rng.random((b, t)) < p_match
    for j in range(1, t):
        ids[:, j] = np.where(hit[:, j], posterior[:, j - 1], ids[:, j])
    return ids
