"""Rollback cache for GatedDeltaNet layers during speculative verify.

Mirrors ``dflash_mlx/recurrent_rollback_cache.py`` (``RecurrentRollbackCache``)
and the restore policy of ``dflash_mlx/engine/target_qwen_gdn.py:1025-1055``:

* ``arm_rollback`` snapshots ``[conv_state, ssm_state]`` (``:96-103``);
* ``record_tape`` keeps the verify forward's innovation tape, k, g and qkv
  (``:110-121``);
* ``rollback(n_accepted)`` restores the snapshot and replays
  ``n_accepted + 1`` steps of the tape (``:142-165``), rebuilding the conv
  state from the last ``conv_kernel_size - 1`` inputs (``:123-140``);
* ``restore_after_acceptance`` skips the replay entirely when every drafted
  token was accepted (``target_qwen_gdn.py:1034-1039``).

Per-sequence acceptance (``rollback`` with a tensor of counts) replays all
sequences of a batch in one launch; the snapshot is restored in place
instead of re-binding a new array, and sequences with nothing to replay are
not touched by the kernel.
"""

from __future__ import annotations

import time

from typing import Any, Optional, Sequence, Union

import torch

from .kernels import tape_replay_


class RecurrentRollbackCache:
    def __init__(self, size: int = 2, *, conv_kernel_size: int = 4):
        self.cache: list[Optional[torch.Tensor]] = [None] * size
        self.conv_kernel_size = int(conv_kernel_size)
        self.clear_transients()

    def __getitem__(self, idx: int):
        return self.cache[idx]

    def __setitem__(self, idx: int, value: Any) -> None:
        self.cache[idx] = value

    @property
    def state(self):
        return self.cache

    def clear_transients(self) -> None:
        self._armed = False
        self._tape = None
        self._tape_k = None
        self._tape_g = None
        self._tape_qkv = None
        self._snapshot = None

    def checkpoint(self) -> None:
        self._snapshot = [None if c is None else c.clone() for c in self.cache]

    def arm_rollback(self, prefix_len: int = 0) -> None:
        del prefix_len
        self.clear_transients()
        self._armed = True
        self.checkpoint()

    def record_tape(self, *, tape: torch.Tensor, k: torch.Tensor, g: torch.Tensor,
                    qkv: Optional[torch.Tensor] = None) -> None:
        self._tape = tape.contiguous()
        self._tape_k = k.contiguous()
        self._tape_g = g.contiguous()
        self._tape_qkv = None if qkv is None else qkv.contiguous()

    def _rebuild_conv_state(self, accepted_steps: torch.Tensor) -> Optional[torch.Tensor]:
        """Last ``conv_kernel_size - 1`` conv inputs after ``accepted_steps[b]``
        accepted steps of each sequence (``recurrent_rollback_cache.py:123-140``)."""
        if self._tape_qkv is None:
            return self.cache[0]
        keep = self.conv_kernel_size - 1
        if keep <= 0:
            return None
        prefix = self._snapshot[0] if self._snapshot is not None else None
        if prefix is None:
            prefix = torch.zeros((self._tape_qkv.shape[0], keep, self._tape_qkv.shape[-1]),
                                 dtype=self._tape_qkv.dtype, device=self._tape_qkv.device)
        conv_input = torch.cat([prefix, self._tape_qkv], dim=1)
        length = int(conv_input.shape[1])
        a = accepted_steps.to(device=conv_input.device, dtype=torch.long).reshape(-1, 1)
        idx = (a + torch.arange(keep, device=conv_input.device)).clamp(max=length - 1)
        idx = idx[:, :, None].expand(-1, -1, conv_input.shape[-1])
        return torch.gather(conv_input, 1, idx).contiguous()

    def rollback(self, n_accepted: Union[int, Sequence[int], torch.Tensor]) -> None:
        if self._snapshot is None:
            self.clear_transients()
            return
        state_now = self.cache[1]
        snap_state = self._snapshot[1]
        self.cache = list(self._snapshot)
        if (self._tape is not None and self._tape_k is not None and self._tape_g is not None
                and snap_state is not None):
            if isinstance(n_accepted, int):
                steps = torch.full((snap_state.shape[0],), int(n_accepted) + 1, dtype=torch.int32)
            else:
                steps = torch.as_tensor(n_accepted, dtype=torch.int32).reshape(-1) + 1
                if steps.numel() == 1:   # one count for every sequence of the batch
                    steps = steps.expand(snap_state.shape[0])
            # reuse the live state buffer: restore the snapshot into it, replay in place
            target = state_now if state_now is not None and state_now.shape == snap_state.shape \
                else torch.empty_like(snap_state)
            target.copy_(snap_state)
            tape_replay_(target, self._tape, self._tape_k, self._tape_g, steps)
            self.cache[1] = target
            self.cache[0] = self._rebuild_conv_state(steps)
        self.clear_transients()


def arm_rollback(cache_entries, *, prefix_len: int) -> None:
    """``target_qwen_gdn.py:1003-1006``: arm every entry that supports rollback."""
    for entry in cache_entries:
        if hasattr(entry, "arm_rollback"):
            entry.arm_rollback(prefix_len=int(prefix_len))


def clear_rollback_state(entry) -> None:
    """``target_qwen_gdn.py:1008-1023``: drop an entry's tape and snapshot."""
    if hasattr(entry, "clear_transients"):
        entry.clear_transients()
        return
    for name in ("_tape", "_tape_k", "_tape_g", "_tape_qkv", "_snapshot"):
        if hasattr(entry, name):
            setattr(entry, name, None)
    if hasattr(entry, "_armed"):
        entry._armed = False


def restore_after_acceptance(cache_entries, *, target_len: int, acceptance_length: int,
                             drafted_tokens: int = 0) -> int:
    """``target_qwen_gdn.py:1025-1055``: full acceptance clears the recurrent
    entries' transients without replaying; otherwise they roll back to
    ``acceptance_length`` accepted drafts.  Attention caches (``trim`` /
    ``offset`` / ``crop``) are cut back to ``target_len``.  Returns the host
    time spent in rollback and trim calls, in ns (the replays themselves are
    asynchronous GPU work)."""
    replay_ns = 0
    fully_accepted = acceptance_length == drafted_tokens
    for entry in cache_entries:
        if hasattr(entry, "rollback"):
            if fully_accepted:
                clear_rollback_state(entry)
                continue
            t0 = time.perf_counter_ns()
            entry.rollback(acceptance_length)
            replay_ns += time.perf_counter_ns() - t0
        elif hasattr(entry, "trim"):
            offset = int(getattr(entry, "offset", 0) or 0)
            if offset > target_len:
                t0 = time.perf_counter_ns()
                entry.trim(offset - target_len)
                replay_ns += time.perf_counter_ns() - t0
        elif hasattr(entry, "offset"):
            offset = int(getattr(entry, "offset", 0) or 0)
            if offset > target_len:
                entry.offset = target_len
        elif hasattr(entry, "crop"):
            entry.crop(target_len)
    return replay_ns


def cleanup_generation_caches(target_cache: list, draft_cache: list) -> None:
    """``target_qwen_gdn.py:1057-1066``: drop transients, empty both lists."""
    for entry in target_cache:
        if hasattr(entry, "clear_transients"):
            entry.clear_transients()
    draft_cache.clear()
    target_cache.clear()
