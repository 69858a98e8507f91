"""lm_head verify epilogue on B200: argmax over the vocabulary and greedy
acceptance without materialising logits.

Mirrors the reference's verify tail (``dflash_mlx/engine/spec_epoch.py:2067-2072``):
``logits_from_hidden`` (``engine/target_qwen_gdn.py:774-778``) ->
``greedy_tokens_with_mask`` (``engine/sampling.py:47-55``) ->
``match_acceptance_length`` (``engine/acceptance.py:9-16``) -> next staged token
``posterior[acceptance]`` (``spec_epoch.py:2129``).

* :func:`lm_head_argmax_keys` -- one vocabulary shard -> one 64-bit key per
  hidden row (order-preserving logit image in the high word, ``~id`` in the
  low word; the max over shards is the global argmax with lowest-id ties).
* :func:`verify_accept` -- reduce the keys of all shards and run the
  acceptance scan on device.
* :func:`lm_head_verify` -- both, for one device or, with a process group,
  for a vocabulary split across ranks (all-gather of the keys).
* :func:`match_acceptance_length` -- the reference helper on device tensors.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._runtime import require_cuda, stream_ptr, workspace


def workspace_bytes(rows: int, dim: int, vocab: int) -> int:
    st = ctypes.c_int(0)
    n = _lib.load().dfl_lmhead_workspace_bytes(int(rows), int(dim), int(vocab), ctypes.byref(st))
    _lib.check("dfl_lmhead_workspace_bytes", st.value)
    return int(n)


def lm_head_argmax_keys(hidden: torch.Tensor, weight: torch.Tensor, *, v_begin: int = 0,
                        suppress_token_mask: Optional[torch.Tensor] = None,
                        out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Keys ``int64 [R]`` of ``argmax_v bf16(hidden @ weight.T)`` over one shard.

    ``hidden`` bf16 ``[..., D]`` (flattened to ``R`` rows), ``weight`` bf16
    ``[V_shard, D]`` holding global ids ``v_begin ..``; ``suppress_token_mask``
    is a bool/uint8 mask over the *global* vocabulary (or None).
    """
    require_cuda(hidden, "hidden")
    require_cuda(weight, "weight")
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise NotImplementedError("hidden and lm_head weight must be bfloat16")
    d = hidden.shape[-1]
    h2 = hidden.reshape(-1, d).contiguous()
    w = weight.contiguous()
    if w.shape[1] != d:
        raise ValueError(f"weight {tuple(w.shape)} does not match hidden dim {d}")
    r, v = h2.shape[0], w.shape[0]
    if v_begin < 0:
        raise ValueError(f"v_begin must be >= 0, got {v_begin}")
    if out is None:
        out = torch.empty(r, dtype=torch.int64, device=h2.device)
    else:
        require_cuda(out, "out")
        if out.dtype != torch.int64 or out.numel() != r or not out.is_contiguous() or out.device != h2.device:
            raise ValueError(f"out must be a contiguous int64 tensor of {r} keys on {h2.device}")
    sup_ptr = None
    if suppress_token_mask is not None:
        sup = suppress_token_mask.to(device=h2.device, dtype=torch.uint8).contiguous()
        if sup.numel() < v_begin + v:
            raise ValueError("suppress mask shorter than the vocabulary")
        sup_ptr = sup.data_ptr()
    with torch.cuda.device(h2.device):
        ws = workspace(h2.device, workspace_bytes(r, d, v))
        st = _lib.load().dfl_lmhead_argmax(h2.data_ptr(), w.data_ptr(), r, d, v, int(v_begin),
                                           sup_ptr, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                           stream_ptr(h2.device))
    _lib.check("dfl_lmhead_argmax", st)
    return out


def verify_accept(keys: torch.Tensor, verify_ids: Optional[torch.Tensor], *, block: int = 16):
    """Reduce shard keys ``[G, B*T]`` (or ``[B*T]``) and score the drafts.

    Returns (posterior int32 [B, T], acceptance int32 [B], next_token int32 [B],
    max_logit fp32 [B, T]).  ``verify_ids`` int32 [B, T] or None.
    """
    require_cuda(keys, "keys")
    if keys.dtype != torch.int64:
        raise ValueError(f"keys must be the int64 keys of lm_head_argmax_keys, got {keys.dtype}")
    keys = keys.reshape(-1, keys.shape[-1]) if keys.dim() > 1 else keys.reshape(1, -1)
    g, r = keys.shape
    if r % block != 0:
        raise ValueError(f"rows {r} not a multiple of the verify block {block}")
    b = r // block
    dev = keys.device
    post = torch.empty((b, block), dtype=torch.int32, device=dev)
    acc = torch.empty(b, dtype=torch.int32, device=dev)
    nxt = torch.empty(b, dtype=torch.int32, device=dev)
    mx = torch.empty((b, block), dtype=torch.float32, device=dev)
    vid = None
    if verify_ids is not None:
        vid = verify_ids.to(device=dev, dtype=torch.int32).reshape(b, block).contiguous()
    keys = keys.contiguous()
    with torch.cuda.device(dev):
        st = _lib.load().dfl_lmhead_accept(keys.data_ptr(), g, None if vid is None else vid.data_ptr(),
                                           b, block, post.data_ptr(), acc.data_ptr(), nxt.data_ptr(),
                                           mx.data_ptr(), stream_ptr(dev))
    _lib.check("dfl_lmhead_accept", st)
    return post, acc, nxt, mx


def lm_head_verify(hidden: torch.Tensor, weight: torch.Tensor, verify_ids: Optional[torch.Tensor],
                   *, suppress_token_mask: Optional[torch.Tensor] = None, v_begin: int = 0,
                   group=None, block: int = 16):
    """Posterior tokens, acceptance lengths and next staged tokens for verify blocks.

    With ``group`` (a torch.distributed process group, NCCL on GPUs) each rank
    holds a vocabulary shard starting at ``v_begin``; the per-row keys are
    all-gathered (8 bytes per row per rank) and every rank reduces them.
    """
    keys = lm_head_argmax_keys(hidden, weight, v_begin=v_begin,
                               suppress_token_mask=suppress_token_mask)
    if group is not None:
        keys = gather_keys(keys, group)
    return verify_accept(keys, verify_ids, block=block)


# ------------------------------------------------- vocabulary split (host side)
def vocab_shard(vocab: int, rank: int, world: int):
    """``(v_begin, v_len)`` of rank ``rank``'s contiguous lm_head row range when
    ``vocab`` rows are split over ``world`` ranks (ceil-sized shards; the last
    ones may be shorter or empty)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    per = (int(vocab) + world - 1) // world
    begin = min(int(vocab), rank * per)
    return begin, min(int(vocab), begin + per) - begin


def gather_keys(keys: torch.Tensor, group) -> torch.Tensor:
    """All-gather one shard's row keys ``[R]`` into ``[world, R]`` (rank order)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    keys = keys.reshape(-1).contiguous()
    gathered = torch.empty((world, keys.numel()), dtype=keys.dtype, device=keys.device)
    dist.all_gather_into_tensor(gathered.view(-1), keys, group=group)
    return gathered


_SIGN64 = -(1 << 63)


def make_keys(values: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
    """The kernels' 64-bit row key, as int64 bits: high word an order-preserving
    image of the fp32 ``values``, low word ``0xFFFFFFFF - ids``.  The unsigned
    maximum of keys is the largest value with ties to the lowest id (-0 is
    folded into +0 so that equal values tie)."""
    v = values.to(torch.float32) + 0.0
    u = v.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    ordered = torch.where(u >= (1 << 31), (~u) & 0xFFFFFFFF, u | (1 << 31))
    low = 0xFFFFFFFF - (ids.to(torch.int64) & 0xFFFFFFFF)
    # (ordered << 32) as unsigned bits, built without signed overflow
    return (((ordered - (1 << 31)) << 32) | low) ^ _SIGN64


def reduce_keys(keys: torch.Tensor) -> torch.Tensor:
    """Unsigned maximum over the leading (shard) axis of int64-held keys."""
    return (keys ^ _SIGN64).amax(dim=0) ^ _SIGN64


def decode_keys(keys: torch.Tensor):
    """``(values fp32, ids int32)`` of row keys (inverse of :func:`make_keys`)."""
    hi = (keys >> 32) & 0xFFFFFFFF
    u = torch.where(hi >= (1 << 31), hi & 0x7FFFFFFF, (~hi) & 0xFFFFFFFF)
    values = (u - ((u >= (1 << 31)).to(torch.int64) << 32)).to(torch.int32).view(torch.float32)
    ids = (0xFFFFFFFF - (keys & 0xFFFFFFFF)).to(torch.int32)
    return values, ids


def match_acceptance_length(drafted_tokens: torch.Tensor, posterior_tokens: torch.Tensor) -> torch.Tensor:
    """``engine/acceptance.py:9-16`` on device: length of the common prefix.

    Accepts ``[L]`` (returns a 0-d int32 tensor) or ``[B, L]`` (returns ``[B]``).
    """
    require_cuda(posterior_tokens, "posterior_tokens")
    single = drafted_tokens.dim() <= 1
    d = drafted_tokens.to(device=posterior_tokens.device, dtype=torch.int32).reshape(
        1 if single else drafted_tokens.shape[0], -1).contiguous()
    p = posterior_tokens.to(dtype=torch.int32).reshape(d.shape).contiguous()
    b, l = d.shape
    out = torch.empty(b, dtype=torch.int32, device=p.device)
    with torch.cuda.device(p.device):
        st = _lib.load().dfl_match_acceptance(d.data_ptr(), p.data_ptr(), b, l, out.data_ptr(),
                                              stream_ptr(p.device))
    _lib.check("dfl_match_acceptance", st)
    return out[0] if single else out
