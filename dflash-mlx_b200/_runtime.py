"""Torch-side plumbing for the C ABI: stream handles, zero-initialised
workspaces (one per device and stream), tensor checks.

PyTorch is used here only for device memory and streams; every kernel
launch goes through libdflash_b200.so.
"""

from __future__ import annotations

import threading

import torch

_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def stream_ptr(device: torch.device) -> int:
    """Raw cudaStream_t of torch's current stream on ``device``."""
    return int(torch.cuda.current_stream(device).cuda_stream)


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A zero-filled uint8 scratch buffer of at least ``nbytes`` for the
    current stream of ``device``.

    Kernels that use it leave it zeroed again, so one buffer serves every
    call issued on that stream in order.  Different streams get different
    buffers, because calls on different streams may overlap.
    """
    dev = torch.device(device)
    key = (dev.index if dev.index is not None else torch.cuda.current_device(),
           stream_ptr(dev))
    with _ws_lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(int(nbytes), 1 << 20)
            if buf is not None:
                size = max(size, 2 * buf.numel())
            buf = torch.zeros(size, dtype=torch.uint8, device=dev)
            _workspaces[key] = buf
        return buf


def reset_workspaces() -> int:
    """Zero every cached workspace again; returns how many were cleared.

    Kernels leave their workspace zero when they finish normally.  A kernel
    that gave up on a bounded wait (the device error word is set) can leave
    partial sums behind, so after a reported device error every buffer is
    cleared before the next call uses it.
    """
    with _ws_lock:
        bufs = list(_workspaces.values())
        for buf in bufs:
            buf.zero_()
        for dev in {buf.device for buf in bufs if buf.is_cuda}:
            torch.cuda.synchronize(dev)
    return len(bufs)


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (dflash-b200 has no CPU path)")


def as_u32_bits(w: torch.Tensor) -> torch.Tensor:
    """Packed weights as a contiguous 32-bit tensor (int32 or uint32 storage)."""
    if w.dtype not in (torch.int32, torch.uint32):
        raise TypeError(f"packed weights must be uint32/int32, got {w.dtype}")
    return w.contiguous()
