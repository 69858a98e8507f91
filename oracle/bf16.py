"""bfloat16 helpers in plain NumPy (bit patterns stored as uint16).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).
Rounding is round-to-nearest-even, the rounding MLX and CUDA use when an
fp32 value is cast to bf16 (``static_cast<T>`` in
``dflash_mlx/verify_qmm.py:249``).
"""

from __future__ import annotations

import numpy as np


def to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    b = np.asarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def from_f32(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bit patterns, round-to-nearest-even.

    NaNs are kept quiet NaNs; infinities stay infinities.
    """
    f = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    bias = ((u >> np.uint64(16)) & np.uint64(1)) + np.uint64(0x7FFF)
    r = ((u + bias) >> np.uint64(16)).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def round_f32(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 and return them as float32."""
    return to_f32(from_f32(x))
