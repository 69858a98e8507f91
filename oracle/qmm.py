"""Oracle for the M=16 int4 verify qmm (dense) -- TEST INFRASTRUCTURE ONLY.

Restates the reference's quantized matmul ``y = x @ W.T`` with MLX's affine
layout, as every verify kernel reads it:

* ``w_q`` is uint32 ``[N, K/8]``; nibble ``ki`` of word ``pack`` sits at bits
  ``4*ki .. 4*ki+3`` and holds column ``k = 8*pack + ki`` (low nibble first),
  ``dflash_mlx/verify_qmm.py:243-250`` (also ``:97-115`` for M=4).
* ``scales`` / ``biases`` are ``[N, K/group_size]`` in the activation dtype;
  group ``k // group_size``.
* Dequantisation is ``float(nib) * s + b`` in fp32, then rounded to the
  activation dtype before the MMA (``verify_qmm.py:249``:
  ``T(float(nib) * s + b)``).  Accumulation is fp32
  (``simdgroup_matrix<float>`` accumulators, ``verify_qmm.py:228-232``) and
  the output is rounded to the activation dtype (``verify_qmm.py:290``).

bf16 tensors are passed as uint16 bit patterns (see ``oracle/bf16.py``).
"""

from __future__ import annotations

import numpy as np

from . import bf16

GROUP_SIZE = 64
BITS = 4


def pack_nibbles(q: np.ndarray) -> np.ndarray:
    """uint8 nibbles ``[N, K]`` (values 0..15) -> uint32 ``[N, K/8]``, low nibble first."""
    q = np.asarray(q, dtype=np.uint32)
    n, k = q.shape
    assert k % 8 == 0
    q = q.reshape(n, k // 8, 8)
    out = np.zeros((n, k // 8), dtype=np.uint32)
    for ki in range(8):
        out |= (q[:, :, ki] & np.uint32(0xF)) << np.uint32(4 * ki)
    return out


def unpack_nibbles(w_q: np.ndarray) -> np.ndarray:
    """uint32 ``[N, K/8]`` -> uint8 nibbles ``[N, K]`` (inverse of :func:`pack_nibbles`)."""
    w_q = np.asarray(w_q, dtype=np.uint32)
    n, kp = w_q.shape
    out = np.empty((n, kp, 8), dtype=np.uint8)
    for ki in range(8):
        out[:, :, ki] = (w_q >> np.uint32(4 * ki)) & np.uint32(0xF)
    return out.reshape(n, kp * 8)


def pair_pack(w_q: np.ndarray) -> np.ndarray:
    """MLX-packed uint32 ``[N, K/8]`` -> the kernel's pair-packed order.

    Not a reference format: a load-time layout of this build in which nibble
    ``j`` of word ``p`` holds column ``8p + 2j`` and nibble ``4 + j`` column
    ``8p + 2j + 1`` (j = 0..3), so that the kernel's mask/shift dequantiser
    emits columns in natural order.  Used only to check the repack kernel.
    """
    nib = unpack_nibbles(w_q)
    n, k = nib.shape
    g = nib.reshape(n, k // 8, 8)
    order = np.array([0, 2, 4, 6, 1, 3, 5, 7])  # nibble slot -> column within 8
    return pack_nibbles(g[:, :, order].reshape(n, k))


def _to_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16.to_f32(bits)
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)


def _round(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16.round_f32(x)
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def _from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16.from_f32(x)
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def dequantize(w_q: np.ndarray, scales: np.ndarray, biases: np.ndarray,
               group_size: int = GROUP_SIZE, dtype: str = "bf16") -> np.ndarray:
    """Dequantised weights ``float(nib) * s + b`` rounded to the activation
    dtype (``verify_qmm.py:249``), as float32 values.  ``scales`` / ``biases``
    are bit patterns of that dtype ("bf16" or "f16")."""
    nib = unpack_nibbles(w_q).astype(np.float32)
    n, k = nib.shape
    s = np.repeat(_to_f32(scales, dtype), group_size, axis=1)[:, :k]
    b = np.repeat(_to_f32(biases, dtype), group_size, axis=1)[:, :k]
    return _round(nib * s + b, dtype)


def qmm(x: np.ndarray, w_q: np.ndarray, scales: np.ndarray, biases: np.ndarray,
        group_size: int = GROUP_SIZE, accum=np.float64, dtype: str = "bf16") -> np.ndarray:
    """``y = x @ dequant(W).T`` -> bit patterns ``[M, N]`` of ``dtype``.

    ``x`` holds bits of ``dtype`` ("bf16" or "f16") ``[M, K]``.  ``accum``
    selects the accumulation dtype: float64 for golden values, float32 for the
    timed CPU restatement.
    """
    xf = _to_f32(x, dtype).astype(accum)
    n = w_q.shape[0]
    y = np.empty((xf.shape[0], n), dtype=np.float32)
    step = 2048
    for r0 in range(0, n, step):
        w = dequantize(w_q[r0:r0 + step], scales[r0:r0 + step], biases[r0:r0 + step],
                       group_size, dtype).astype(accum)
        y[:, r0:r0 + step] = (xf @ w.T).astype(np.float32)
    return _from_f32(y, dtype)


def qmm_f32(x: np.ndarray, w_q: np.ndarray, scales: np.ndarray, biases: np.ndarray,
            group_size: int = GROUP_SIZE) -> np.ndarray:
    """Unrounded float32 result of :func:`qmm` (float64 accumulation)."""
    w = dequantize(w_q, scales, biases, group_size).astype(np.float64)
    return (bf16.to_f32(x).astype(np.float64) @ w.T).astype(np.float32)


def affine_quantize(w: np.ndarray, group_size: int = GROUP_SIZE, dtype: str = "bf16"):
    """Min/max affine 4-bit quantiser used only to build test inputs.

    The reference's parity harness quantises random fp weights with
    ``mx.quantize`` before calling the kernel
    (``tests/test_verify_qmm_parity.py:29-30,51-53``).  This is a plain
    restatement of the published affine scheme (scale = range / 15,
    bias = group minimum, q = round((w - bias) / scale)); the kernels under
    test only see its output, so the exact tie rules of MLX's quantiser do
    not affect parity.  Returns (w_q uint32, scales bits, biases bits) with
    scales/biases in ``dtype`` ("bf16" or "f16").
    """
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % group_size == 0
    g = w.reshape(n, k // group_size, group_size)
    wmin = g.min(axis=2)
    wmax = g.max(axis=2)
    scale = np.maximum((wmax - wmin) / 15.0, 1e-7).astype(np.float32)
    s_bits = _from_f32(scale, dtype)
    b_bits = _from_f32(wmin, dtype)
    s = _to_f32(s_bits, dtype)[:, :, None]
    b = _to_f32(b_bits, dtype)[:, :, None]
    q = np.clip(np.rint((g - b) / s), 0, 15).astype(np.uint8).reshape(n, k)
    return pack_nibbles(q), s_bits, b_bits


def synth_weights(rng: np.random.Generator, n: int, k: int, group_size: int = GROUP_SIZE,
                  dtype: str = "bf16"):
    """Synthetic weight distribution of the benchmark's dense qmm.

    q ~ U{0..15}; scales bf16 ~ U(0.004, 0.02) per (row, group);
    biases = -8*scale + N(0, 0.1*scale).  Returns (w_q, scales, biases).
    """
    q = rng.integers(0, 16, size=(n, k), dtype=np.uint8)
    g = k // group_size
    s = rng.uniform(0.004, 0.02, size=(n, g)).astype(np.float32)
    b = (-8.0 * s + rng.standard_normal((n, g)).astype(np.float32) * 0.1 * s).astype(np.float32)
    return pack_nibbles(q), _from_f32(s, dtype), _from_f32(b, dtype)


def synth_x(rng: np.random.Generator, m: int, k: int, dtype: str = "bf16") -> np.ndarray:
    """Activations ~ N(0, 1) as bit patterns of ``dtype``."""
    return _from_f32(rng.standard_normal((m, k)).astype(np.float32), dtype)


def max_abs_rel(y: np.ndarray, ref: np.ndarray, dtype: str = "bf16"):
    """The reference harness metric (``tests/test_verify_qmm_parity.py:68-70``)."""
    a = _to_f32(y, dtype).astype(np.float64)
    r = _to_f32(ref, dtype).astype(np.float64)
    max_abs = float(np.max(np.abs(a - r))) if a.size else 0.0
    max_rel = max_abs / (float(np.max(np.abs(r))) + 1e-3) if r.size else 0.0
    return max_abs, max_rel
