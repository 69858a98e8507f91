"""GPU parity of the int4 g64 verify qmm against the CPU oracle.

Mirrors the reference's harness ``tests/test_verify_qmm_parity.py``:
real MLP shapes (``:16-21``), 30 seeded random shapes with
M in {1,4,8,12,15,16}, K = 64*[2,40), N = 8*[1,64) (``:32-42``), inputs
N(0,1)/sqrt(K) quantised to 4 bits (``:44-53``), and its metric
max_abs / (max|ref| + 1e-3) (``:68-70``).  On top
(seed 0), M up to 32, K/N tails, and bitwise determinism of the split-K
reduction.

Tolerances: elementwise |y - ref| <= 1e-2 + 2e-2 |ref| (bf16 out, fp32
accumulate), and for the reference-style inputs max_abs <= 8e-3 and
max_rel <= 2e-2 as in the reference.
"""

from __future__ import annotations

import zlib
import numpy as np
import pytest

from conftest import bf16_to_np_bits, to_dev_bf16, to_dev_u32
from oracle import bf16 as obf16
from oracle import qmm as oqmm

pytestmark = pytest.mark.gpu

ATOL = 1e-2
RTOL = 2e-2


def _run(pkg, dev, x, w_q, s, b):
    y = pkg.verify_matmul(to_dev_bf16(x, dev), to_dev_u32(w_q, dev), to_dev_bf16(s, dev),
                          to_dev_bf16(b, dev))
    return bf16_to_np_bits(y)


def _assert_close(y_bits, ref_bits, what=""):
    y = obf16.to_f32(y_bits).astype(np.float64)
    r = obf16.to_f32(ref_bits).astype(np.float64)
    err = np.abs(y - r)
    bad = err > ATOL + RTOL * np.abs(r)
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} outside tolerance, "
                           f"max err {err.max():.4g}")


def test_config0_dense_16x4096x4096(pkg, dev):
    rng = np.random.default_rng(0)
    w_q, s, b = oqmm.synth_weights(rng, 4096, 4096)
    x = oqmm.synth_x(rng, 16, 4096)
    y = _run(pkg, dev, x, w_q, s, b)
    _assert_close(y, oqmm.qmm(x, w_q, s, b), "config0")


REAL_SHAPES = [
    ("gate_proj", 16, 5120, 17408),
    ("down_proj", 16, 17408, 5120),
    ("q_proj", 16, 5120, 6144),
    ("k_proj", 16, 5120, 1024),
    ("o_proj", 16, 6144, 5120),
]


# tests/test_verify_qmm_parity.py:23-27 (the reference's M = 4 verify shapes)
REAL_M4_SHAPES = [
    ("gate_proj_m4", 4, 5120, 17408),
    ("down_proj_m4", 4, 17408, 5120),
]


@pytest.mark.parametrize("name,M,K,N", REAL_M4_SHAPES)
def test_real_shapes_m4_reference_harness(pkg, dev, name, M, K, N):
    x, w_q, s, b = _ref_style_case(name, M, K, N)
    y = _run(pkg, dev, x, w_q, s, b)
    max_abs, max_rel = oqmm.max_abs_rel(y, oqmm.qmm(x, w_q, s, b, accum=np.float32))
    assert y.shape == (M, N)
    assert max_abs <= 8e-3 and max_rel <= 2e-2, (name, max_abs, max_rel)


@pytest.mark.parametrize("name,M,K,N", REAL_SHAPES)
def test_real_shapes_baseline_distribution(pkg, dev, name, M, K, N):
    rng = np.random.default_rng(zlib.crc32(name.encode()) & 0xFFFF)
    w_q, s, b = oqmm.synth_weights(rng, N, K)
    x = oqmm.synth_x(rng, M, K)
    y = _run(pkg, dev, x, w_q, s, b)
    _assert_close(y, oqmm.qmm(x, w_q, s, b, accum=np.float32), name)


def _ref_style_case(name, M, K, N):
    # tests/test_verify_qmm_parity.py:44-53: x, w ~ N(0,1)/sqrt(K), then quantise
    rng = np.random.default_rng(zlib.crc32(f"{name}-{M}-{K}-{N}-64".encode()) & 0xFFFF)
    scale = 1.0 / np.sqrt(max(K, 1))
    x = obf16.from_f32((rng.standard_normal((M, K)) * scale).astype(np.float32))
    w = obf16.round_f32((rng.standard_normal((N, K)) * scale).astype(np.float32))
    w_q, s, b = oqmm.affine_quantize(w)
    return x, w_q, s, b


def _gen_random_shapes(n=30, seed=0xDF1A):
    rng = np.random.default_rng(seed)
    shapes = []
    m_levels = [1, 4, 8, 12, 15, 16]
    for i in range(n):
        m = m_levels[i % len(m_levels)]
        k = int(rng.integers(2, 40)) * 64
        nn = int(rng.integers(1, 64)) * 8
        shapes.append((f"rnd{i:02d}", m, k, nn))
    return shapes


@pytest.mark.parametrize("name,M,K,N", _gen_random_shapes(30))
def test_random_shapes_reference_harness(pkg, dev, name, M, K, N):
    x, w_q, s, b = _ref_style_case(name, M, K, N)
    y = _run(pkg, dev, x, w_q, s, b)
    ref = oqmm.qmm(x, w_q, s, b)
    max_abs, max_rel = oqmm.max_abs_rel(y, ref)
    assert max_abs <= 8e-3, f"{name} M={M} K={K} N={N} abs={max_abs:.4g}"
    assert max_rel <= 2e-2, f"{name} M={M} K={K} N={N} rel={max_rel:.4g}"
    _assert_close(y, ref, name)


@pytest.mark.parametrize("name,M,K,N", [
    ("gate_proj_m16", 16, 5120, 17408),
    ("down_proj_m16", 16, 17408, 5120),
    ("gate_proj_m4", 4, 5120, 17408),
])
def test_real_mlp_shapes_reference_harness(pkg, dev, name, M, K, N):
    x, w_q, s, b = _ref_style_case(name, M, K, N)
    y = _run(pkg, dev, x, w_q, s, b)
    ref = oqmm.qmm(x, w_q, s, b, accum=np.float32)
    max_abs, max_rel = oqmm.max_abs_rel(y, ref)
    assert max_abs <= 8e-3 and max_rel <= 2e-2, (name, max_abs, max_rel)


@pytest.mark.parametrize("M,K,N", [
    (32, 4096, 1024),    # MT=32 tile
    (17, 1600, 384),     # MT=32 with ragged M, K % 512 != 0 (plain-load scales)
    (16, 640, 200),      # ragged N, K tail inside one unit
    (1, 64, 8),          # smallest K
    (3, 8192, 136),      # long K, many stream-K segments per tile
    (16, 512, 128 * 300),  # many tiles, one unit per tile (no split)
    # several units per CTA where every unit (K = 512) or every fifth unit
    # (K = 2560) starts a new scale/bias chunk: the producer runs far ahead
    # of the dequant warps and must never wait on the MMAs
    (16, 512, 128 * 740),
    (16, 2560, 128 * 160),
    (32, 512, 128 * 600),
])
def test_edge_shapes(pkg, dev, M, K, N):
    rng = np.random.default_rng(M * 131 + K * 7 + N)
    w_q, s, b = oqmm.synth_weights(rng, N, K)
    x = oqmm.synth_x(rng, M, K)
    y = _run(pkg, dev, x, w_q, s, b)
    _assert_close(y, oqmm.qmm(x, w_q, s, b), f"{M}x{K}x{N}")


def test_rows_beyond_32_are_chunked(pkg, dev):
    rng = np.random.default_rng(7)
    w_q, s, b = oqmm.synth_weights(rng, 512, 1024)
    x = oqmm.synth_x(rng, 80, 1024)
    y = _run(pkg, dev, x, w_q, s, b)
    _assert_close(y, oqmm.qmm(x, w_q, s, b), "m80")


def test_deterministic_and_workspace_reusable(pkg, dev):
    rng = np.random.default_rng(11)
    w_q, s, b = oqmm.synth_weights(rng, 1024, 6144)
    x = oqmm.synth_x(rng, 16, 6144)
    y1 = _run(pkg, dev, x, w_q, s, b)
    y2 = _run(pkg, dev, x, w_q, s, b)
    assert np.array_equal(y1, y2)
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0


def test_dequant_is_exact(pkg, dev):
    # one-hot activations select single dequantised weights: y[m, n] = w[n, k_m]
    rng = np.random.default_rng(3)
    k, n = 1024, 256
    w_q, s, b = oqmm.synth_weights(rng, n, k)
    cols = rng.choice(k, size=16, replace=False)
    xf = np.zeros((16, k), dtype=np.float32)
    xf[np.arange(16), cols] = 1.0
    x = obf16.from_f32(xf)
    y = _run(pkg, dev, x, w_q, s, b)
    w = oqmm.dequantize(w_q, s, b)
    assert np.array_equal(obf16.to_f32(y), w[:, cols].T)


def test_verify_linear_matches_direct_call(pkg, dev):
    """VerifyQuantizedLinear(x) is bit-identical to verify_matmul on the same
    weights (reference tests/test_verify_linear_parity.py:53-63), for M = 16
    and for other row counts (which the reference sends to stock qmm)."""
    import torch

    rng = np.random.default_rng(21)
    w_q, s, b = oqmm.synth_weights(rng, 1024, 512)
    ql = pkg.QuantizedLinear(to_dev_u32(w_q, dev), to_dev_bf16(s, dev), to_dev_bf16(b, dev))
    verify = pkg.VerifyQuantizedLinear.from_quantized(ql)
    for m in (16, 1, 8, 32, 40):
        x = to_dev_bf16(oqmm.synth_x(rng, m, 512), dev)
        direct = pkg.verify_matmul(x, ql.weight, ql.scales, ql.biases, transpose=True,
                                   group_size=64, bits=4)
        assert torch.equal(verify(x), direct)
        assert torch.equal(ql(x), direct)


def test_workspace_shared_with_lm_head_is_left_zero(pkg, dev):
    """The qmm and the lm_head share one workspace per stream.  Every kernel
    must leave it all zero: an lm_head call over many rows followed by a
    split-K qmm on the same stream gives the oracle's result, and the buffer
    is zero after each call."""
    import torch

    from dflash_mlx_b200 import _runtime

    rng = np.random.default_rng(77)
    h = obf16.from_f32(rng.standard_normal((2048, 256)).astype(np.float32))
    w = obf16.from_f32((rng.standard_normal((3000, 256)) * 0.02).astype(np.float32))
    pkg.lm_head_argmax_keys(to_dev_bf16(h, dev), to_dev_bf16(w, dev))
    torch.cuda.synchronize(dev)
    ws = _runtime.workspace(dev, 1)
    assert int(ws.count_nonzero()) == 0
    w_q, s, b = oqmm.synth_weights(rng, 6144, 5120)
    x = oqmm.synth_x(rng, 16, 5120)
    y = _run(pkg, dev, x, w_q, s, b)
    _assert_close(y, oqmm.qmm(x, w_q, s, b, accum=np.float32), "qmm after lm_head")
    torch.cuda.synchronize(dev)
    assert int(_runtime.workspace(dev, 1).count_nonzero()) == 0
